"""Torch-facing ops over the C ABI. Every call launches on torch's current CUDA stream, allocates
only its output (and nothing when `out=` is given), and raises on any error status.

DiT (engine/fused.py:293-298):
    dit_qkv_prologue  — the `qkv` producer (engine/fused.py:117-180) without the per-batch ctx copy
    dit_attention     — the attention over [latent | ctx] keys, y in (B, L, H, hd)
    sdpa              — drop-in for F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    dit_gate          — the `gate` consumer (engine/fused.py:182-190): y · sigmoid(gate), optional FP8 out
    dit_attention_layer — the whole block (producer, attention, gate) in two launches, bf16
Qwen3 talker (qwen3/kernels.py:622-624):
    decode_attention  — one layer's decode step with the reference kernel's argument list
    decode_attention_block — the layer's rms_gemv(qkv) -> attention -> gemv(o) in one launch
    prefill_attention — the prompt's causal attention (qwen3/fast.py:251-263), tensor cores
"""

from __future__ import annotations

import contextlib
import ctypes
import os

import torch

from . import _lib
from ._lib import SK_BF16, SK_E4M3, SK_F32, check, lib


_NVTX = os.environ.get("SOKUTOU_B200_NVTX") == "1"


def _nvtx(name: str):
    """An NVTX range per op launch (SOKUTOU_B200_NVTX=1) so a profiler can select one op's kernels
    (ncu --nvtx --nvtx-include "sk_decode_attention/"); a no-op otherwise."""
    return torch.cuda.nvtx.range(name) if _NVTX else contextlib.nullcontext()


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return SK_BF16
    if dt == torch.float32:
        return SK_F32
    raise TypeError(f"unsupported dtype {dt}: bfloat16 or float32")


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda_contig(name: str, t: torch.Tensor) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.is_contiguous(), f"{name} must be contiguous")


def device_error(reset: bool = True) -> int:
    """The device error word of the current device (0 = none); synchronises the device."""
    code = ctypes.c_int(0)
    with _nvtx("sk_device_error"):
        check(lib().sk_device_error(ctypes.byref(code), int(reset)), "sk_device_error")
    return code.value


# ---- DiT ----------------------------------------------------------------------------------------

def dit_qkv_prologue(o4: torch.Tensor, qk_w: torch.Tensor, freqs: torch.Tensor, B: int, L: int, H: int, hd: int,
                     eps: float, out: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None):
    """q, k_lat, v_lat (each (B, H, L, hd), o4's dtype) from o4 (B*L, 4*H*hd) = [q | k | v | gate].

    qk_w: float32 (2, H, hd) q_norm/k_norm weights; freqs: float32 (>= L, hd/2, 2) RoPE (cos, sin).
    """
    for n, t in (("o4", o4), ("qk_w", qk_w), ("freqs", freqs)):
        _cuda_contig(n, t)
    _need(o4.shape == (B * L, 4 * H * hd), f"o4 must be ({B * L}, {4 * H * hd}), got {tuple(o4.shape)}")
    _need(qk_w.dtype == torch.float32 and qk_w.numel() == 2 * H * hd, "qk_w must be float32 (2, H, hd)")
    _need(freqs.dtype == torch.float32 and freqs.shape[0] >= L and freqs.shape[1:] == (hd // 2, 2),
          "freqs must be float32 (>= L, hd/2, 2)")
    if out is None:
        out = tuple(torch.empty((B, H, L, hd), device=o4.device, dtype=o4.dtype) for _ in range(3))
    q, k, v = out
    for n, t in (("q", q), ("k_lat", k), ("v_lat", v)):
        _cuda_contig(n, t)
        _need(t.shape == (B, H, L, hd) and t.dtype == o4.dtype, f"{n} must be ({B}, {H}, {L}, {hd}) {o4.dtype}")
    with _nvtx("sk_dit_qkv_prologue"):
        check(lib().sk_dit_qkv_prologue(_ptr(o4), _ptr(qk_w), _ptr(freqs), _ptr(q), _ptr(k), _ptr(v), B, L, H, hd,
                                        float(eps), _dtype_code(o4.dtype), _stream()), "sk_dit_qkv_prologue")
    return q, k, v


def dit_attention(q: torch.Tensor, k_lat: torch.Tensor, v_lat: torch.Tensor, k_ctx: torch.Tensor | None = None,
                  v_ctx: torch.Tensor | None = None, bias: torch.Tensor | None = None, scale: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q·kᵀ·scale + bias)·v over keys [latent | ctx]; returns y (B, L, H, hd).

    q: (B, H, L, hd); k_lat/v_lat: (B, H, Lk, hd); k_ctx/v_ctx: (S, H, hd) shared by every batch row,
    or (B, S, H, hd) per row; bias: additive (K,) shared or (B, K) / (B, 1, 1, K) per row, q's dtype.
    bfloat16 runs on the tensor cores, float32 on the fp32 CUDA-core kernel.
    """
    _cuda_contig("q", q)
    B, H, L, hd = q.shape
    dt = q.dtype
    _cuda_contig("k_lat", k_lat)
    _cuda_contig("v_lat", v_lat)
    _need(k_lat.shape == v_lat.shape and k_lat.shape[:2] == (B, H) and k_lat.shape[3] == hd,
          "k_lat/v_lat must be (B, H, Lk, hd)")
    Lk = k_lat.shape[2]
    S, ctx_bs = 0, 0
    if k_ctx is not None:
        _cuda_contig("k_ctx", k_ctx)
        _cuda_contig("v_ctx", v_ctx)
        _need(k_ctx.shape == v_ctx.shape, "k_ctx and v_ctx differ in shape")
        if k_ctx.dim() == 3:
            S = k_ctx.shape[0]
            _need(k_ctx.shape[1:] == (H, hd), "k_ctx must be (S, H, hd) or (B, S, H, hd)")
        else:
            _need(k_ctx.dim() == 4 and k_ctx.shape[0] == B and k_ctx.shape[2:] == (H, hd),
                  "k_ctx must be (S, H, hd) or (B, S, H, hd)")
            S, ctx_bs = k_ctx.shape[1], k_ctx.stride(0)
    K = Lk + S
    bias_bs = 0
    if bias is not None:
        _cuda_contig("bias", bias)
        _need(bias.dtype == dt, "bias must have q's dtype")
        _need(bias.numel() in (K, B * K), f"bias must hold K={K} or B*K values")
        bias_bs = K if bias.numel() == B * K else 0
    for t in (k_lat, v_lat, k_ctx, v_ctx):
        _need(t is None or t.dtype == dt, "q, k, v must share one dtype")
    if out is None:
        out = torch.empty((B, L, H, hd), device=q.device, dtype=dt)
    _cuda_contig("out", out)
    _need(out.shape == (B, L, H, hd) and out.dtype == dt, "out must be (B, L, H, hd) in q's dtype")
    with _nvtx("sk_dit_attention"):
        check(lib().sk_dit_attention(_ptr(q), _ptr(k_lat), _ptr(v_lat), _ptr(k_ctx), _ptr(v_ctx), _ptr(bias), _ptr(out),
                                     B, H, L, Lk, S, hd, ctx_bs, bias_bs, _dtype_code(dt), float(scale or 0.0), _stream()),
              "sk_dit_attention")
    return out


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Drop-in for `F.scaled_dot_product_attention(q, k, v, attn_mask=bias)` at engine/fused.py:295.

    q (B, H, L, hd), k/v (B, H, K, hd), attn_mask additive (B or 1, 1, 1, K) or bool (True = keep).
    Returns (B, H, L, hd) whose memory is (B, L, H, hd)-contiguous, so `y.transpose(1, 2)` is
    contiguous as the `gate` kernel reads it (engine/fused.py:296-298).
    """
    bias = None
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            bias = torch.zeros(attn_mask.shape, device=q.device, dtype=q.dtype).masked_fill_(~attn_mask, float("-inf"))
        else:
            bias = attn_mask
        bias = bias.reshape(-1, k.shape[2]).contiguous()
    y = dit_attention(q, k, v, None, None, bias)
    return y.transpose(1, 2)


def dit_attention_layer(o4: torch.Tensor, qk_w: torch.Tensor, freqs: torch.Tensor, B: int, L: int, H: int, hd: int,
                        eps: float, k_ctx: torch.Tensor | None = None, v_ctx: torch.Tensor | None = None,
                        bias: torch.Tensor | None = None, scale: float | None = None,
                        out: torch.Tensor | None = None,
                        qkv_bufs: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """One DiT layer's attention block (engine/fused.py:293-298): the `qkv` producer, the attention over
    [latent | ctx] keys and the `gate` consumer, in two launches (the gate read from o4 by the attention
    epilogue). o4 (B*L, 4*H*hd) bf16; qk_w float32 (2, H, hd); freqs float32 (>= L, hd/2, 2);
    k_ctx/v_ctx (S, H, hd) shared or (B, S, H, hd); bias as for dit_attention; qkv_bufs: (B, H, L, hd)
    bf16 scratch for q, k, v (allocated here when not given). Returns (B*L, H*hd) bf16 =
    y · sigmoid(gate)."""
    for n, t in (("o4", o4), ("qk_w", qk_w), ("freqs", freqs)):
        _cuda_contig(n, t)
    _need(o4.dtype == torch.bfloat16, "the fused layer runs in bfloat16 (use the separate ops for float32)")
    D = H * hd
    _need(o4.shape == (B * L, 4 * D), f"o4 must be ({B * L}, {4 * D}), got {tuple(o4.shape)}")
    _need(qk_w.dtype == torch.float32 and qk_w.numel() == 2 * D, "qk_w must be float32 (2, H, hd)")
    _need(freqs.dtype == torch.float32 and freqs.shape[0] >= L and freqs.shape[1:] == (hd // 2, 2),
          "freqs must be float32 (>= L, hd/2, 2)")
    S, ctx_bs = 0, 0
    if k_ctx is not None:
        _cuda_contig("k_ctx", k_ctx)
        _cuda_contig("v_ctx", v_ctx)
        _need(k_ctx.shape == v_ctx.shape and k_ctx.dtype == o4.dtype and v_ctx.dtype == o4.dtype,
              "k_ctx and v_ctx must match in shape and be bfloat16")
        if k_ctx.dim() == 3:
            S = k_ctx.shape[0]
            _need(k_ctx.shape[1:] == (H, hd), "k_ctx must be (S, H, hd) or (B, S, H, hd)")
        else:
            _need(k_ctx.dim() == 4 and k_ctx.shape[0] == B and k_ctx.shape[2:] == (H, hd),
                  "k_ctx must be (S, H, hd) or (B, S, H, hd)")
            S, ctx_bs = k_ctx.shape[1], k_ctx.stride(0)
    K = L + S
    bias_bs = 0
    if bias is not None:
        _cuda_contig("bias", bias)
        _need(bias.dtype == o4.dtype, "bias must be bfloat16")
        _need(bias.numel() in (K, B * K), f"bias must hold K={K} or B*K values")
        bias_bs = K if bias.numel() == B * K else 0
    if out is None:
        out = torch.empty((B * L, D), device=o4.device, dtype=o4.dtype)
    _cuda_contig("out", out)
    _need(out.numel() == B * L * D and out.dtype == o4.dtype, f"out must hold {B * L}x{D} bfloat16")
    if qkv_bufs is None:
        qkv_bufs = tuple(torch.empty((B, H, L, hd), device=o4.device, dtype=o4.dtype) for _ in range(3))
    for n, t in zip(("q_buf", "k_buf", "v_buf"), qkv_bufs):
        _cuda_contig(n, t)
        _need(t.shape == (B, H, L, hd) and t.dtype == o4.dtype, f"{n} must be ({B}, {H}, {L}, {hd}) bfloat16")
    with _nvtx("sk_dit_attention_layer"):
        check(lib().sk_dit_attention_layer(_ptr(o4), _ptr(qk_w), _ptr(freqs), _ptr(k_ctx), _ptr(v_ctx), _ptr(bias),
                                           _ptr(out), _ptr(qkv_bufs[0]), _ptr(qkv_bufs[1]), _ptr(qkv_bufs[2]), B, H, L,
                                           S, hd, ctx_bs, bias_bs, float(eps), SK_BF16, float(scale or 0.0), _stream()),
              "sk_dit_attention_layer")
    return out


# ---- Qwen3 decode --------------------------------------------------------------------------------

def dit_gate(y: torch.Tensor, o4: torch.Tensor, out: torch.Tensor | None = None, fp8_scale: float | None = None
             ) -> torch.Tensor:
    """out = y · sigmoid(gate) with gate = o4[:, 3D:4D]; y (B, L, H, hd) or (B·L, D), o4 (B·L, 4·D).

    Returns (B·L, D) in y's dtype, or raw FP8 e4m3 bytes (torch.uint8) of value·fp8_scale when
    fp8_scale is given (the reference's FP8 GEMM input, engine/fused.py:52-76).
    """
    _cuda_contig("y", y)
    _cuda_contig("o4", o4)
    _need(y.dtype == o4.dtype, "y and o4 must share a dtype")
    rows = o4.shape[0]
    D = o4.shape[1] // 4
    _need(o4.dim() == 2 and o4.shape[1] == 4 * D and y.numel() == rows * D, "o4 must be (rows, 4*D) and y hold rows*D")
    code = _dtype_code(y.dtype)
    out_code = code if fp8_scale is None else SK_E4M3
    odt = y.dtype if fp8_scale is None else torch.uint8
    if out is None:
        out = torch.empty((rows, D), device=y.device, dtype=odt)
    _cuda_contig("out", out)
    _need(out.dtype == odt and out.numel() == rows * D, f"out must hold {rows}x{D} {odt}")
    with _nvtx("sk_dit_gate"):
        check(lib().sk_dit_gate(_ptr(y), _ptr(o4), _ptr(out), rows, D, code, out_code,
                                float(fp8_scale if fp8_scale is not None else 1.0), _stream()), "sk_dit_gate")
    return out


def dit_linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, tile_n: int = 0) -> torch.Tensor:
    """y = x · wᵀ (F.linear without bias, engine/fused.py:262-264) on the tcgen05 GEMM, bf16 in and out,
    fp32 accumulation. x (M, K), w (N, K); returns (M, N). tile_n: the CTA tile's width (64, 128, 256;
    0 = chosen per call)."""
    _cuda_contig("x", x)
    _cuda_contig("w", w)
    _need(x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16, "dit_linear runs bf16 (fp32: use F.linear)")
    _need(x.dim() == 2 and w.dim() == 2 and x.shape[1] == w.shape[1], "x must be (M, K) and w (N, K)")
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=x.dtype)
    _cuda_contig("out", out)
    _need(out.dtype == x.dtype and out.shape == (M, N), f"out must be ({M}, {N}) bf16")
    with _nvtx("sk_dit_linear"):
        check(lib().sk_dit_linear_ex(_ptr(x), _ptr(w), _ptr(out), M, N, K, _dtype_code(x.dtype), int(tile_n),
                                     _stream()), "sk_dit_linear")
    return out


def dit_linear_fp8(x8: torch.Tensor, w8: torch.Tensor, inv_scale_x: torch.Tensor, inv_scale_w: torch.Tensor,
                   out: torch.Tensor | None = None, tile_n: int = 0) -> torch.Tensor:
    """y = (x8 · w8ᵀ) · inv_scale_x · inv_scale_w in bf16 — torch._scaled_mm(x8, w8.t(), inv_x, inv_w,
    out_dtype=bf16) of engine/fp8.py:87-89 on the tcgen05 kind::f8f6f4 GEMM. x8 (M, K) and w8 (N, K) are
    e4m3 tensors (torch.float8_e4m3fn, or their raw bytes as torch.uint8); the scales are one-element
    fp32 device tensors."""
    for name, t in (("x8", x8), ("w8", w8)):
        _cuda_contig(name, t)
        _need(t.element_size() == 1 and t.dim() == 2, f"{name} must be 2-D e4m3 (or uint8) bytes")
    for name, t in (("inv_scale_x", inv_scale_x), ("inv_scale_w", inv_scale_w)):
        _cuda_contig(name, t)
        _need(t.dtype == torch.float32 and t.numel() == 1, f"{name} must be one fp32 element")
    _need(x8.shape[1] == w8.shape[1], "x8 must be (M, K) and w8 (N, K)")
    M, K = x8.shape
    N = w8.shape[0]
    if out is None:
        out = torch.empty((M, N), device=x8.device, dtype=torch.bfloat16)
    _cuda_contig("out", out)
    _need(out.dtype == torch.bfloat16 and out.shape == (M, N), f"out must be ({M}, {N}) bf16")
    with _nvtx("sk_dit_linear_fp8"):
        check(lib().sk_dit_linear_fp8(_ptr(x8), _ptr(w8), _ptr(out), _ptr(inv_scale_x), _ptr(inv_scale_w), M, N, K,
                                      int(tile_n), _stream()), "sk_dit_linear_fp8")
    return out


def decode_workspace_bytes(max_len: int, nq: int, nkv: int, hd: int = 128, cache_dtype: torch.dtype = torch.bfloat16) -> int:
    return int(lib().sk_decode_workspace_bytes(max_len, nq, nkv, hd, _dtype_code(cache_dtype)))


def decode_workspace(max_len: int, nq: int, nkv: int, device, hd: int = 128,
                     cache_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """A zero-filled workspace for decode_attention (allocate before graph capture)."""
    n = decode_workspace_bytes(max_len, nq, nkv, hd, cache_dtype)
    return torch.zeros(max(n, 16), dtype=torch.uint8, device=device)


def decode_attention(qkv: torch.Tensor, qn: torch.Tensor, kn: torch.Tensor, eps: float, rope: torch.Tensor,
                     Kc: torch.Tensor, Vc: torch.Tensor, pos_ptr: torch.Tensor | None, pos_add: int, max_len: int,
                     nq: int, nkv: int, out: torch.Tensor, workspace: torch.Tensor | None,
                     kv_stable: bool = False) -> torch.Tensor:
    """One talker layer's decode attention with the reference kernel's arguments
    (qwen3/kernels.py:341-344): writes K/V at pos = pos_ptr[0] + pos_add and out (nq*128 fp32).

    kv_stable: the kernel launched just before on this stream writes neither the position nor this
    layer's cache, so the cache reads may overlap it (SK_DECODE_KV_STABLE)."""
    hd = Kc.shape[-1]
    for n, t in (("qkv", qkv), ("qn", qn), ("kn", kn), ("rope", rope), ("Kc", Kc), ("Vc", Vc), ("out", out)):
        _cuda_contig(n, t)
    _need(qkv.dtype == torch.float32 and qkv.numel() == (nq + 2 * nkv) * hd, "qkv must be float32 [(nq+2nkv)*hd]")
    _need(out.dtype == torch.float32 and out.numel() == nq * hd, "out must be float32 [nq*hd]")
    _need(rope.dtype == torch.float32 and rope.numel() >= max_len * hd, "rope must be float32 [max_len][hd]")
    _need(Kc.shape == Vc.shape and Kc.numel() == nkv * max_len * hd and Kc.dtype == Vc.dtype,
          "Kc/Vc must be [nkv][max_len][hd]")
    if pos_ptr is not None:
        _need(pos_ptr.is_cuda and pos_ptr.dtype == torch.int64, "pos_ptr must be a CUDA int64 tensor")
    ws_n = 0 if workspace is None else workspace.numel() * workspace.element_size()
    with _nvtx("sk_decode_attention_ex"):
        check(lib().sk_decode_attention_ex(_ptr(qkv), _ptr(qn), _ptr(kn), float(eps), _ptr(rope), _ptr(Kc), _ptr(Vc),
                                           _ptr(pos_ptr), int(pos_add), int(max_len), int(nq), int(nkv), int(hd),
                                           _ptr(out), _ptr(workspace), ws_n, _dtype_code(Kc.dtype),
                                           _lib.SK_DECODE_KV_STABLE if kv_stable else 0, _stream()),
              "sk_decode_attention")
    return out


def decode_requests(reqs: list[dict], device) -> torch.Tensor:
    """The device array of SkDecodeRequest descriptors for decode_attention_grouped, one per dict with the
    tensors qkv, qn, kn, rope, Kc, Vc, out, the optional pos_ptr (CUDA int64) and the ints/floats pos_add,
    eps. Build it before graph capture and keep the tensors alive while it is used."""
    arr = (_lib.SkDecodeRequest * len(reqs))()
    for i, r in enumerate(reqs):
        for n in ("qkv", "qn", "kn", "rope", "Kc", "Vc", "out"):
            _cuda_contig(n, r[n])
        _need(r["qkv"].dtype == torch.float32 and r["out"].dtype == torch.float32, "qkv and out must be float32")
        pp = r.get("pos_ptr")
        if pp is not None:
            _need(pp.is_cuda and pp.dtype == torch.int64, "pos_ptr must be a CUDA int64 tensor")
        arr[i] = _lib.SkDecodeRequest(_ptr(r["qkv"]), _ptr(r["qn"]), _ptr(r["kn"]), _ptr(r["rope"]), _ptr(r["Kc"]),
                                      _ptr(r["Vc"]), _ptr(pp), _ptr(r["out"]), int(r.get("pos_add", 0)),
                                      float(r["eps"]), (ctypes.c_int * 2)(0, 0))
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return host.to(device)


def decode_attention_grouped(reqs_dev: torch.Tensor, n: int, max_len: int, nq: int, nkv: int,
                             cache_dtype: torch.dtype = torch.bfloat16, kv_stable: bool = False) -> None:
    """n independent decode requests (descriptors from decode_requests) in one launch: each does exactly what
    decode_attention does with its own arguments; all share max_len, nq, nkv and the cache dtype."""
    _need(reqs_dev.is_cuda and reqs_dev.dtype == torch.uint8 and reqs_dev.numel() >= 80 * n,
          "reqs_dev must be the device descriptor array of decode_requests")
    with _nvtx("sk_decode_attention_grouped"):
        check(lib().sk_decode_attention_grouped(_ptr(reqs_dev), int(n), int(max_len), int(nq), int(nkv), 128,
                                                _dtype_code(cache_dtype),
                                                _lib.SK_DECODE_KV_STABLE if kv_stable else 0, _stream()),
              "sk_decode_attention_grouped")


def decode_block_workspace(max_len: int, nq: int, nkv: int, device, hd: int = 128) -> torch.Tensor:
    """A zero-filled workspace for decode_attention_block (allocate before graph capture)."""
    n = int(lib().sk_decode_block_workspace_bytes(max_len, nq, nkv, hd))
    return torch.zeros(max(n, 16), dtype=torch.uint8, device=device)


def decode_attention_block(h: torch.Tensor, in_norm: torch.Tensor, eps_in: float, w_qkv: torch.Tensor,
                           qn: torch.Tensor, kn: torch.Tensor, eps: float, rope: torch.Tensor, Kc: torch.Tensor,
                           Vc: torch.Tensor, pos_ptr: torch.Tensor | None, pos_add: int, max_len: int, nq: int,
                           nkv: int, w_o: torch.Tensor, workspace: torch.Tensor, kv_stable: bool = False) -> torch.Tensor:
    """One talker layer's attention block in one launch (the reference's rms_gemv(qkv) -> attn -> gemv(o),
    qwen3/kernels.py:619-624): h (fp32 [hidden]) += W_o · attn(W_qkv · RMSNorm(h) ⊙ in_norm), K/V appended
    at pos = pos_ptr[0] + pos_add. Weights bf16 or fp32 (w_qkv [(nq+2nkv)·128][hidden], w_o [hidden][nq·128]);
    caches bf16 or fp32 [nkv][max_len][128]. Returns h (updated in place)."""
    hd = Kc.shape[-1]
    hidden = h.numel()
    for n, t in (("h", h), ("in_norm", in_norm), ("w_qkv", w_qkv), ("qn", qn), ("kn", kn), ("rope", rope), ("Kc", Kc),
                 ("Vc", Vc), ("w_o", w_o), ("workspace", workspace)):
        _cuda_contig(n, t)
    _need(h.dtype == torch.float32 and in_norm.dtype == torch.float32 and in_norm.numel() == hidden,
          "h and in_norm must be float32 [hidden]")
    _need(w_qkv.dtype == w_o.dtype and w_qkv.dtype in (torch.bfloat16, torch.float32), "weights: one of bf16, fp32")
    _need(w_qkv.numel() == (nq + 2 * nkv) * hd * hidden, "w_qkv must be [(nq+2nkv)*hd][hidden]")
    _need(w_o.numel() == hidden * nq * hd, "w_o must be [hidden][nq*hd]")
    _need(Kc.shape == Vc.shape and Kc.numel() == nkv * max_len * hd and Kc.dtype == Vc.dtype,
          "Kc/Vc must be [nkv][max_len][hd]")
    _need(rope.dtype == torch.float32 and rope.numel() >= max_len * hd, "rope must be float32 [max_len][hd]")
    if pos_ptr is not None:
        _need(pos_ptr.is_cuda and pos_ptr.dtype == torch.int64, "pos_ptr must be a CUDA int64 tensor")
    ws_n = workspace.numel() * workspace.element_size()
    with _nvtx("sk_decode_attention_block"):
        check(lib().sk_decode_attention_block(_ptr(h), _ptr(in_norm), float(eps_in), _ptr(w_qkv), _ptr(qn), _ptr(kn),
                                              float(eps), _ptr(rope), _ptr(Kc), _ptr(Vc), _ptr(pos_ptr), int(pos_add),
                                              int(max_len), int(nq), int(nkv), int(hd), _ptr(w_o), int(hidden),
                                              _dtype_code(w_qkv.dtype), _dtype_code(Kc.dtype), _ptr(workspace), ws_n,
                                              _lib.SK_DECODE_KV_STABLE if kv_stable else 0, _stream()),
              "sk_decode_attention_block")
    return h


def prefill_attention(qkv_rows: torch.Tensor, qn: torch.Tensor, kn: torch.Tensor, eps: float, rope: torch.Tensor,
                      Kc: torch.Tensor, Vc: torch.Tensor, pos0: int, max_len: int, nq: int, nkv: int,
                      out: torch.Tensor | None = None, q_buf: torch.Tensor | None = None) -> torch.Tensor:
    """The prompt's causal attention for one talker layer (the HF SDPA prefill, qwen3/fast.py:251-263):
    qkv_rows float32 (T, (nq + 2*nkv)*128), one row per prompt token at positions pos0..pos0+T-1;
    appends k/v to the caches and returns (T, nq*128) in the cache dtype (bf16: tensor cores; fp32:
    the fp32 parity mode)."""
    hd = Kc.shape[-1]
    for n, t in (("qkv_rows", qkv_rows), ("qn", qn), ("kn", kn), ("rope", rope), ("Kc", Kc), ("Vc", Vc)):
        _cuda_contig(n, t)
    T = qkv_rows.shape[0]
    _need(qkv_rows.dtype == torch.float32 and qkv_rows.shape == (T, (nq + 2 * nkv) * hd),
          "qkv_rows must be float32 (T, (nq+2nkv)*hd)")
    dt = Kc.dtype
    _need(dt in (torch.bfloat16, torch.float32) and Vc.dtype == dt, "caches must both be bfloat16 or float32")
    if out is None:
        out = torch.empty((T, nq * hd), device=Kc.device, dtype=dt)
    if q_buf is None:
        q_buf = torch.empty((nq, T, hd), device=Kc.device, dtype=dt)
    _cuda_contig("out", out)
    _cuda_contig("q_buf", q_buf)
    _need(out.numel() == T * nq * hd and out.dtype == dt, f"out must hold T*nq*hd {dt}")
    _need(q_buf.numel() >= nq * T * hd and q_buf.dtype == dt, f"q_buf must hold nq*T*hd {dt}")
    with _nvtx("sk_prefill_attention"):
        check(lib().sk_prefill_attention(_ptr(qkv_rows), _ptr(qn), _ptr(kn), float(eps), _ptr(rope), _ptr(Kc), _ptr(Vc),
                                         int(pos0), int(T), int(max_len), int(nq), int(nkv), int(hd), _ptr(out),
                                         _ptr(q_buf), _dtype_code(Kc.dtype), _stream()), "sk_prefill_attention")
    return out


def version() -> int:
    return int(lib().sk_version())


__all__ = ["dit_qkv_prologue", "dit_attention", "sdpa", "decode_attention", "decode_workspace",
           "decode_attention_block", "decode_block_workspace", "decode_attention_grouped", "decode_requests",
           "decode_workspace_bytes", "device_error", "version", "_lib"]
