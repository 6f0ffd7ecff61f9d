"""CPU oracle of the Irodori-TTS DiT attention as the sokutou engine runs it — TEST INFRASTRUCTURE.

Restates, in numpy float64:
  - the Q/K/V producer `qkv` (engine/fused.py:117-180; same math as engine/fast.py:156-168):
    per-head RMSNorm of q and k with per-head weights, RoPE on heads h < H/2 with interleaved
    pairs (2i, 2i+1), v untouched;
  - the CFG key mask (engine/bucket.py:252-258) and its additive form (engine/fused.py:373-378);
  - the attention itself, F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    (engine/fused.py:295): softmax(q·kᵀ/sqrt(hd) + bias)·v, non-causal, keys ordered
    [latent | text | speaker] (engine/fast.py:167-168);
  - the consumer `gate` (engine/fused.py:182-190): y · sigmoid(gate) in float32, rounded once, with
    the FP8 e4m3 output form (engine/fused.py:52-76).
  - the projections around them, `mm` = F.linear(x, w) (engine/fused.py:262-264): x · wᵀ in float64,
    rounded once to the output type.

The RoPE frequency table of Irodori-TTS (`model._rope_freqs`, engine/fast.py:264) lives in the
third-party package irodori_tts @ 7ed4374 (not present here); `rope_freqs` restates the
standard formula with theta = 1e4 that BASELINE names.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module.
"""

from __future__ import annotations

import numpy as np

NEG_INF = float("-inf")


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32/64 values to bfloat16 (round to nearest even) and return them as float32.

    Same rounding as the reference's `ST` (engine/fused.py:38-43) and torch's bfloat16 cast.
    NaN maps to the canonical quiet NaN 0x7fc0.
    """
    f = np.asarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, 0x7FC0, r).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32).reshape(f.shape)


def rope_freqs(n_pos: int, hd: int, theta: float = 1e4) -> np.ndarray:
    """(n_pos, hd/2, 2) float32 table of (cos, sin) of pos * theta^(-2i/hd).

    The real view of the complex table the engine precomputes (engine/fast.py:264,
    engine/fused.py:347). Computed in float64, stored float32 like the engine's table.
    """
    inv = 1.0 / (theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    ang = np.arange(n_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def qkv_prologue(o4: np.ndarray, qk_w: np.ndarray, freqs: np.ndarray, B: int, L: int, H: int, hd: int,
                 eps: float, out_bf16: bool):
    """Q/K/V producer of one layer (engine/fused.py:117-180, the p < L branch).

    o4: (B*L, 4*H*hd) rows [q | k | v | gate]; qk_w: (2, H, hd); freqs: (>= L, hd/2, 2).
    Returns q, k_lat, v_lat, each (B, H, L, hd). Sum of squares in float64 as the kernel does
    (engine/fused.py:143); the product x * r * w and the rotation in float64 here (the kernel uses
    float32; the difference is far below the bf16 store). When out_bf16, values are rounded to
    bfloat16 like the kernel's `ST` store.
    """
    D = H * hd
    x = np.asarray(o4, dtype=np.float64).reshape(B, L, 4, H, hd)
    qk = x[:, :, :2]                                            # (B, L, 2, H, hd)
    ss = (qk * qk).sum(-1, keepdims=True)
    r = 1.0 / np.sqrt(ss / hd + eps)                            # rsqrt(mean + eps), engine/fused.py:148
    qk = qk * r * np.asarray(qk_w, np.float64).reshape(1, 1, 2, H, hd)
    half = H // 2                                               # rotated heads, engine/fused.py:152,167
    fr = np.asarray(freqs[:L], np.float64)                      # (L, hd/2, 2)
    c = fr[None, :, None, None, :, 0]
    s = fr[None, :, None, None, :, 1]
    a0 = qk[:, :, :, :half, 0::2]
    a1 = qk[:, :, :, :half, 1::2]
    rot = qk.copy()
    rot[:, :, :, :half, 0::2] = a0 * c - a1 * s                 # engine/fused.py:169
    rot[:, :, :, :half, 1::2] = a0 * s + a1 * c
    q = rot[:, :, 0].transpose(0, 2, 1, 3)                      # (B, H, L, hd)
    k = rot[:, :, 1].transpose(0, 2, 1, 3)
    v = x[:, :, 2].transpose(0, 2, 1, 3)
    if out_bf16:
        q, k, v = (bf16_round(t).astype(np.float64) for t in (q, k, v))
    return np.ascontiguousarray(q), np.ascontiguousarray(k), np.ascontiguousarray(v)


def cfg_key_mask(lb: int, tb: int, n_spk: int, seq_len: int, n_text: int) -> np.ndarray:
    """(3, lb + tb + n_spk) bool: which keys each CFG row sees (engine/bucket.py:252-258).

    Row 0 cond: valid latent + valid text + all speaker. Row 1 text-uncond: valid latent + all
    speaker. Row 2 speaker-uncond: valid latent + valid text. Padding is masked in every row.
    """
    m = np.zeros((3, lb + tb + n_spk), dtype=bool)
    m[:, :seq_len] = True
    m[0, lb:lb + n_text] = True
    m[2, lb:lb + n_text] = True
    m[0:2, lb + tb:] = True
    return m


def additive_bias(mask: np.ndarray) -> np.ndarray:
    """0 where a key is visible, -inf where it is not (engine/fused.py:377)."""
    return np.where(mask, 0.0, NEG_INF)


def dit_attention(q, k_lat, v_lat, k_ctx=None, v_ctx=None, bias=None, scale=None) -> np.ndarray:
    """y = softmax(q·kᵀ·scale + bias)·v per (b, h), float64; returns (B, L, H, hd).

    q: (B, H, L, hd); k_lat/v_lat: (B, H, Lk, hd); k_ctx/v_ctx: (B or 1, S, H, hd) — the
    conditioning keys appended after the latent keys (engine/fast.py:167-168); bias: (B or 1, K).
    scale defaults to 1/sqrt(hd) (torch SDPA default, engine/fused.py:295). Rows whose keys are all
    masked give 0, as torch's CPU SDPA does.
    """
    q = np.asarray(q, np.float64)
    B, H, L, hd = q.shape
    k = np.asarray(k_lat, np.float64)
    v = np.asarray(v_lat, np.float64)
    if k_ctx is not None:
        kc = np.broadcast_to(np.asarray(k_ctx, np.float64), (B,) + np.shape(k_ctx)[1:]).transpose(0, 2, 1, 3)
        vc = np.broadcast_to(np.asarray(v_ctx, np.float64), (B,) + np.shape(v_ctx)[1:]).transpose(0, 2, 1, 3)
        k = np.concatenate([k, kc], axis=2)
        v = np.concatenate([v, vc], axis=2)
    if scale is None or scale <= 0:
        scale = 1.0 / np.sqrt(hd)
    s = np.einsum("bhld,bhkd->bhlk", q, k) * scale
    if bias is not None:
        bb = np.broadcast_to(np.asarray(bias, np.float64).reshape(-1, k.shape[2]), (B, k.shape[2]))
        s = s + bb[:, None, None, :]
    m = s.max(-1, keepdims=True)
    m = np.where(np.isneginf(m), 0.0, m)
    p = np.exp(s - m)
    den = p.sum(-1, keepdims=True)
    y = np.einsum("bhlk,bhkd->bhld", p, v) / np.where(den == 0, 1.0, den)
    return np.ascontiguousarray(y.transpose(0, 2, 1, 3))


def dit_attention_torch_cpu(q, k_lat, v_lat, k_ctx, v_ctx, bias, threads: int | None = None):
    """The reference's own CPU arithmetic for the timed baseline: the ctx keys copied into every
    batch row (engine/fused.py:127-136) and torch's F.scaled_dot_product_attention in float32
    (engine/fused.py:295). Inputs are torch CPU tensors; returns y (B, L, H, hd) float32."""
    import torch
    import torch.nn.functional as F

    if threads:
        torch.set_num_threads(threads)
    B = q.shape[0]
    k = torch.cat([k_lat, k_ctx.expand(B, -1, -1, -1).transpose(1, 2)], dim=2)
    v = torch.cat([v_lat, v_ctx.expand(B, -1, -1, -1).transpose(1, 2)], dim=2)
    y = F.scaled_dot_product_attention(q, k, v, attn_mask=bias.reshape(-1, 1, 1, k.shape[2]))
    return y.transpose(1, 2)


# ---- attention consumer: gate ------------------------------------------------------------------------

def _e4m3_table() -> np.ndarray:
    """Values of the 127 non-negative finite e4m3 codes 0x00..0x7e (bias 7, 3 mantissa bits,
    subnormal step 2^-9), indexed by code."""
    codes = np.arange(0x7F)
    e, m = codes >> 3, codes & 7
    return np.where(e == 0, m * 2.0 ** -9, (1 + m / 8.0) * 2.0 ** (e - 7.0))


def e4m3_encode(x) -> np.ndarray:
    """float32 -> e4m3 code (uint8) as the reference's FP8 writer defines it (engine/fused.py:60-72):
    nearest representable value with ties to the even code, magnitudes at or past 448 -> ±448 (0x7e),
    NaN -> 0x7f, sign kept (also for zero). Written as a nearest-neighbour search over the code
    table rather than bit arithmetic."""
    f = np.asarray(x, dtype=np.float32)
    a = np.abs(f).astype(np.float64)
    sign = (f.view(np.uint32) >> 24).astype(np.uint8) & 0x80
    tab = _e4m3_table()
    a_c = np.minimum(np.nan_to_num(a, nan=0.0, posinf=448.0), 448.0)
    hi = np.clip(np.searchsorted(tab, a_c, side="left"), 0, len(tab) - 1)   # first value >= a
    lo = np.clip(hi - 1, 0, len(tab) - 1)
    d_hi, d_lo = tab[hi] - a_c, a_c - tab[lo]
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(a_c >= 448.0, 0x7E, code).astype(np.uint8)
    out = (code | sign).astype(np.uint8)
    return np.where(np.isnan(f), np.uint8(0x7F), out).astype(np.uint8)


def e4m3_decode(c) -> np.ndarray:
    c = np.asarray(c, dtype=np.uint8)
    mag = _e4m3_table()[np.minimum(c & 0x7F, 0x7E)]
    mag = np.where((c & 0x7F) == 0x7F, np.nan, mag)
    return np.where(c & 0x80, -mag, mag).astype(np.float32)


def linear(x, w, out: str = "f32") -> np.ndarray:
    """F.linear(x, w) without bias (engine/fused.py:262-264): x (M, K) · w (N, K)ᵀ in float64, rounded
    once to `out` ("f32" or "bf16", round to nearest even)."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    y = y.astype(np.float32)
    return bf16_round(y) if out == "bf16" else y


def linear_fp8(x8, w8, inv_scale_x: float, inv_scale_w: float) -> np.ndarray:
    """torch._scaled_mm(x8, w8.t(), inv_x, inv_w, out_dtype=bf16) (engine/fp8.py:87-89): the e4m3 codes
    x8 (M, K) and w8 (N, K) decoded exactly, multiplied in float64, times inv_x · inv_w (float32),
    rounded once to bf16 (returned as float32)."""
    x = e4m3_decode(np.asarray(x8, np.uint8)).astype(np.float64)
    w = e4m3_decode(np.asarray(w8, np.uint8)).astype(np.float64)
    s = np.float64(np.float32(inv_scale_x) * np.float32(inv_scale_w))
    return bf16_round((x @ w.T * s).astype(np.float32))


def gate(y, o4, out: str = "f32", out_scale: float = 1.0) -> np.ndarray:
    """out[r, c] = y[r, c] · (1 / (1 + exp(-o4[r, 3D + c]))) in float32 (engine/fused.py:182-190),
    then rounded once: out = "f32" (as is), "bf16" (round to nearest even, returned as float32) or
    "e4m3" (codes of value · out_scale). y: (rows, D) or anything holding rows·D values."""
    o4 = np.asarray(o4, dtype=np.float32)
    rows, D = o4.shape[0], o4.shape[1] // 4
    yv = np.asarray(y, dtype=np.float32).reshape(rows, D)
    g = o4[:, 3 * D:]
    with np.errstate(over="ignore"):
        sig = np.float32(1.0) / (np.float32(1.0) + np.exp(-g, dtype=np.float32))
    r = (yv * sig).astype(np.float32)
    if out == "f32":
        return r
    if out == "bf16":
        return bf16_round(r)
    if out == "e4m3":
        return e4m3_encode((r * np.float32(out_scale)).astype(np.float32))
    raise ValueError(out)


def attention_layer(o4, qk_w, freqs, B: int, L: int, H: int, hd: int, eps: float, k_ctx=None, v_ctx=None,
                    bias=None, bf16: bool = True) -> np.ndarray:
    """The attention block of one DiT layer as the engine runs it (engine/fused.py:293-298): the `qkv`
    producer, SDPA over [latent | ctx] keys, the `gate` consumer. With bf16, q/k/v and the SDPA output
    are rounded to bfloat16 between the steps as the engine's buffers hold them, and the gated product
    is rounded once. Returns (B*L, H*hd) as float32."""
    q, k, v = qkv_prologue(o4, qk_w, freqs, B, L, H, hd, eps, bf16)
    y = dit_attention(q, k, v, k_ctx, v_ctx, bias)
    y = y.reshape(B * L, H * hd).astype(np.float32)
    if bf16:
        y = bf16_round(y)
    return gate(y, o4, "bf16" if bf16 else "f32")
