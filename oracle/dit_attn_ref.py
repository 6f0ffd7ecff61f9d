"""CPU oracle of the Irodori-TTS DiT attention as the sokutou engine runs it — TEST INFRASTRUCTURE.

Restates, in numpy float64:
  - the Q/K/V producer `qkv` (engine/fused.py:117-180; same math as engine/fast.py:156-168):
    per-head RMSNorm of q and k with per-head weights, RoPE on heads h < H/2 with interleaved
    pairs (2i, 2i+1), v untouched;
  - the CFG key mask (engine/bucket.py:252-258) and its additive form (engine/fused.py:373-378);
  - the attention itself, F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    (engine/fused.py:295): softmax(q·kᵀ/sqrt(hd) + bias)·v, non-causal, keys ordered
    [latent | text | speaker] (engine/fast.py:167-168).

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
