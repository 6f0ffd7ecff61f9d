"""CPU oracle of the Qwen3-TTS talker decode attention — TEST INFRASTRUCTURE.

Restates the reference engine's NVRTC kernel `attn` (qwen3/kernels.py:338-414) in numpy:
  (1) k <- RMSNorm(k)·kn, rotate-half RoPE, written to the cache at `pos`; v written raw
      (qwen3/kernels.py:354-367); the cache stores bf16 (or fp32 in the fp32 mode, ACT_F32);
  (2) q <- RMSNorm(q)·qn, RoPE, × 1/sqrt(128) (qwen3/kernels.py:369-380);
  (3) scores over T = pos + 1 cached keys, read back in the cache dtype (:383-392);
  (4) softmax (:394-408); (5) out = Σ p·V / Σ p (:410-413).
GQA: q head qh uses kv head qh // (nq // nkv) (the kernel's kvh*2 + part, :369).
The RoPE table follows qwen3/kernels.py:473-477: row pos = [cos(pos·f) | sin(pos·f)] for the 64
inverse frequencies f = theta^(-2i/128) of the model's rotary embedding (transformers' default
rope init; attention_scaling 1).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module.
"""

from __future__ import annotations

import numpy as np

from .dit_attn_ref import bf16_round


def rope_table(max_len: int, hd: int = 128, theta: float = 1e6) -> np.ndarray:
    """float32 (max_len, hd): [cos | sin] of pos * inv_freq (qwen3/kernels.py:473-477).

    inv_freq is transformers' default rope init, computed with torch's float32 pow exactly as the
    model builds it (one ulp there moves the angle at position 1000 by ~1e-4); the angle is formed
    in float32 like the reference (f = arange * inv_freq), cos/sin in float64, stored float32.
    """
    import torch

    inv = (1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))).numpy()
    f = (np.arange(max_len, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return np.concatenate([np.cos(f.astype(np.float64)), np.sin(f.astype(np.float64))], axis=1).astype(np.float32)


def _rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


def _rope(x: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)   # d<64 ? -x[d+64] : x[d-64]
    return x * c + rot * s


def store_round(x: np.ndarray, cache_dtype: str) -> np.ndarray:
    """Value as the cache holds it (qwen3/kernels.py:55-56 STC): bf16 RNE or exact fp32."""
    return bf16_round(x) if cache_dtype == "bf16" else np.asarray(x, np.float32)


def decode_step(qkv, qn, kn, eps, rope, Kc, Vc, pos: int, nq: int, nkv: int, cache_dtype: str = "bf16"):
    """One decode step of one layer. Mutates Kc/Vc at `pos` and returns out: float64 (nq*hd,).

    qkv: (nq + 2*nkv)*hd float32; qn, kn: (hd,); rope: (max_len, hd); Kc, Vc: (nkv, max_len, hd)
    float32 or float64 arrays whose values are representable in `cache_dtype` (float64 caches avoid
    a conversion per call).
    """
    hd = Kc.shape[-1]
    half = hd // 2
    x = np.asarray(qkv, np.float64)
    q = x[: nq * hd].reshape(nq, hd)
    k = x[nq * hd: (nq + nkv) * hd].reshape(nkv, hd)
    v = x[(nq + nkv) * hd:].reshape(nkv, hd)
    row = np.asarray(rope[pos], np.float64)
    c = np.concatenate([row[:half], row[:half]])
    s = np.concatenate([row[half:], row[half:]])
    kr = _rope(_rms(k, np.asarray(kn, np.float64), eps), c, s)
    Kc[:, pos] = store_round(kr, cache_dtype)
    Vc[:, pos] = store_round(v, cache_dtype)
    qr = _rope(_rms(q, np.asarray(qn, np.float64), eps), c, s) / np.sqrt(hd)
    T = pos + 1
    g = nq // nkv
    K = np.asarray(Kc[:, :T], np.float64)
    V = np.asarray(Vc[:, :T], np.float64)
    sc = np.matmul(K, qr.reshape(nkv, g, hd).transpose(0, 2, 1))      # (nkv, T, g)
    p = np.exp(sc - sc.max(axis=1, keepdims=True))
    out = np.matmul(p.transpose(0, 2, 1), V) / p.sum(axis=1)[:, :, None]  # (nkv, g, hd)
    return out.reshape(-1)


def prefill(qkv_rows, qn, kn, eps, rope, Kc, Vc, pos0: int, nq: int, nkv: int, cache_dtype: str = "bf16"):
    """The prompt's causal attention (the HF talker's SDPA prefill, qwen3/fast.py:251-263) as a run of
    decode steps: token t at position pos0 + t appends its k/v and attends over rows [0, pos0 + t] —
    causal attention over the same cache, by construction. Mutates Kc/Vc; returns float64 (T, nq*hd)."""
    rows = np.asarray(qkv_rows)
    return np.stack([decode_step(rows[t], qn, kn, eps, rope, Kc, Vc, pos0 + t, nq, nkv, cache_dtype)
                     for t in range(rows.shape[0])])


def decode_step_f32(qkv, qn, kn, eps, rope, Kc, Vc, pos: int, nq: int, nkv: int, cache_dtype: str = "bf16"):
    """Same step in float32 arithmetic (numpy), used as the timed CPU port baseline."""
    hd = Kc.shape[-1]
    half = hd // 2
    x = np.asarray(qkv, np.float32)
    q = x[: nq * hd].reshape(nq, hd)
    k = x[nq * hd: (nq + nkv) * hd].reshape(nkv, hd)
    v = x[(nq + nkv) * hd:].reshape(nkv, hd)
    row = rope[pos]
    c = np.concatenate([row[:half], row[:half]])
    s = np.concatenate([row[half:], row[half:]])
    kr = _rope(_rms(k, kn, np.float32(eps)), c, s)
    Kc[:, pos] = store_round(kr, cache_dtype)
    Vc[:, pos] = store_round(v, cache_dtype)
    qr = _rope(_rms(q, qn, np.float32(eps)), c, s) * np.float32(1.0 / np.sqrt(hd))
    T = pos + 1
    g = nq // nkv
    qg = qr.reshape(nkv, g, hd)
    sc = np.einsum("hgd,htd->hgt", qg, Kc[:, :T])
    p = np.exp(sc - sc.max(-1, keepdims=True))
    out = np.einsum("hgt,htd->hgd", p, Vc[:, :T]) / p.sum(-1, keepdims=True)
    return out.reshape(-1)


def rms_gemv(h, nw, eps: float, W):
    """out = W · RMSNorm(h) with the RMSNorm weight nw — the reference's `rms_gemv` (qwen3/kernels.py:271-275:
    gemv_core :152-255 + rms_gemv_body :257-270): x = h ⊙ nw, inv = 1/sqrt(Σh²/K + eps), out[r] =
    (Σ_k W[r,k]·x[k])·inv. float64; W as stored (bf16 or fp32 values)."""
    h = np.asarray(h, np.float64)
    x = h * np.asarray(nw, np.float64)
    inv = 1.0 / np.sqrt((h * h).mean() + eps)
    return (np.asarray(W, np.float64) @ x) * inv


def gemv_acc(x, W, out):
    """out + W · x — the reference's `gemv` with accumulate = 1 (qwen3/kernels.py:301-305, gemv_body :285-300):
    the o projection added into the residual stream. float64."""
    return np.asarray(out, np.float64) + np.asarray(W, np.float64) @ np.asarray(x, np.float64)


def decode_block(h, in_norm, eps_in: float, w_qkv, qn, kn, eps: float, rope, Kc, Vc, pos: int, nq: int, nkv: int,
                 w_o, cache_dtype: str = "bf16"):
    """One talker layer's attention block as the reference launches it at qwen3/kernels.py:619-624:
    rms_gemv(qkv) -> attn -> gemv(o) accumulating into the residual h. Mutates Kc/Vc at `pos` (the
    attention appends k/v); returns the new h (float64)."""
    qkv = rms_gemv(h, in_norm, eps_in, w_qkv)
    att = decode_step(qkv, qn, kn, eps, rope, Kc, Vc, pos, nq, nkv, cache_dtype)
    return gemv_acc(att, w_o, h)


def talker_greedy(weights: dict, n_layers: int, nq: int, nkv: int, hd: int, max_len: int, prompt_len: int,
                  n_new: int, eps: float, rope, cache_dtype: str = "f32"):
    """Greedy tokens of the synthetic talker stack, float64 (see sokutou_b200.workloads.SyntheticTalker).

    Per position: h = input row; for each layer h += W_o · attn(W_qkv · rmsnorm(h)); token =
    argmax(W_out · rmsnorm(h)). Positions 0..prompt_len-1 take the prompt rows; each later position
    takes the embedding of the previous token. Returns the tokens of positions prompt_len-1 ...
    prompt_len-1+n_new (n_new + 1 tokens).
    """
    w = {k: np.asarray(v, np.float64) for k, v in weights.items()}
    Kc = np.zeros((n_layers, nkv, max_len, hd))
    Vc = np.zeros((n_layers, nkv, max_len, hd))
    rms = lambda h: h / np.sqrt((h * h).mean() + eps)
    tokens = []
    tok = None
    for pos in range(prompt_len + n_new):
        h = w["prompt"][pos] if pos < prompt_len else w["emb"][tok]
        for li in range(n_layers):
            qkv = w["w_qkv"][li] @ rms(h)
            att = decode_step(qkv, w["qn"][li], w["kn"][li], eps, rope, Kc[li], Vc[li], pos, nq, nkv, cache_dtype)
            h = h + w["w_o"][li] @ att
        if pos >= prompt_len - 1:
            tok = int(np.argmax(w["w_out"] @ rms(h)))
            tokens.append(tok)
    return tokens


def decode_block_pair(h2, in_norm, eps_in: float, w_qkv, qn, kn, eps: float, rope, Kc, Vc, nq: int, nkv: int, w_o,
                      cache_dtype: str = "bf16"):
    """The attention half of the code predictor's paired pass over positions 0 and 1
    (qwen3/kernels.py:600-617, `_cp_layers_pair`): `rms_gemv2` projects both rows first (each row's own
    RMSNorm), then `attn` runs position 0 (appending its k/v at row 0 of the 16-row cache) and then
    position 1 (appending at row 1 and attending over rows 0..1), then `gemv2` adds W_o · att to both
    residual rows. Mutates Kc/Vc; returns the two new rows of h (float64). (The reference skips row 0's
    o projection in the stack's last layer; that choice sits outside the attention block.)"""
    qkv = [rms_gemv(h2[r], in_norm, eps_in, w_qkv) for r in (0, 1)]
    att = [decode_step(qkv[r], qn, kn, eps, rope, Kc, Vc, r, nq, nkv, cache_dtype) for r in (0, 1)]
    return [gemv_acc(att[r], w_o, h2[r]) for r in (0, 1)]
