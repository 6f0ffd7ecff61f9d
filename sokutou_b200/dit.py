"""The DiT attention call site of the sokutou engine, on the B200 kernels.

Mirrors the attention section of one `FusedCore` layer (engine/fused.py:277-298):

    o4 = mm(h, w_qkvg)                                           # (B*L, 4D) = [q | k | v | gate]
    qkv kernel      -> q (B,H,L,hd), k/v (B,H,L+S,hd) with ctx copied per batch row
    y = F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    gate kernel reads y.transpose(1, 2)  (B, L, H·hd)

Here the producer writes only the latent keys and the attention reads the conditioning (text +
speaker) K/V in place from the per-layer `(S, H, hd)` buffer all CFG rows share, so the per-batch
copy of engine/fused.py:127-136 disappears. Buffers are allocated once per shape, before any CUDA
graph capture, as the reference allocates its own (engine/fused.py:277-282).
"""

from __future__ import annotations

import torch

from . import ops


def cfg_key_mask(lb: int, tb: int, n_spk: int, seq_len: int, n_text: int, device=None) -> torch.Tensor:
    """(3, lb + tb + n_spk) bool, the CFG key mask of engine/bucket.py:252-258.

    Row 0 cond: valid latent + valid text + every speaker key; row 1 text-uncond: no text;
    row 2 speaker-uncond: no speaker. Padding keys are masked in every row.
    """
    m = torch.zeros((3, lb + tb + n_spk), dtype=torch.bool, device=device)
    m[:, :seq_len] = True
    m[0, lb:lb + n_text] = True
    m[2, lb:lb + n_text] = True
    m[0:2, lb + tb:] = True
    return m


def cfg_bias(lb: int, tb: int, n_spk: int, seq_len: int, n_text: int, device=None,
             dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """(3, K) additive bias, 0 / -inf (engine/fused.py:373-378). Row 0 alone serves batch-1 steps
    (engine/fused.py:447)."""
    m = cfg_key_mask(lb, tb, n_spk, seq_len, n_text, device)
    return torch.zeros(m.shape, dtype=dtype, device=device).masked_fill_(~m, float("-inf"))


class DitLayerAttention:
    """The attention block of one DiT layer for a fixed (B, L, H, hd, S) shape: Q/K/V producer,
    attention and `gate` consumer (engine/fused.py:293-298), buffers allocated once (before capture).

    `__call__(o4, qk_w, freqs, ctx_k, ctx_v, bias)` returns y · sigmoid(gate) as (B*L, H*hd) in o4's
    dtype — the input of the w_o GEMM. ctx_k/ctx_v: (S, H, hd), the layer's conditioning keys (text
    then speaker, already k-normed, engine/fast.py:327-338); bias: (B, L + S) or (L + S,).
    bf16 runs the fused block by default (two launches; `fused=False`: the three separate launches,
    which give the same bits); float32 always runs the three separate launches.
    `attention(...)` stops before the gate and returns y (B, L, H, hd).
    """

    def __init__(self, B: int, L: int, H: int, hd: int, S: int, dtype: torch.dtype, device, eps: float = 1e-6,
                 fused: bool = True):
        self.B, self.L, self.H, self.hd, self.S, self.eps = B, L, H, hd, S, eps
        self.fused = fused and dtype == torch.bfloat16
        mk = lambda: torch.empty((B, H, L, hd), dtype=dtype, device=device)
        self.q, self.k, self.v = mk(), mk(), mk()
        self.y = torch.empty((B, L, H, hd), dtype=dtype, device=device)
        self.out = torch.empty((B * L, H * hd), dtype=dtype, device=device)

    def attention(self, o4, qk_w, freqs, ctx_k, ctx_v, bias):
        ops.dit_qkv_prologue(o4, qk_w, freqs, self.B, self.L, self.H, self.hd, self.eps, out=(self.q, self.k, self.v))
        return ops.dit_attention(self.q, self.k, self.v, ctx_k, ctx_v, bias, out=self.y)

    def __call__(self, o4, qk_w, freqs, ctx_k, ctx_v, bias):
        if self.fused:
            return ops.dit_attention_layer(o4, qk_w, freqs, self.B, self.L, self.H, self.hd, self.eps, ctx_k, ctx_v,
                                           bias, out=self.out, qkv_bufs=(self.q, self.k, self.v))
        self.attention(o4, qk_w, freqs, ctx_k, ctx_v, bias)
        return ops.dit_gate(self.y, o4, out=self.out)
