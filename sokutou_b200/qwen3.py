"""The Qwen3-TTS talker decode-attention call site of the sokutou engine, on the B200 kernel.

Mirrors the attention state of `Qwen3Kernels` (qwen3/kernels.py:483-706): the per-layer KV caches
(HF StaticCache tensors `[nkv][max_cache][128]`, qwen3/kernels.py:702-705), the RoPE table
(qwen3/kernels.py:473-477), the device-side position (qwen3/fast.py:102) and the per-layer launch
of qwen3/kernels.py:622-624, plus the caller-owned split-KV workspace the B200 kernel needs.
"""

from __future__ import annotations

import torch

from . import ops


def rope_table(max_len: int, theta: float, hd: int = 128, device=None) -> torch.Tensor:
    """float32 (max_len, hd) = [cos(pos·f) | sin(pos·f)] with f = theta^(-2i/hd) computed in float32
    as transformers' default rope init does (qwen3/kernels.py:473-477)."""
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.int64, device=device).float() / hd))
    f = torch.arange(max_len, device=device, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat([f.cos(), f.sin()], dim=1).contiguous()


class TalkerAttention:
    """KV caches, RoPE table, position and workspace of one talker stack.

    `attn(layer, qkv, qn, kn, out, pos_add=0)` runs one layer's decode attention exactly where
    `_layers` launches the reference kernel; the position is read on the device from `self.pos`
    (advance it with `self.pos.add_(1)` inside the captured frame, qwen3/kernels.py:692).
    """

    def __init__(self, n_layers: int, nq: int, nkv: int, max_len: int, theta: float, eps: float, device,
                 cache_dtype: torch.dtype = torch.bfloat16, hd: int = 128, use_pos: bool = True):
        self.n_layers, self.nq, self.nkv, self.hd, self.max_len, self.eps = n_layers, nq, nkv, hd, max_len, eps
        self.k = torch.zeros((n_layers, nkv, max_len, hd), dtype=cache_dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.rope = rope_table(max_len, theta, hd, device)
        self.pos = torch.zeros((1,), dtype=torch.int64, device=device) if use_pos else None
        self.ws = ops.decode_workspace(max_len, nq, nkv, device, hd, cache_dtype)
        self.block_ws = ops.decode_block_workspace(max_len, nq, nkv, device, hd)

    def attn(self, layer: int, qkv: torch.Tensor, qn: torch.Tensor, kn: torch.Tensor, out: torch.Tensor,
             pos_add: int = 0, kv_stable: bool = False) -> torch.Tensor:
        """kv_stable: the kernel launched just before writes neither self.pos nor this layer's cache (true
        after the layer's qkv projection; false right after the position advance)."""
        return ops.decode_attention(qkv, qn, kn, self.eps, self.rope, self.k[layer], self.v[layer], self.pos, pos_add,
                                    self.max_len, self.nq, self.nkv, out, self.ws, kv_stable)

    def block(self, layer: int, h: torch.Tensor, in_norm: torch.Tensor, eps_in: float, w_qkv: torch.Tensor,
              qn: torch.Tensor, kn: torch.Tensor, w_o: torch.Tensor, pos_add: int = 0,
              kv_stable: bool = False) -> torch.Tensor:
        """The layer's whole attention block — rms_gemv(qkv), the decode attention and gemv(o) into the
        residual h (qwen3/kernels.py:619-624) — in one launch; h (fp32 [hidden]) is updated in place."""
        return ops.decode_attention_block(h, in_norm, eps_in, w_qkv, qn, kn, self.eps, self.rope, self.k[layer],
                                          self.v[layer], self.pos, pos_add, self.max_len, self.nq, self.nkv, w_o,
                                          self.block_ws, kv_stable)
