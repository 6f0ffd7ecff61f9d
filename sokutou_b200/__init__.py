"""sokutou_b200 — the B200-native attention path of the sokutou TTS engine.

Two attention shapes, each a drop-in for one call site of the reference engine:
  * DiT attention (Irodori-TTS flow-matching, CFG-batched, key-padding bias): `ops.dit_attention`,
    `ops.sdpa`, `ops.dit_qkv_prologue`, `dit.DitLayerAttention` — engine/fused.py:293-298.
  * Qwen3-TTS talker decode attention (GQA, QK-RMSNorm + RoPE + KV append fused): `ops.decode_attention`,
    `qwen3.TalkerAttention` — qwen3/kernels.py:338-414, 622-624.
The kernels live in the in-tree shared library `lib/libsokutou_b200.so` (C ABI:
include/sokutou_b200.h), built for sm_100a by `python -m sokutou_b200.build`.
"""

from . import ops
from .ops import decode_attention, device_error, dit_attention, dit_qkv_prologue, sdpa

__all__ = ["ops", "decode_attention", "device_error", "dit_attention", "dit_qkv_prologue", "sdpa"]
