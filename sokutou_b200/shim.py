"""Drop-in shims for the reference engine's two attention call sites, so that an engine instance runs its
attention on this library without edits to its code.

DiT (engine/fused.py:295): `FusedCore.__call__` calls `F.scaled_dot_product_attention(q, k, v,
attn_mask=bias)` through its module's global `F` (torch.nn.functional). `install_sdpa(module)` replaces
that global with a namespace whose `scaled_dot_product_attention` is `ops.sdpa` and whose every other
attribute is torch.nn.functional's own; `.restore()` (or leaving the `with` block) puts the module back.

Qwen3 (qwen3/kernels.py:575-577, 600-627): `Qwen3Kernels._launch` calls its NVRTC kernels through the
dict `self.k` as `k[name]((grid,), (block,), args, shared_mem=...)`, the tensor arguments already
turned into raw addresses (`_ptr`, qwen3/kernels.py:418-422: numpy uintp, 0 for None) and the scalars
numpy int32 / float32. `DecodeAttnKernel` is such a callable for "attn": it takes the same argument
tuple (qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, nkv, out) and runs
sk_decode_attention on torch's current stream with a split-KV workspace of its own (one per instance,
sized for the largest max_len it will see; the talker and the code predictor share it, as they share the
reference's one kernel). `patch_kernels(engine, ...)` puts one into `engine.k["attn"]`.
"""

from __future__ import annotations

import types

import torch

from . import _lib, ops
from ._lib import SK_BF16, SK_F32, check


class SdpaPatch:
    """The swap done by install_sdpa; `restore()` undoes it (also on leaving a `with` block)."""

    def __init__(self, module, name: str, original):
        self.module, self.name, self.original = module, name, original

    def restore(self) -> None:
        setattr(self.module, self.name, self.original)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.restore()
        return False


def _sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, **kw):
    """torch's SDPA signature, for the arguments the engine passes (engine/fused.py:295); any other use
    is refused rather than computed differently."""
    if dropout_p or is_causal or scale is not None or kw:
        raise NotImplementedError("sokutou_b200 SDPA drop-in: only (q, k, v, attn_mask=...) as engine/fused.py:295 "
                                  "calls it")
    return ops.sdpa(query, key, value, attn_mask=attn_mask)


def install_sdpa(module, name: str = "F") -> SdpaPatch:
    """Make `module.<name>.scaled_dot_product_attention` (the engine's `F`) the library's DiT attention."""
    original = getattr(module, name)
    ns = types.SimpleNamespace(**{k: getattr(original, k) for k in dir(original) if not k.startswith("__")})
    ns.scaled_dot_product_attention = _sdpa
    setattr(module, name, ns)
    return SdpaPatch(module, name, original)


class DecodeAttnKernel:
    """Stands in for the reference's compiled `attn` kernel (qwen3/kernels.py:338-414) in its kernel dict."""

    def __init__(self, max_len: int, nq: int, nkv: int, cache_dtype: torch.dtype, device, hd: int = 128,
                 workspace: torch.Tensor | None = None):
        if cache_dtype not in (torch.bfloat16, torch.float32):
            raise TypeError("the cache is bfloat16 (wd bf16 / i8g32) or float32 (wd f32)")
        self.max_len, self.nq, self.nkv, self.hd = int(max_len), int(nq), int(nkv), int(hd)
        self.code = SK_BF16 if cache_dtype == torch.bfloat16 else SK_F32
        self.workspace = (workspace if workspace is not None
                          else ops.decode_workspace(max_len, nq, nkv, device, hd=hd, cache_dtype=cache_dtype))

    def __call__(self, grid, block, args, shared_mem: int = 0, **kw):
        """The reference's launch: grid (nkv,), block (256,) and shared_mem are its own kernel's and play
        no part here; args is the converted tuple of qwen3/kernels.py:622-624 (or :607-609)."""
        if len(args) != 13:
            raise TypeError(f"attn takes 13 arguments (qkv, qn, kn, eps, rope, Kc, Vc, pos_ptr, pos_add, max_len, nq, "
                            f"nkv, out), got {len(args)}")
        qkv, qn, kn, eps, rope, kc, vc, pos_ptr, pos_add, max_len, nq, nkv, out = args
        ws = self.workspace
        check(_lib.lib().sk_decode_attention(int(qkv), int(qn), int(kn), float(eps), int(rope), int(kc), int(vc),
                                             int(pos_ptr), int(pos_add), int(max_len), int(nq), int(nkv), self.hd,
                                             int(out), ws.data_ptr(), ws.numel() * ws.element_size(), self.code,
                                             torch.cuda.current_stream().cuda_stream),
              "sk_decode_attention")


def patch_kernels(engine, max_len: int, nq: int, nkv: int, cache_dtype: torch.dtype, device) -> DecodeAttnKernel:
    """Put a DecodeAttnKernel into `engine.k["attn"]` (Qwen3Kernels.__init__ builds that dict at
    qwen3/kernels.py:504); returns it. max_len: the talker's max_cache (the larger of the two stacks)."""
    kern = DecodeAttnKernel(max_len, nq, nkv, cache_dtype, device)
    engine.k["attn"] = kern
    return kern
