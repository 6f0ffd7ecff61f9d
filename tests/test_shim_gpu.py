"""The drop-in shims on the B200, driven the way the reference engine drives its call sites: the DiT
attention through a module's swapped `F.scaled_dot_product_attention(q, k, v, attn_mask=bias)`
(engine/fused.py:295), and the talker / code-predictor decode through the kernel-dict call of
Qwen3Kernels._launch (qwen3/kernels.py:575-577, 622-624, 607-609) with its converted argument tuple.
Bars: the same bits as the library's own ops on the same inputs, and the float64 oracle's bars."""

import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from oracle import decode_attn_ref as Q
from sokutou_b200 import ops, shim

pytestmark = pytest.mark.gpu


def _ptr(t):
    """Qwen3Kernels' conversion of a launch argument (qwen3/kernels.py:418-422)."""
    return np.uintp(0) if t is None else np.uintp(t.data_ptr())


def test_sdpa_swap_in_a_module_gives_the_library_result(cuda):
    m = types.ModuleType("engine_fused_like")
    m.F = F

    def attend(q, k, v, bias):  # the call as engine/fused.py:295 writes it
        return m.F.scaled_dot_product_attention(q, k, v, attn_mask=bias)

    torch.manual_seed(0)
    B, H, L, K, hd = 3, 4, 130, 330, 64
    q = torch.randn(B, H, L, hd, device=cuda).bfloat16()
    k, v = (torch.randn(B, H, K, hd, device=cuda).bfloat16() for _ in range(2))
    bias = torch.zeros(B, 1, 1, K, device=cuda)
    bias[1, ..., 200:] = float("-inf")
    bias = bias.bfloat16()
    with shim.install_sdpa(m):
        y = attend(q, k, v, bias)
    assert m.F is F
    want = ops.sdpa(q, k, v, attn_mask=bias)
    torch.cuda.synchronize()
    assert torch.equal(y, want)
    assert y.transpose(1, 2).is_contiguous()  # what the engine's gate reads (engine/fused.py:296-298)
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=bias.float())
    assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("cdt", [torch.bfloat16, torch.float32])
def test_decode_kernel_dict_call(cuda, cdt):
    """Talker form (device position) and code-predictor form (pos_ptr None, pos_add = g) through the
    stand-in placed in a kernel dict, against ops.decode_attention on copies of the same caches."""
    g = torch.Generator().manual_seed(3)
    nq, nkv, hd, max_len, T = 16, 8, 128, 1536, 1120
    engine = types.SimpleNamespace(k={"attn": None})
    kern = shim.patch_kernels(engine, max_len, nq, nkv, cdt, cuda)
    assert engine.k["attn"] is kern
    rope = torch.from_numpy(Q.rope_table(max_len)).to(cuda)
    qkv = torch.randn((nq + 2 * nkv) * hd, generator=g).to(cuda)
    qn = (1 + 0.02 * torch.randn(hd, generator=g)).to(cuda)
    kn = (1 + 0.02 * torch.randn(hd, generator=g)).to(cuda)
    Kc = torch.randn(nkv, max_len, hd, generator=g).to(cdt).to(cuda)
    Vc = torch.randn(nkv, max_len, hd, generator=g).to(cdt).to(cuda)
    pos = torch.tensor([T - 1], dtype=torch.int64, device=cuda)
    for pos_ptr, pos_add, ml in ((pos, 0, max_len), (None, 9, 16)):
        K1, V1 = Kc[:, :ml].contiguous(), Vc[:, :ml].contiguous()
        K2, V2 = K1.clone(), V1.clone()
        out1 = torch.empty(nq * hd, device=cuda)
        out2 = torch.empty(nq * hd, device=cuda)
        eps = 1e-6
        args = (_ptr(qkv), _ptr(qn), _ptr(kn), np.float32(eps), _ptr(rope), _ptr(K1), _ptr(V1), _ptr(pos_ptr),
                np.int32(pos_add), np.int32(ml), np.int32(nq), np.int32(nkv), _ptr(out1))
        engine.k["attn"]((nkv,), (256,), args, shared_mem=2 * ml * 4)
        ws = ops.decode_workspace(ml, nq, nkv, cuda, cache_dtype=cdt)
        ops.decode_attention(qkv, qn, kn, eps, rope, K2, V2, pos_ptr, pos_add, ml, nq, nkv, out2, ws)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        assert torch.equal(out1, out2) and torch.equal(K1, K2) and torch.equal(V1, V2)
        p = (T - 1) if pos_ptr is not None else pos_add
        Kh = Kc[:, :ml].float().cpu().numpy().astype(np.float64)
        Vh = Vc[:, :ml].float().cpu().numpy().astype(np.float64)
        ref = Q.decode_step(qkv.cpu().numpy(), qn.cpu().numpy(), kn.cpu().numpy(), eps, rope.cpu().numpy(), Kh, Vh, p,
                            nq, nkv, "bf16" if cdt == torch.bfloat16 else "f32")
        tol = 1e-5 if cdt == torch.float32 else 1e-2
        assert rel_l2(out1.cpu().numpy().astype(np.float64), ref) <= tol
