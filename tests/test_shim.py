"""The drop-in shims on the host: the SDPA swap in a module's `F` (engine/fused.py:29,295) and the
argument forwarding of the `attn` stand-in called as the reference's kernel dict calls its kernels
(qwen3/kernels.py:575-577, 622-624) — against a fake of the C library, so no GPU is needed."""

import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from sokutou_b200 import _lib, shim


def test_install_sdpa_swaps_only_sdpa_and_restores():
    m = types.ModuleType("fake_engine_fused")
    m.F = F
    with shim.install_sdpa(m) as patch:
        assert m.F is not F
        assert m.F.scaled_dot_product_attention is shim._sdpa
        assert m.F.linear is F.linear and m.F.silu is F.silu
        with pytest.raises(NotImplementedError):
            m.F.scaled_dot_product_attention(None, None, None, is_causal=True)
        with pytest.raises(NotImplementedError):
            m.F.scaled_dot_product_attention(None, None, None, dropout_p=0.1)
    assert m.F is F
    patch.restore()  # idempotent
    assert m.F is F


class _FakeLib:
    def __init__(self):
        self.calls = []

    def sk_decode_attention(self, *args):
        self.calls.append(args)
        return 0


def test_decode_attn_kernel_forwards_the_reference_arguments(monkeypatch):
    fake = _FakeLib()
    monkeypatch.setattr(_lib, "lib", lambda: fake)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: types.SimpleNamespace(cuda_stream=1234))
    ws = torch.zeros(4096, dtype=torch.uint8)
    kern = shim.DecodeAttnKernel(1536, 16, 8, torch.bfloat16, "cpu", workspace=ws)
    # the tuple as Qwen3Kernels._launch builds it: np.uintp addresses (0 for pos_ptr=None), numpy scalars
    args = (np.uintp(0x1000), np.uintp(0x2000), np.uintp(0x3000), np.float32(1e-6), np.uintp(0x4000),
            np.uintp(0x5000), np.uintp(0x6000), np.uintp(0), np.int32(3), np.int32(16), np.int32(16), np.int32(8),
            np.uintp(0x7000))
    kern((8,), (256,), args, shared_mem=2 * 16 * 4)
    (got,) = fake.calls
    assert got[:8] == (0x1000, 0x2000, 0x3000, pytest.approx(1e-6), 0x4000, 0x5000, 0x6000, 0)
    assert got[8:14] == (3, 16, 16, 8, 128, 0x7000)
    assert got[14] == ws.data_ptr() and got[15] == 4096 and got[16] == _lib.SK_BF16 and got[17] == 1234
    with pytest.raises(TypeError):
        kern((8,), (256,), args[:12])
    fake_f32 = shim.DecodeAttnKernel(16, 16, 8, torch.float32, "cpu", workspace=ws)
    fake_f32((8,), (256,), args)
    assert fake.calls[-1][16] == _lib.SK_F32


def test_decode_attn_kernel_raises_on_error_status(monkeypatch):
    fake = _FakeLib()
    fake.sk_decode_attention = lambda *a: -5
    monkeypatch.setattr(_lib, "lib", lambda: fake)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: types.SimpleNamespace(cuda_stream=0))
    kern = shim.DecodeAttnKernel(64, 16, 8, torch.bfloat16, "cpu", workspace=torch.zeros(16, dtype=torch.uint8))
    with pytest.raises(_lib.SokutouError, match="WORKSPACE"):
        kern((8,), (256,), tuple([np.uintp(1)] * 3 + [np.float32(1e-6)] + [np.uintp(1)] * 4 + [np.int32(0)] * 4 +
                                 [np.uintp(1)]))
