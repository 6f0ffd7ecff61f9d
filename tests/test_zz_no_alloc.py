"""sk_decode_attention_noalloc — the decode attention for callers that cannot allocate device memory
when they attend (a serving process that reserves its device memory at start-up, a driver inside a
CUDA graph capture, a foreign-language binding that only passes buffers it owns). It keeps its
split-KV scratch in a fixed array inside the library instead of a caller workspace.

Checked through the C ABI against sk_decode_attention on identical inputs, two calls in a row with
different cache lengths (so the second call reuses the scratch the first one left behind), within the
decode tolerance of the other tests (relative L2 <= 1e-5). The cache lengths are long enough that the
split-KV path with the scratch runs (shorter caches are merged inside one thread-block cluster and
need no scratch at all). Collected last so that a failure here
leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import decode_attn_ref as Q

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _case(dev, max_len, T, cache_dtype, seed, nq=16, nkv=8):
    g = torch.Generator().manual_seed(seed)
    Kc = torch.randn(nkv, max_len, 128, generator=g).to(cache_dtype).to(dev)
    Vc = torch.randn(nkv, max_len, 128, generator=g).to(cache_dtype).to(dev)
    qkv = torch.randn((nq + 2 * nkv) * 128, generator=g).to(dev)
    qn = (1 + 0.02 * torch.randn(128, generator=g)).to(dev)
    kn = (1 + 0.02 * torch.randn(128, generator=g)).to(dev)
    rope = torch.from_numpy(Q.rope_table(max_len)).to(dev)
    pos = torch.tensor([T - 1], dtype=torch.int64, device=dev)
    return Kc, Vc, qkv, qn, kn, rope, pos


@pytest.mark.parametrize("cache_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_point(cuda, cache_dtype):
    from sokutou_b200 import _lib
    lib = _lib.lib()
    code = 0 if cache_dtype == torch.bfloat16 else 1
    stream = torch.cuda.current_stream().cuda_stream
    nq, nkv = 16, 8
    long_len = 6144 if cache_dtype == torch.bfloat16 else 3072
    for call, (max_len, T) in enumerate([(long_len, long_len - 100), (long_len - 256, 1500)]):
        Kc, Vc, qkv, qn, kn, rope, pos = _case(cuda, max_len, T, cache_dtype, seed=10 + call)
        Kc2, Vc2 = Kc.clone(), Vc.clone()
        ref = torch.empty(nq * 128, device=cuda)
        ws = torch.zeros(lib.sk_decode_workspace_bytes(max_len, nq, nkv, 128, code), dtype=torch.uint8, device=cuda)
        rc = lib.sk_decode_attention(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), ctypes.c_float(1e-6),
                                     rope.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), pos.data_ptr(), 0, max_len, nq,
                                     nkv, 128, ref.data_ptr(), ws.data_ptr(), ws.numel(), code, stream)
        assert rc == 0
        out = torch.full((nq * 128,), float("nan"), device=cuda)
        rc = lib.sk_decode_attention_noalloc(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), ctypes.c_float(1e-6),
                                             rope.data_ptr(), Kc2.data_ptr(), Vc2.data_ptr(), pos.data_ptr(), 0,
                                             max_len, nq, nkv, 128, out.data_ptr(), code, stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) <= TOL
        assert torch.equal(Kc, Kc2) and torch.equal(Vc, Vc2)
    err = ctypes.c_int(-1)
    assert lib.sk_device_error(ctypes.byref(err), 1) == 0 and err.value == 0


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    from sokutou_b200 import _lib
    lib = _lib.lib()
    dummy = torch.zeros(16, device=cuda)
    p = dummy.data_ptr()
    # nkv = 8 with max_len 16384 needs ~2 MiB of partials: refused before any launch
    rc = lib.sk_decode_attention_noalloc(p, p, p, ctypes.c_float(1e-6), p, p, p, None, 0, 16384, 16, 8, 128, p, 0,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == -6
