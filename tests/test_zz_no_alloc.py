"""sk_decode_attention_noalloc — the decode attention for callers that cannot allocate device memory
when they attend (a serving process that reserves its device memory at start-up, a foreign-language
binding that only passes buffers it owns). It keeps its split-KV scratch in a fixed array inside the
library instead of a caller workspace.

Checked through the C ABI against sk_decode_attention on identical inputs and against the float64
oracle, two calls in a row with different cache lengths (so the second call reuses the scratch the
first one left behind), within the decode tolerance of the other tests (relative L2 <= 1e-5). The
cache lengths are long enough that the split-KV path with the scratch runs (shorter caches are merged
inside one thread-block cluster and need no scratch at all). Also: the first call of a fresh process
made on a non-blocking stream (the scratch must be cleared before that call's kernel runs), the exact
size limit, and two calls captured into a CUDA graph after a warm-up call. Collected last so that a
failure here leaves every other test already run.
"""

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import decode_attn_ref as Q

pytestmark = pytest.mark.gpu

TOL = 1e-5
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


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


def _oracle(Kc, Vc, qkv, qn, kn, rope, T, nq, nkv, cache_dtype):
    """The float64 oracle on the caches as they were before the call (the oracle appends row T-1)."""
    Kn = Kc.float().cpu().numpy().astype(np.float64)
    Vn = Vc.float().cpu().numpy().astype(np.float64)
    return Q.decode_step(qkv.cpu().numpy(), qn.cpu().numpy(), kn.cpu().numpy(), 1e-6, rope.cpu().numpy(), Kn, Vn,
                         T - 1, nq, nkv, "bf16" if cache_dtype == torch.bfloat16 else "f32")


def _noalloc(lib, a, max_len, out, code, stream, nq=16, nkv=8):
    Kc, Vc, qkv, qn, kn, rope, pos = a
    return lib.sk_decode_attention_noalloc(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), ctypes.c_float(1e-6),
                                           rope.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), pos.data_ptr(), 0, max_len,
                                           nq, nkv, 128, out.data_ptr(), code, stream)


@pytest.mark.parametrize("cache_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_point_and_oracle(cuda, cache_dtype):
    from sokutou_b200 import _lib
    lib = _lib.lib()
    code = 0 if cache_dtype == torch.bfloat16 else 1
    stream = torch.cuda.current_stream().cuda_stream
    nq, nkv = 16, 8
    long_len = 6144 if cache_dtype == torch.bfloat16 else 3072
    for call, (max_len, T) in enumerate([(long_len, long_len - 100), (long_len - 256, 1500)]):
        a = _case(cuda, max_len, T, cache_dtype, seed=10 + call)
        Kc, Vc, qkv, qn, kn, rope, pos = a
        want = _oracle(Kc, Vc, qkv, qn, kn, rope, T, nq, nkv, cache_dtype)
        Kc2, Vc2 = Kc.clone(), Vc.clone()
        ref = torch.empty(nq * 128, device=cuda)
        ws = torch.zeros(lib.sk_decode_workspace_bytes(max_len, nq, nkv, 128, code), dtype=torch.uint8, device=cuda)
        rc = lib.sk_decode_attention(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), ctypes.c_float(1e-6),
                                     rope.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), pos.data_ptr(), 0, max_len, nq,
                                     nkv, 128, ref.data_ptr(), ws.data_ptr(), ws.numel(), code, stream)
        assert rc == 0
        out = torch.full((nq * 128,), float("nan"), device=cuda)
        assert _noalloc(lib, (Kc2, Vc2, qkv, qn, kn, rope, pos), max_len, out, code, stream) == 0
        torch.cuda.synchronize()
        assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) <= TOL
        assert rel_l2(out.cpu().numpy(), want) <= TOL
        assert torch.equal(Kc, Kc2) and torch.equal(Vc, Vc2)
    err = ctypes.c_int(-1)
    assert lib.sk_device_error(ctypes.byref(err), 1) == 0 and err.value == 0


def test_noalloc_size_limit_is_exact(cuda):
    """nkv * ceil(max_len / 64) * 1040 bytes of partials must fit 1 MiB - 4 KiB: at nkv = 8 the largest
    cache is 8000 positions (125 chunks); 8001 needs a 126th chunk and is refused before any launch."""
    from sokutou_b200 import _lib
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    nq, nkv, max_len, T = 16, 8, 8000, 8000
    a = _case(cuda, max_len, T, torch.bfloat16, seed=31)
    Kc, Vc, qkv, qn, kn, rope, pos = a
    want = _oracle(Kc, Vc, qkv, qn, kn, rope, T, nq, nkv, torch.bfloat16)
    out = torch.full((nq * 128,), float("nan"), device=cuda)
    assert _noalloc(lib, a, max_len, out, 0, stream) == 0
    torch.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), want) <= TOL
    dummy = torch.zeros(16, device=cuda)
    p = dummy.data_ptr()
    for too_long in (8001, 16384):
        rc = lib.sk_decode_attention_noalloc(p, p, p, ctypes.c_float(1e-6), p, p, p, None, 0, too_long, 16, 8, 128, p,
                                             0, stream)
        assert rc == -6


def test_noalloc_captured_in_a_graph(cuda):
    """After one warm-up call, two calls (different positions) captured into a CUDA graph and replayed
    give the workspace entry point's results."""
    from sokutou_b200 import _lib
    lib = _lib.lib()
    nq, nkv, max_len = 16, 8, 6144
    a = _case(cuda, max_len, 5000, torch.bfloat16, seed=41)
    Kc, Vc, qkv, qn, kn, rope, pos = a
    pos2 = torch.tensor([5999], dtype=torch.int64, device=cuda)
    out1 = torch.empty(nq * 128, device=cuda)
    out2 = torch.empty(nq * 128, device=cuda)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        assert _noalloc(lib, a, max_len, out1, 0, st.cuda_stream) == 0  # warm-up (also looks the scratch up)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    Kg, Vg = Kc.clone(), Vc.clone()  # the graph's own caches, as they were before the calls
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        s = torch.cuda.current_stream().cuda_stream
        assert _noalloc(lib, (Kg, Vg, qkv, qn, kn, rope, pos), max_len, out1, 0, s) == 0
        assert _noalloc(lib, (Kg, Vg, qkv, qn, kn, rope, pos2), max_len, out2, 0, s) == 0
    Kr, Vr = Kc.clone(), Vc.clone()  # the reference run starts from the same caches as the replay
    Kg.copy_(Kc)
    Vg.copy_(Vc)
    gr.replay()
    torch.cuda.synchronize()
    ws = torch.zeros(lib.sk_decode_workspace_bytes(max_len, nq, nkv, 128, 0), dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    for p_t, o_g in ((pos, out1), (pos2, out2)):
        ref = torch.empty(nq * 128, device=cuda)
        rc = lib.sk_decode_attention(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), ctypes.c_float(1e-6),
                                     rope.data_ptr(), Kr.data_ptr(), Vr.data_ptr(), p_t.data_ptr(), 0, max_len, nq,
                                     nkv, 128, ref.data_ptr(), ws.data_ptr(), ws.numel(), 0, stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert rel_l2(o_g.cpu().numpy(), ref.cpu().numpy()) <= TOL
    assert torch.equal(Kg, Kr) and torch.equal(Vg, Vr)
    del gr


_FRESH = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from oracle import decode_attn_ref as Q
from sokutou_b200 import _lib
lib = _lib.lib()
dev = torch.device("cuda:0")
nq, nkv, max_len, T = 16, 8, 6144, 6000
g = torch.Generator().manual_seed(51)
# this process's first noalloc call goes on a non-blocking stream, which the legacy default stream
# (where the library clears its scratch) does not order against
Kc = torch.randn(nkv, max_len, 128, generator=g).bfloat16().to(dev)
Vc = torch.randn(nkv, max_len, 128, generator=g).bfloat16().to(dev)
qkv = torch.randn((nq + 2 * nkv) * 128, generator=g).to(dev)
qn = (1 + 0.02 * torch.randn(128, generator=g)).to(dev)
kn = (1 + 0.02 * torch.randn(128, generator=g)).to(dev)
rope = torch.from_numpy(Q.rope_table(max_len)).to(dev)
pos = torch.tensor([T - 1], dtype=torch.int64, device=dev)
want = Q.decode_step(qkv.cpu().numpy(), qn.cpu().numpy(), kn.cpu().numpy(), 1e-6, rope.cpu().numpy(),
                     Kc.float().cpu().numpy().astype(np.float64), Vc.float().cpu().numpy().astype(np.float64),
                     T - 1, nq, nkv, "bf16")
torch.cuda.synchronize()
st = torch.cuda.Stream()  # non-blocking: not ordered against the legacy default stream
outs = []
for i in range(2):
    out = torch.full((nq * 128,), float("nan"), device=dev)
    with torch.cuda.stream(st):
        rc = lib.sk_decode_attention_noalloc(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), ctypes.c_float(1e-6),
                                             rope.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), pos.data_ptr(), 0, max_len,
                                             nq, nkv, 128, out.data_ptr(), 0, st.cuda_stream)
    assert rc == 0, rc
    outs.append(out)
st.synchronize()
for out in outs:
    o = out.cpu().numpy().astype(np.float64)
    r = float(np.linalg.norm(o - want) / np.linalg.norm(want))
    print("rel", r)
    assert r <= 1e-5, r
err = ctypes.c_int(-1)
assert lib.sk_device_error(ctypes.byref(err), 1) == 0 and err.value == 0, err.value
print("ok")
"""


def test_noalloc_first_call_of_a_process_on_a_non_blocking_stream(cuda):
    """A fresh process whose first noalloc call goes on a torch non-blocking stream: the scratch is
    cleared and the clear has finished before that call's kernel runs."""
    r = subprocess.run([sys.executable, "-c", _FRESH, ROOT], cwd=ROOT, capture_output=True, text=True, timeout=600)
    tail = "\n".join((r.stdout + r.stderr).strip().splitlines()[-10:])
    assert r.returncode == 0 and "ok" in r.stdout, tail
