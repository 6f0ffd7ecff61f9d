"""sk_decode_attention_grouped — R independent decode requests in one launch — through the C ABI
(ops.decode_attention_grouped): every request appends exactly the cache rows sk_decode_attention appends
on its own arguments and gives its output (bit for bit where sk_decode_attention also runs the cluster
kernel; to 1e-6 where it runs the split-KV workspace kernel, whose chunks sum in another order), and
matches the float64 oracle within the decode bars (fp32 caches relative L2 <= 1e-5, bf16 <= 1e-2).
Requests with different lengths in one launch, graph replay with positions read on the device, a
request whose position is out of range.
"""

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import decode_attn_ref as Q
from sokutou_b200 import ops

pytestmark = pytest.mark.gpu

FP32_TOL, BF16_TOL = 1e-5, 1e-2
NQ, NKV, HD = 16, 8, 128


def host(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _requests(dev, Ts, max_len, cdt, seed):
    g = torch.Generator().manual_seed(seed)
    rope = torch.from_numpy(Q.rope_table(max_len)).to(dev)
    out = []
    for T in Ts:
        r = {
            "qkv": torch.randn((NQ + 2 * NKV) * HD, generator=g).to(dev),
            "qn": (1 + 0.02 * torch.randn(HD, generator=g)).to(dev),
            "kn": (1 + 0.02 * torch.randn(HD, generator=g)).to(dev),
            "rope": rope,
            "Kc": torch.randn(NKV, max_len, HD, generator=g).to(cdt).to(dev),
            "Vc": torch.randn(NKV, max_len, HD, generator=g).to(cdt).to(dev),
            "pos_ptr": torch.tensor([T - 1], dtype=torch.int64, device=dev),
            "out": torch.full((NQ * HD,), float("nan"), device=dev),
            "pos_add": 0,
            "eps": 1e-6,
        }
        out.append(r)
    return out


def _single(r, max_len, cdt):
    """The same request through sk_decode_attention on copies of its caches."""
    K, V = r["Kc"].clone(), r["Vc"].clone()
    o = torch.empty(NQ * HD, device=K.device)
    ws = ops.decode_workspace(max_len, NQ, NKV, K.device, cache_dtype=cdt)
    ops.decode_attention(r["qkv"], r["qn"], r["kn"], r["eps"], r["rope"], K, V, r["pos_ptr"], r["pos_add"], max_len, NQ,
                         NKV, o, ws)
    return o, K, V


@pytest.mark.parametrize("cdt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("Ts", [[1120], [1, 64, 65, 700, 1500], [200 + 97 * i for i in range(12)]])
def test_grouped_matches_single_requests_and_oracle(cuda, cdt, Ts):
    max_len = 1536
    reqs = _requests(cuda, Ts, max_len, cdt, seed=len(Ts))
    want = [_single(r, max_len, cdt) for r in reqs]
    refs = []
    for r, T in zip(reqs, Ts):
        Kh, Vh = host(r["Kc"]), host(r["Vc"])
        refs.append(Q.decode_step(r["qkv"].cpu().numpy(), r["qn"].cpu().numpy(), r["kn"].cpu().numpy(), 1e-6,
                                  r["rope"].cpu().numpy(), Kh, Vh, T - 1, NQ, NKV,
                                  "bf16" if cdt == torch.bfloat16 else "f32"))
    dev_reqs = ops.decode_requests(reqs, cuda)
    ops.decode_attention_grouped(dev_reqs, len(reqs), max_len, NQ, NKV, cdt)
    torch.cuda.synchronize()
    tol = FP32_TOL if cdt == torch.float32 else BF16_TOL
    for r, (o, K, V), ref in zip(reqs, want, refs):
        assert rel_l2(host(r["out"]), host(o)) <= 1e-6
        assert torch.equal(r["Kc"], K) and torch.equal(r["Vc"], V)
        assert rel_l2(host(r["out"]), ref) <= tol
    assert ops.device_error() == 0


def test_grouped_graph_replay_reads_positions_on_device(cuda):
    """One captured launch for 6 requests plus their position advances, replayed for several steps: the
    same outputs and caches as the one-request launches step by step."""
    max_len, steps, cdt = 1024, 4, torch.bfloat16
    Ts = [300, 301, 512, 700, 900, 1000]
    reqs = _requests(cuda, Ts, max_len, cdt, seed=7)
    twins = [{k: (v.clone() if torch.is_tensor(v) and k in ("Kc", "Vc", "pos_ptr", "out") else v) for k, v in r.items()}
             for r in reqs]
    dev_reqs = ops.decode_requests(reqs, cuda)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):  # warm-up launch (the tensors are reset below)
        ops.decode_attention_grouped(dev_reqs, len(reqs), max_len, NQ, NKV, cdt)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    for r, t in zip(reqs, twins):
        r["Kc"].copy_(t["Kc"])
        r["Vc"].copy_(t["Vc"])
        r["pos_ptr"].copy_(t["pos_ptr"])
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        ops.decode_attention_grouped(dev_reqs, len(reqs), max_len, NQ, NKV, cdt)
        for r in reqs:
            r["pos_ptr"].add_(1)
    ws = ops.decode_workspace(max_len, NQ, NKV, cuda, cache_dtype=cdt)
    for _ in range(steps):
        gr.replay()
        for t in twins:
            ops.decode_attention(t["qkv"], t["qn"], t["kn"], 1e-6, t["rope"], t["Kc"], t["Vc"], t["pos_ptr"], 0,
                                 max_len, NQ, NKV, t["out"], ws)
            t["pos_ptr"].add_(1)
        torch.cuda.synchronize()
        for r, t in zip(reqs, twins):
            assert rel_l2(host(r["out"]), host(t["out"])) <= 1e-6
    for r, t in zip(reqs, twins):
        assert torch.equal(r["Kc"], t["Kc"]) and torch.equal(r["Vc"], t["Vc"])
        assert torch.equal(r["pos_ptr"], t["pos_ptr"])
    del gr
    assert ops.device_error() == 0


def test_grouped_request_out_of_range(cuda):
    """A request whose device position is past its cache records SK_DEVERR_POS_RANGE and writes nothing;
    the other requests of the launch are computed as usual."""
    max_len, cdt = 512, torch.bfloat16
    reqs = _requests(cuda, [100, 200, 300], max_len, cdt, seed=3)
    reqs[1]["pos_ptr"].fill_(max_len)
    K1, V1 = reqs[1]["Kc"].clone(), reqs[1]["Vc"].clone()
    want = [_single(r, max_len, cdt) if i != 1 else None for i, r in enumerate(reqs)]
    ops.device_error()  # the single-request references above also met the bad position: clear
    dev_reqs = ops.decode_requests(reqs, cuda)
    ops.decode_attention_grouped(dev_reqs, 3, max_len, NQ, NKV, cdt)
    torch.cuda.synchronize()
    assert ops.device_error() == 1
    assert torch.isnan(reqs[1]["out"]).all()
    assert torch.equal(reqs[1]["Kc"], K1) and torch.equal(reqs[1]["Vc"], V1)
    for i in (0, 2):
        assert rel_l2(host(reqs[i]["out"]), host(want[i][0])) <= 1e-6


def test_grouped_argument_errors(cuda):
    from sokutou_b200 import _lib
    lib = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    dummy = torch.zeros(64, dtype=torch.uint8, device=cuda)
    assert lib.sk_decode_attention_grouped(None, 1, 512, NQ, NKV, HD, 0, 0, st) == -1
    assert lib.sk_decode_attention_grouped(dummy.data_ptr(), 0, 512, NQ, NKV, HD, 0, 0, st) == -1
    assert lib.sk_decode_attention_grouped(dummy.data_ptr(), 1, 512, NQ, NKV, 64, 0, 0, st) == -2
    assert lib.sk_decode_attention_grouped(dummy.data_ptr(), 1, 8192, NQ, NKV, HD, 0, 0, st) == -2  # too long
