"""sk_decode_attention_block — one talker layer's rms_gemv(qkv) -> attention -> gemv(o) (the three
launches of qwen3/kernels.py:619-624) in one launch — against the float64 oracle's decode_block, through
the C ABI (ops.decode_attention_block). Bars as the decode tests: fp32 caches and weights relative L2
<= 1e-5, bf16 <= 1e-2 (both far looser than what the kernel reaches: fp32 accumulation throughout, the
cache's bf16 rounding mirrored by the oracle). Also: the appended cache rows, graph replay reading the
position on the device, the same bits as the plain launch when the launch is flagged KV-stable, the
full c3 greedy decode run through the block kernel (every token equal to the oracle's), argument errors.
"""

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import decode_attn_ref as Q
from sokutou_b200 import ops, qwen3, workloads as W

pytestmark = pytest.mark.gpu

FP32_TOL, BF16_TOL = 1e-5, 1e-2


def host(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _case(dev, hidden, max_len, T, wdt, cdt, seed, nq=16, nkv=8, hd=128):
    g = torch.Generator().manual_seed(seed)
    Dq = (nq + 2 * nkv) * hd
    x = {
        "h": torch.randn(hidden, generator=g),
        "in_norm": 1 + 0.1 * torch.randn(hidden, generator=g),
        "w_qkv": (torch.randn(Dq, hidden, generator=g) / hidden ** 0.5).to(wdt),
        "w_o": (torch.randn(hidden, nq * hd, generator=g) / (nq * hd) ** 0.5).to(wdt),
        "qn": 1 + 0.02 * torch.randn(hd, generator=g),
        "kn": 1 + 0.02 * torch.randn(hd, generator=g),
        "Kc": torch.randn(nkv, max_len, hd, generator=g).to(cdt),
        "Vc": torch.randn(nkv, max_len, hd, generator=g).to(cdt),
    }
    d = {k: v.to(dev).contiguous() for k, v in x.items()}
    d["rope"] = torch.from_numpy(Q.rope_table(max_len)).to(dev)
    d["pos"] = torch.tensor([T - 1], dtype=torch.int64, device=dev)
    return d


def _oracle(d, T, cdt, nq=16, nkv=8, eps=1e-6, eps_in=1e-6):
    Kh, Vh = host(d["Kc"]), host(d["Vc"])
    h = Q.decode_block(host(d["h"]), host(d["in_norm"]), eps_in, host(d["w_qkv"]), host(d["qn"]), host(d["kn"]), eps,
                       d["rope"].cpu().numpy(), Kh, Vh, T - 1, nq, nkv, host(d["w_o"]),
                       "bf16" if cdt == torch.bfloat16 else "f32")
    return h, Kh, Vh


def _run(d, max_len, ws=None, pos_add=0, kv_stable=False, nq=16, nkv=8):
    ws = ws if ws is not None else ops.decode_block_workspace(max_len, nq, nkv, d["h"].device)
    ops.decode_attention_block(d["h"], d["in_norm"], 1e-6, d["w_qkv"], d["qn"], d["kn"], 1e-6, d["rope"], d["Kc"],
                               d["Vc"], d["pos"], pos_add, max_len, nq, nkv, d["w_o"], ws, kv_stable)
    return ws


@pytest.mark.parametrize("wdt,cdt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                     (torch.bfloat16, torch.float32), (torch.float32, torch.bfloat16)])
@pytest.mark.parametrize("hidden,T", [(256, 1), (256, 65), (2048, 1120), (1024, 1500), (2048, 64)])
def test_block_matches_oracle(cuda, wdt, cdt, hidden, T):
    max_len = 1536
    d = _case(cuda, hidden, max_len, T, wdt, cdt, seed=T + hidden)
    want, Kh, Vh = _oracle(d, T, cdt)
    _run(d, max_len)
    torch.cuda.synchronize()
    tol = FP32_TOL if (wdt, cdt) == (torch.float32, torch.float32) else BF16_TOL
    err = rel_l2(host(d["h"]), want)
    assert err <= tol, err
    # every row but the appended one is untouched; the appended one is what the oracle stores, to the
    # precision of the qkv projection (fp32 in the kernel, float64 in the oracle) and the cache's rounding
    Ka, Va = host(d["Kc"]), host(d["Vc"])
    rows = [r for r in range(max_len) if r != T - 1]
    np.testing.assert_array_equal(Ka[:, rows], Kh[:, rows])
    np.testing.assert_array_equal(Va[:, rows], Vh[:, rows])
    row_tol = FP32_TOL if cdt == torch.float32 else BF16_TOL
    assert rel_l2(Ka[:, T - 1], Kh[:, T - 1]) <= row_tol
    assert rel_l2(Va[:, T - 1], Vh[:, T - 1]) <= row_tol
    assert ops.device_error() == 0


def test_block_matches_separate_launches(cuda):
    """The block gives what the three separate steps give (torch fp32 projections around
    sk_decode_attention), fp32 weights and caches."""
    max_len, T, hidden, nq, nkv = 1536, 700, 2048, 16, 8
    d = _case(cuda, hidden, max_len, T, torch.float32, torch.float32, seed=5)
    K2, V2 = d["Kc"].clone(), d["Vc"].clone()
    h = d["h"].clone()
    xs = h * d["in_norm"] * torch.rsqrt((h * h).mean() + 1e-6)
    qkv = (d["w_qkv"] @ xs).contiguous()
    att = torch.empty(nq * 128, device=cuda)
    ws = ops.decode_workspace(max_len, nq, nkv, cuda, cache_dtype=torch.float32)
    ops.decode_attention(qkv, d["qn"], d["kn"], 1e-6, d["rope"], K2, V2, d["pos"], 0, max_len, nq, nkv, att, ws)
    h_sep = h + d["w_o"] @ att
    _run(d, max_len)
    torch.cuda.synchronize()
    assert rel_l2(host(d["h"]), host(h_sep)) <= FP32_TOL
    # the caches agree everywhere but the appended row, which comes from two different fp32 projections
    rows = [r for r in range(max_len) if r != T - 1]
    assert torch.equal(d["Kc"][:, rows], K2[:, rows]) and torch.equal(d["Vc"][:, rows], V2[:, rows])
    assert rel_l2(host(d["Kc"][:, T - 1]), host(K2[:, T - 1])) <= FP32_TOL
    assert rel_l2(host(d["Vc"][:, T - 1]), host(V2[:, T - 1])) <= FP32_TOL


def test_block_graph_replay_and_kv_stable_bits(cuda):
    """A 4-layer stack of blocks plus the position advance captured once and replayed for several steps:
    the same bits as eager launches; layers 1-3 flagged KV-stable change nothing."""
    s = W.C3
    n_layers, max_len, hidden, steps = 4, 512, 2048, 5
    g = torch.Generator(device=cuda).manual_seed(3)
    Dq = (s.nq + 2 * s.nkv) * s.hd
    wq = (torch.randn(n_layers, Dq, hidden, device=cuda, generator=g) / hidden ** 0.5).bfloat16()
    wo = (torch.randn(n_layers, hidden, s.nq * s.hd, device=cuda, generator=g) / 2048 ** 0.5).bfloat16()
    nw = 1 + 0.1 * torch.randn(n_layers, hidden, device=cuda, generator=g)
    qn = 1 + 0.02 * torch.randn(n_layers, s.hd, device=cuda, generator=g)
    kn = 1 + 0.02 * torch.randn(n_layers, s.hd, device=cuda, generator=g)
    h0 = torch.randn(hidden, device=cuda, generator=g)
    res = {}
    for mode in ("eager", "graph", "graph_stable"):
        ta = qwen3.TalkerAttention(n_layers, s.nq, s.nkv, max_len, s.theta, s.eps, cuda, torch.bfloat16)
        ta.k.copy_(torch.randn(ta.k.shape, device=cuda, generator=torch.Generator(device=cuda).manual_seed(9)))
        ta.v.copy_(torch.randn(ta.v.shape, device=cuda, generator=torch.Generator(device=cuda).manual_seed(10)))
        ta.pos.fill_(200)
        h = h0.clone()
        outs = []

        def step():
            for li in range(n_layers):
                ta.block(li, h, nw[li], 1e-6, wq[li], qn[li], kn[li], wo[li], kv_stable=(mode == "graph_stable" and li > 0))
            ta.pos.add_(1)

        if mode == "eager":
            for _ in range(steps):
                step()
                outs.append(h.clone())
        else:
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                step()  # warm-up step (position 200), then the state is reset
            torch.cuda.current_stream().wait_stream(st)
            ta.k.copy_(torch.randn(ta.k.shape, device=cuda, generator=torch.Generator(device=cuda).manual_seed(9)))
            ta.v.copy_(torch.randn(ta.v.shape, device=cuda, generator=torch.Generator(device=cuda).manual_seed(10)))
            ta.pos.fill_(200)
            h.copy_(h0)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step()
            for _ in range(steps):
                gr.replay()
                outs.append(h.clone())
            del gr
        torch.cuda.synchronize()
        res[mode] = (torch.stack(outs), ta.k.clone(), ta.v.clone(), int(ta.pos.item()))
    for mode in ("graph", "graph_stable"):
        assert torch.equal(res[mode][0], res["eager"][0]), mode
        assert torch.equal(res[mode][1], res["eager"][1]) and torch.equal(res[mode][2], res["eager"][2]), mode
        assert res[mode][3] == res["eager"][3] == 200 + steps
    assert ops.device_error() == 0


def test_c3_greedy_tokens_through_the_block_fp32(cuda):
    """The full c3 decode (28 layers, 96-token prompt, decode to T = 1120) with every layer's attention
    block as one launch (fp32 weights and caches): every greedy token equals the float64 oracle's."""
    s = W.C3
    talker = W.SyntheticTalker(s, seed=0)
    n_new = s.T_final - s.prompt
    toks, _ = talker.generate(cuda, n_new, cache_dtype=torch.float32, fused=True)
    ref = Q.talker_greedy(talker.numpy_weights(), s.n_layers, s.nq, s.nkv, s.hd, s.prompt + n_new, s.prompt, n_new,
                          s.eps, Q.rope_table(s.prompt + n_new), "f32")
    assert len(toks) == len(ref) == n_new + 1
    first = next((i for i, (a, b) in enumerate(zip(toks, ref)) if a != b), None)
    assert first is None, f"first differing token at {first}"
    assert ops.device_error() == 0


def test_block_errors(cuda):
    from sokutou_b200 import _lib
    max_len, T = 256, 10
    d = _case(cuda, 256, max_len, T, torch.bfloat16, torch.bfloat16, seed=1)
    ws = ops.decode_block_workspace(max_len, 16, 8, cuda)
    small = torch.zeros(64, dtype=torch.uint8, device=cuda)
    with pytest.raises(_lib.SokutouError, match="WORKSPACE"):
        _run(d, max_len, ws=small)
    # a position read on the device outside the cache: error word, nothing written
    K0, V0, h0 = d["Kc"].clone(), d["Vc"].clone(), d["h"].clone()
    d["pos"].fill_(max_len)
    _run(d, max_len, ws=ws)
    assert ops.device_error() == 1
    assert torch.equal(d["Kc"], K0) and torch.equal(d["Vc"], V0) and torch.equal(d["h"], h0)
    # the workspace is still usable after that early exit
    d["pos"].fill_(T - 1)
    want, _, _ = _oracle(d, T, torch.bfloat16)
    _run(d, max_len, ws=ws)
    torch.cuda.synchronize()
    assert rel_l2(host(d["h"]), want) <= BF16_TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("wdt,cdt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16)])
def test_code_predictor_form_positions_from_pos_add(cuda, wdt, cdt):
    """The code predictor's call form (qwen3/kernels.py:600-617, `_layers(C, ..., pos_ptr=None,
    pos_add=g)`): no device position, the write index is pos_add itself, a 16-row cache
    (max_len = G = 16) filled position by position 0..15, a 1024-wide hidden state. Every step against the
    float64 oracle, which appends to its own copy of the caches."""
    max_len, hidden = 16, 1024
    d = _case(cuda, hidden, max_len, 1, wdt, cdt, seed=31)
    d["Kc"].zero_()
    d["Vc"].zero_()
    Kh, Vh = host(d["Kc"]), host(d["Vc"])
    ws = ops.decode_block_workspace(max_len, 16, 8, cuda)
    tol = FP32_TOL if (wdt, cdt) == (torch.float32, torch.float32) else BF16_TOL
    for g in range(max_len):
        want = Q.decode_block(host(d["h"]), host(d["in_norm"]), 1e-6, host(d["w_qkv"]), host(d["qn"]), host(d["kn"]),
                              1e-6, d["rope"].cpu().numpy(), Kh, Vh, g, 16, 8, host(d["w_o"]),
                              "bf16" if cdt == torch.bfloat16 else "f32")
        ops.decode_attention_block(d["h"], d["in_norm"], 1e-6, d["w_qkv"], d["qn"], d["kn"], 1e-6, d["rope"], d["Kc"],
                                   d["Vc"], None, g, max_len, 16, 8, d["w_o"], ws)
        torch.cuda.synchronize()
        assert rel_l2(host(d["h"]), want) <= tol, g
        # the next step starts from the same state on both sides: the oracle's h, the kernel's appended
        # rows (they differ from the oracle's by the fp32 rounding of the projection)
        d["h"].copy_(torch.from_numpy(want).float())
        Kh[:, g], Vh[:, g] = host(d["Kc"])[:, g], host(d["Vc"])[:, g]
    assert ops.device_error() == 0


@pytest.mark.parametrize("wdt,cdt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16)])
def test_code_predictor_pair_as_two_launches(cuda, wdt, cdt):
    """The code predictor's paired pass (qwen3/kernels.py:600-617: both rows projected, then attention at
    position 0 and at position 1, then the o projection of both rows) is the same arithmetic as two block
    launches in a row — row 0 at pos_add 0, then row 1 at pos_add 1 — because row 1's projection reads
    only its own residual row: against the oracle's restatement of the paired pass, with each row's h
    and the two appended cache rows."""
    max_len, hidden = 16, 1024
    d = _case(cuda, hidden, max_len, 1, wdt, cdt, seed=47)
    d["Kc"].zero_()
    d["Vc"].zero_()
    g = torch.Generator().manual_seed(48)
    h2 = torch.randn(2, hidden, generator=g).to(cuda)
    Kh, Vh = host(d["Kc"]), host(d["Vc"])
    want = Q.decode_block_pair(host(h2), host(d["in_norm"]), 1e-6, host(d["w_qkv"]), host(d["qn"]), host(d["kn"]),
                               1e-6, d["rope"].cpu().numpy(), Kh, Vh, 16, 8, host(d["w_o"]),
                               "bf16" if cdt == torch.bfloat16 else "f32")
    ws = ops.decode_block_workspace(max_len, 16, 8, cuda)
    rows = [h2[0].clone(), h2[1].clone()]
    for r in (0, 1):
        ops.decode_attention_block(rows[r], d["in_norm"], 1e-6, d["w_qkv"], d["qn"], d["kn"], 1e-6, d["rope"], d["Kc"],
                                   d["Vc"], None, r, max_len, 16, 8, d["w_o"], ws)
    torch.cuda.synchronize()
    tol = FP32_TOL if (wdt, cdt) == (torch.float32, torch.float32) else BF16_TOL
    for r in (0, 1):
        assert rel_l2(host(rows[r]), want[r]) <= tol, r
        assert rel_l2(host(d["Kc"])[:, r], Kh[:, r]) <= tol and rel_l2(host(d["Vc"])[:, r], Vh[:, r]) <= tol
    assert torch.all(d["Kc"][:, 2:] == 0) and torch.all(d["Vc"][:, 2:] == 0)
    assert ops.device_error() == 0
