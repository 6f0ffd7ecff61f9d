"""Qwen3 talker decode attention on the B200 against the CPU oracle and the transformers-made golden
vectors.

Tolerances: per-layer output relative L2 <= 1e-5 in fp32 mode (fp32 cache) and <= 1e-2 in bf16
(the kernel computes in fp32 over the bf16 cache exactly like the reference, so bf16 lands near
1e-6 as well); greedy tokens of the full c3 decode identical to the oracle's in fp32 mode.
The appended cache row: exact for V; K within one bf16 ulp (rsqrtf vs exact rsqrt can move a
rounding boundary).
"""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2
from oracle import decode_attn_ref as Q
from sokutou_b200 import ops, qwen3, workloads as W

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
BF16_TOL = 1e-2
CDT = {"bf16": torch.bfloat16, "f32": torch.float32}


def host(t):
    return t.float().cpu().numpy()


def _golden_cache(g, d):
    if str(g["cache"]) == "bf16":
        mk = lambda a: torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).to(d).contiguous()
    else:
        mk = lambda a: torch.from_numpy(a.copy()).to(d).contiguous()
    return mk(g["Kc0"]), mk(g["Vc0"])


@pytest.mark.parametrize("case", ["decode_bf16", "decode_f32", "decode_cp"])
def test_golden(cuda, case):
    g = load_golden(case)
    nq, nkv, pos, max_len = int(g["nq"]), int(g["nkv"]), int(g["pos"]), int(g["max_len"])
    Kc, Vc = _golden_cache(g, cuda)
    f = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(cuda).contiguous()
    out = torch.empty(nq * 128, device=cuda)
    ws = ops.decode_workspace(max_len, nq, nkv, cuda, cache_dtype=Kc.dtype)
    if case == "decode_cp":  # code-predictor form: no position tensor, pos = pos_add
        ops.decode_attention(f(g["qkv"]), f(g["qn"]), f(g["kn"]), float(g["eps"]), f(g["rope"]), Kc, Vc, None, pos,
                             max_len, nq, nkv, out, ws)
    else:
        p = torch.tensor([pos], device=cuda, dtype=torch.int64)
        ops.decode_attention(f(g["qkv"]), f(g["qn"]), f(g["kn"]), float(g["eps"]), f(g["rope"]), Kc, Vc, p, 0,
                             max_len, nq, nkv, out, ws)
    torch.cuda.synchronize()
    assert rel_l2(host(out), g["out"]) < FP32_TOL
    assert np.array_equal(host(Vc[:, pos]), g["v_row"])
    kd = np.abs(host(Kc[:, pos]) - g["k_row"])
    assert np.all(kd <= np.abs(g["k_row"]) * 2 ** -7 + 1e-30)
    assert ops.device_error() == 0


def _random_case(cuda, T, max_len, cache, seed, nq=16, nkv=8):
    rng = np.random.default_rng(seed)
    hd = 128
    cdt = CDT[cache]
    Kc = torch.randn(nkv, max_len, hd, generator=torch.Generator().manual_seed(seed)).to(cdt).to(cuda)
    Vc = torch.randn(nkv, max_len, hd, generator=torch.Generator().manual_seed(seed + 1)).to(cdt).to(cuda)
    qkv = rng.standard_normal((nq + 2 * nkv) * hd).astype(np.float32)
    qn = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    rope = Q.rope_table(max_len)
    return Kc, Vc, qkv, qn, kn, rope


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 128, 500, 1024, 1120, 1500])
@pytest.mark.parametrize("cache", ["bf16", "f32"])
def test_against_oracle(cuda, T, cache):
    max_len = 1536
    nq, nkv = 16, 8
    Kc, Vc, qkv, qn, kn, rope = _random_case(cuda, T, max_len, cache, seed=T)
    Kh, Vh = host(Kc).astype(np.float64), host(Vc).astype(np.float64)
    ref = Q.decode_step(qkv, qn, kn, 1e-6, rope, Kh, Vh, T - 1, nq, nkv, cache)
    f = lambda a: torch.from_numpy(a).to(cuda).contiguous()
    out = torch.empty(nq * 128, device=cuda)
    ws = ops.decode_workspace(max_len, nq, nkv, cuda, cache_dtype=Kc.dtype)
    pos = torch.tensor([T - 1], device=cuda, dtype=torch.int64)
    ops.decode_attention(f(qkv), f(qn), f(kn), 1e-6, f(rope), Kc, Vc, pos, 0, max_len, nq, nkv, out, ws)
    torch.cuda.synchronize()
    assert rel_l2(host(out), ref) < (FP32_TOL if cache == "f32" else BF16_TOL)
    assert np.array_equal(host(Vc[:, T - 1]), Vh[:, T - 1])
    # only position T-1 of the cache changed
    Kc2, Vc2, *_ = _random_case(cuda, T, max_len, cache, seed=T)
    mask = torch.ones(max_len, dtype=torch.bool)
    mask[T - 1] = False
    assert torch.equal(Kc[:, mask], Kc2[:, mask]) and torch.equal(Vc[:, mask], Vc2[:, mask])
    assert ops.device_error() == 0


@pytest.mark.parametrize("cache", ["bf16", "f32"])
def test_long_cache_uses_workspace_kernel(cuda, cache):
    """max_len beyond one cluster's shared memory: the split-KV workspace kernel takes the call."""
    max_len = 6144 if cache == "bf16" else 3072
    T = max_len - 7
    nq, nkv = 16, 8
    Kc, Vc, qkv, qn, kn, rope = _random_case(cuda, T, max_len, cache, seed=99)
    Kh, Vh = host(Kc).astype(np.float64), host(Vc).astype(np.float64)
    ref = Q.decode_step(qkv, qn, kn, 1e-6, rope, Kh, Vh, T - 1, nq, nkv, cache)
    f = lambda a: torch.from_numpy(a).to(cuda).contiguous()
    out = torch.empty(nq * 128, device=cuda)
    ws = ops.decode_workspace(max_len, nq, nkv, cuda, cache_dtype=Kc.dtype)
    pos = torch.tensor([T - 1], device=cuda, dtype=torch.int64)
    for _ in range(2):  # the merge counters are back at zero for the second call
        ops.decode_attention(f(qkv), f(qn), f(kn), 1e-6, f(rope), Kc, Vc, pos, 0, max_len, nq, nkv, out, ws)
        torch.cuda.synchronize()
        assert rel_l2(host(out), ref) < (FP32_TOL if cache == "f32" else BF16_TOL)
    assert ops.device_error() == 0


def test_workspace_counters_return_to_zero(cuda):
    max_len, nq, nkv = 1536, 16, 8
    Kc, Vc, qkv, qn, kn, rope = _random_case(cuda, 1000, max_len, "bf16", seed=1)
    f = lambda a: torch.from_numpy(a).to(cuda).contiguous()
    ws = ops.decode_workspace(max_len, nq, nkv, cuda)
    out = torch.empty(nq * 128, device=cuda)
    pos = torch.tensor([999], device=cuda, dtype=torch.int64)
    outs = []
    for _ in range(3):
        ops.decode_attention(f(qkv), f(qn), f(kn), 1e-6, f(rope), Kc, Vc, pos, 0, max_len, nq, nkv, out, ws)
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    nsplit = (max_len + 63) // 64
    cnt_off = nkv * nsplit * 2 * 128 * 4 + nkv * nsplit * 2 * 2 * 4
    assert int(ws[cnt_off:cnt_off + 4 * nkv].view(torch.int32).abs().sum()) == 0


def test_position_out_of_range_reports_error(cuda):
    """pos_ptr[0] beyond the cache: the kernel writes nothing and records SK_DEVERR_POS_RANGE."""
    max_len, nq, nkv = 128, 16, 8
    Kc, Vc, qkv, qn, kn, rope = _random_case(cuda, 10, max_len, "bf16", seed=2)
    K0, V0 = Kc.clone(), Vc.clone()
    f = lambda a: torch.from_numpy(a).to(cuda).contiguous()
    ws = ops.decode_workspace(max_len, nq, nkv, cuda)
    out = torch.full((nq * 128,), 5.0, device=cuda)
    assert ops.device_error() == 0
    pos = torch.tensor([max_len], device=cuda, dtype=torch.int64)
    ops.decode_attention(f(qkv), f(qn), f(kn), 1e-6, f(rope), Kc, Vc, pos, 0, max_len, nq, nkv, out, ws)
    assert ops.device_error(reset=True) == 1
    assert torch.equal(Kc, K0) and torch.equal(Vc, V0) and torch.all(out == 5.0)
    assert ops.device_error() == 0


def test_graph_replay_reads_position_on_device(cuda):
    """One captured launch serves every step: the position advances on the device between replays."""
    max_len, nq, nkv = 256, 16, 8
    Kc, Vc, qkv, qn, kn, rope = _random_case(cuda, 1, max_len, "f32", seed=4)
    Kh, Vh = host(Kc).astype(np.float64), host(Vc).astype(np.float64)
    f = lambda a: torch.from_numpy(a).to(cuda).contiguous()
    qkv_d, qn_d, kn_d, rope_d = f(qkv), f(qn), f(kn), f(rope)
    ws = ops.decode_workspace(max_len, nq, nkv, cuda, cache_dtype=torch.float32)
    out = torch.empty(nq * 128, device=cuda)
    pos = torch.tensor([100], device=cuda, dtype=torch.int64)
    run = lambda: ops.decode_attention(qkv_d, qn_d, kn_d, 1e-6, rope_d, Kc, Vc, pos, 0, max_len, nq, nkv, out, ws)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()  # warm-up writes position 100
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
        pos.add_(1)
    Q.decode_step(qkv, qn, kn, 1e-6, rope, Kh, Vh, 100, nq, nkv, "f32")
    pos.fill_(101)
    for p in (101, 102, 103):
        g.replay()
        ref = Q.decode_step(qkv, qn, kn, 1e-6, rope, Kh, Vh, p, nq, nkv, "f32")
        torch.cuda.synchronize()
        assert rel_l2(host(out), ref) < FP32_TOL
    assert int(pos.item()) == 104


def test_c3_greedy_tokens_bit_exact_fp32(cuda):
    """Full c3 decode (28 layers, 96-token prompt, decode to T=1120) in fp32 mode: every greedy token
    equals the float64 oracle's."""
    s = W.C3
    talker = W.SyntheticTalker(s, seed=0)
    n_new = s.T_final - s.prompt
    toks, _ = talker.generate(cuda, n_new, cache_dtype=torch.float32)
    ref = Q.talker_greedy(talker.numpy_weights(), s.n_layers, s.nq, s.nkv, s.hd, s.prompt + n_new, s.prompt, n_new,
                          s.eps, Q.rope_table(s.prompt + n_new), "f32")
    assert len(toks) == len(ref) == n_new + 1
    first = next((i for i, (a, b) in enumerate(zip(toks, ref)) if a != b), None)
    assert first is None, f"first differing token at {first}"
    assert len(set(toks)) > 10  # the chain is not stuck on one token
    assert ops.device_error() == 0


def test_bf16_layer_outputs_teacher_forced(cuda):
    """bf16 cache: a short stack decode compared layer by layer with the oracle fed the same qkv."""
    s = W.DecodeShape(n_layers=4, prompt=8, T_final=200)
    talker = W.SyntheticTalker(s, seed=1)
    w = {k: v.to(cuda) for k, v in talker.w.items()}
    ta = qwen3.TalkerAttention(s.n_layers, s.nq, s.nkv, s.T_final, s.theta, s.eps, cuda, torch.bfloat16)
    rope = host(ta.rope)
    Kh = np.zeros((s.n_layers, s.nkv, s.T_final, s.hd))
    Vh = np.zeros_like(Kh)
    att = torch.empty(s.nq * s.hd, device=cuda)
    worst = 0.0
    for pos in range(s.T_final):
        h = w["prompt"][pos % s.prompt]
        for li in range(s.n_layers):
            qkv = (w["w_qkv"][li] @ (h * torch.rsqrt((h * h).mean() + s.eps))).contiguous()
            ta.attn(li, qkv, w["qn"][li], w["kn"][li], att)
            ref = Q.decode_step(host(qkv), host(w["qn"][li]), host(w["kn"][li]), s.eps, rope, Kh[li], Vh[li], pos,
                                s.nq, s.nkv, "bf16")
            worst = max(worst, rel_l2(host(att), ref))
            h = h + w["w_o"][li] @ att
        ta.pos.add_(1)
    assert worst < BF16_TOL


@pytest.mark.parametrize("cache", ["bf16", "f32"])
def test_kv_stable_launch_gives_same_bits(cuda, cache):
    """SK_DECODE_KV_STABLE only moves the position read and the cache copies before the wait for the
    previous kernel: a graph-replayed 4-layer stack (layer 0 after the position advance, the others
    flagged) must give the same outputs and caches, bit for bit, as the plain launches."""
    s = W.C3
    n_layers, max_len, steps = 4, 512, 6
    res = {}
    for flagged in (False, True):
        g = torch.Generator(device=cuda).manual_seed(11)
        ta = qwen3.TalkerAttention(n_layers, s.nq, s.nkv, max_len, s.theta, s.eps, cuda, CDT[cache])
        ta.k.copy_(torch.randn(ta.k.shape, device=cuda, generator=g))
        ta.v.copy_(torch.randn(ta.v.shape, device=cuda, generator=g))
        qkv = torch.randn(n_layers, (s.nq + 2 * s.nkv) * s.hd, device=cuda, generator=g)
        qn = 1 + 0.02 * torch.randn(n_layers, s.hd, device=cuda, generator=g)
        out = torch.empty(steps, n_layers, s.nq * s.hd, device=cuda)

        def step(o):
            for li in range(n_layers):
                ta.attn(li, qkv[li], qn[li], qn[li], o[li], kv_stable=flagged and li > 0)
            ta.pos.add_(1)

        ta.pos.fill_(300)
        buf = torch.empty(n_layers, s.nq * s.hd, device=cuda)
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            step(buf)
        torch.cuda.current_stream().wait_stream(st)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step(buf)
        ta.pos.fill_(310)
        for i in range(steps):
            gr.replay()
            out[i].copy_(buf)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        res[flagged] = (out.cpu(), ta.k.float().cpu(), ta.v.float().cpu())
    for a, b in zip(res[False], res[True]):
        assert torch.equal(a, b)


def _prefill_case(d, max_len, pos0, T, seed, cache="bf16"):
    s = W.C3
    g = torch.Generator().manual_seed(seed)
    Kc = torch.randn(s.nkv, max_len, 128, generator=g).to(CDT[cache])
    Vc = torch.randn(s.nkv, max_len, 128, generator=g).to(CDT[cache])
    rows = torch.randn(T, (s.nq + 2 * s.nkv) * 128, generator=g)
    qn = 1 + 0.02 * torch.randn(128, generator=g)
    kn = 1 + 0.02 * torch.randn(128, generator=g)
    return Kc, Vc, rows, qn, kn


@pytest.mark.parametrize("cache", ["bf16", "f32"])
@pytest.mark.parametrize("pos0,T", [(0, 96), (0, 160), (50, 37), (200, 300), (0, 1), (127, 2)])
def test_prefill_matches_oracle_and_decode_steps(cuda, pos0, T, cache):
    """The causal GQA prefill (bf16: tensor cores; fp32: the parity mode): outputs within the bar of
    the float64 oracle (a run of decode steps), and the appended cache rows bit-identical to those the
    decode kernel writes token by token."""
    s = W.C3
    max_len = 1536
    tol = BF16_TOL if cache == "bf16" else FP32_TOL
    Kc, Vc, rows, qn, kn = _prefill_case(cuda, max_len, pos0, T, seed=pos0 * 7 + T, cache=cache)
    ta = qwen3.TalkerAttention(1, s.nq, s.nkv, max_len, s.theta, s.eps, cuda, CDT[cache])
    rope = ta.rope
    f = lambda t: t.to(cuda).contiguous()
    K1, V1 = f(Kc), f(Vc)
    out = ops.prefill_attention(f(rows), f(qn), f(kn), s.eps, rope, K1, V1, pos0, max_len, s.nq, s.nkv)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    # the same tokens as decode steps on a second copy of the caches
    K2, V2 = f(Kc), f(Vc)
    ta.k[0].copy_(K2)
    ta.v[0].copy_(V2)
    o = torch.empty(s.nq * 128, device=cuda)
    dec = []
    for t in range(T):
        ta.pos.fill_(pos0 + t)
        ta.attn(0, f(rows[t]), f(qn), f(kn), o)
        dec.append(o.clone())
    torch.cuda.synchronize()
    lo, hi = pos0, pos0 + T
    iv = torch.int16 if cache == "bf16" else torch.int32
    assert torch.equal(K1[:, lo:hi].view(iv), ta.k[0][:, lo:hi].view(iv))
    assert torch.equal(V1[:, lo:hi].view(iv), ta.v[0][:, lo:hi].view(iv))
    assert torch.equal(K1[:, :lo].view(iv), f(Kc)[:, :lo].view(iv))  # the prefix untouched
    Kh, Vh = host(f(Kc)).astype(np.float64), host(f(Vc)).astype(np.float64)
    ref = Q.prefill(rows.numpy(), qn.numpy(), kn.numpy(), s.eps, host(rope), Kh, Vh, pos0, s.nq, s.nkv, cache)
    assert rel_l2(host(out), ref) < tol
    assert rel_l2(host(out), host(torch.stack(dec))) < tol


def test_prefill_errors(cuda):
    s = W.C3
    max_len = 64
    K = torch.zeros(s.nkv, max_len, 128, device=cuda, dtype=torch.bfloat16)
    rows = torch.zeros(8, (s.nq + 2 * s.nkv) * 128, device=cuda)
    w = torch.ones(128, device=cuda)
    rope = torch.zeros(max_len, 128, device=cuda)
    with pytest.raises(ValueError):
        ops.prefill_attention(rows, w, w, 1e-6, rope, K, K.float(), 0, max_len, s.nq, s.nkv)  # mixed dtypes
    from sokutou_b200._lib import SokutouError
    with pytest.raises(SokutouError):
        ops.prefill_attention(rows, w, w, 1e-6, rope, K, K.clone(), 60, max_len, s.nq, s.nkv)  # 60 + 8 > 64
