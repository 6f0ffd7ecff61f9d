"""The fused DiT attention block (sk_dit_attention_layer: producer + attention + gate in two launches)
on the B200.

Bars: bit-identical to the three separate entry points (sk_dit_qkv_prologue -> sk_dit_attention ->
sk_dit_gate) on the same inputs; relative L2 <= 1e-2 (the bf16 per-layer bar) against the float64
oracle of the engine's three steps and against the reference DiT core's own golden gated output.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2
from oracle import dit_attn_ref as D
from sokutou_b200 import dit, ops, workloads as W

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2


def _inputs(dev, B, L, H, hd, S, seed, ctx_per_row=False, bias_kind="cfg"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    D_ = H * hd
    o4 = (torch.randn(B * L, 4 * D_, generator=g) * 0.5).bfloat16()
    qk_w = (1 + 0.1 * torch.randn(2, H, hd, generator=g)).float()
    freqs = torch.from_numpy(D.rope_freqs(max(L, 1), hd)).float()
    kc = vc = None
    if S > 0:
        shape = (B, S, H, hd) if ctx_per_row else (S, H, hd)
        kc = torch.randn(shape, generator=g)
        kc = (kc * torch.rsqrt(kc.pow(2).mean(-1, keepdim=True))).bfloat16()
        vc = (torch.randn(shape, generator=g) * 0.5).bfloat16()
    bias = None
    if bias_kind == "cfg" and S > 0:
        tb = min(S, 64 if S >= 64 else S // 2)
        bias = dit.cfg_bias(L, tb, S - tb, max(L - 3, 1), max(tb // 2, 1), device="cpu")[:B].contiguous()
    elif bias_kind == "shared":
        bias = torch.zeros(L + S).bfloat16()
        bias[L // 2:L // 2 + 3] = float("-inf")
    t = lambda x: None if x is None else x.to(dev).contiguous()
    return t(o4), t(qk_w), t(freqs), t(kc), t(vc), t(bias)


def _separate(o4, qk_w, freqs, kc, vc, bias, B, L, H, hd, eps):
    q, k, v = ops.dit_qkv_prologue(o4, qk_w, freqs, B, L, H, hd, eps)
    y = ops.dit_attention(q, k, v, kc, vc, bias)
    return ops.dit_gate(y, o4)


CASES = [  # B, L, H, hd, S
    (3, 128, 12, 64, 256), (1, 128, 12, 64, 256), (3, 256, 12, 64, 256), (3, 512, 12, 64, 256),
    (1, 512, 12, 64, 256), (3, 512, 16, 128, 512), (1, 512, 16, 128, 512),
    (3, 97, 4, 64, 7), (2, 1, 2, 64, 5), (3, 129, 4, 128, 200), (2, 300, 2, 64, 1), (1, 40, 2, 128, 0),
    (3, 640, 2, 64, 40), (2, 384, 2, 128, 130),
]


@pytest.mark.parametrize("B,L,H,hd,S", CASES)
def test_layer_bit_identical_to_separate_calls(cuda, B, L, H, hd, S):
    args = _inputs(cuda, B, L, H, hd, S, seed=B * 1000 + L + hd)
    fused = ops.dit_attention_layer(args[0], args[1], args[2], B, L, H, hd, 1e-6, args[3], args[4], args[5])
    sep = _separate(*args, B, L, H, hd, 1e-6)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    a, b = fused.view(torch.int16).cpu().numpy(), sep.view(torch.int16).cpu().numpy()
    assert np.array_equal(a, b), f"{(a != b).sum()} of {a.size} differ"


@pytest.mark.parametrize("B,L,H,hd,S", [(3, 128, 4, 64, 256), (3, 97, 4, 64, 7), (3, 129, 2, 128, 200),
                                         (1, 512, 2, 128, 512), (3, 512, 16, 128, 512), (3, 768, 12, 64, 256),
                                         (2, 1, 2, 64, 5)])
def test_layer_matches_oracle(cuda, B, L, H, hd, S):
    o4, qk_w, freqs, kc, vc, bias = _inputs(cuda, B, L, H, hd, S, seed=7 + L)
    out = ops.dit_attention_layer(o4, qk_w, freqs, B, L, H, hd, 1e-6, kc, vc, bias).float().cpu().numpy()
    h = lambda t: None if t is None else t.float().cpu().numpy()
    kcn = h(kc)
    want = D.attention_layer(h(o4), h(qk_w), h(freqs), B, L, H, hd, 1e-6,
                             None if kcn is None else kcn[None], None if kc is None else h(vc)[None], h(bias))
    assert rel_l2(out, want) < BF16_TOL


def test_layer_per_row_ctx_and_shared_bias(cuda):
    B, L, H, hd, S = 3, 200, 4, 64, 70
    args = _inputs(cuda, B, L, H, hd, S, seed=11, ctx_per_row=True, bias_kind="shared")
    fused = ops.dit_attention_layer(args[0], args[1], args[2], B, L, H, hd, 1e-6, args[3], args[4], args[5])
    sep = _separate(*args, B, L, H, hd, 1e-6)
    assert torch.equal(fused.view(torch.int16), sep.view(torch.int16))
    o4, qk_w, freqs, kc, vc, bias = (None if t is None else t.float().cpu().numpy() for t in args)
    want = D.attention_layer(o4, qk_w, freqs, B, L, H, hd, 1e-6, kc, vc, bias)
    assert rel_l2(fused.float().cpu().numpy(), want) < BF16_TOL


def test_layer_without_bias(cuda):
    B, L, H, hd, S = 3, 160, 2, 128, 96
    args = list(_inputs(cuda, B, L, H, hd, S, seed=12, bias_kind="none"))
    fused = ops.dit_attention_layer(args[0], args[1], args[2], B, L, H, hd, 1e-6, args[3], args[4], None)
    sep = _separate(*args[:5], None, B, L, H, hd, 1e-6)
    assert torch.equal(fused.view(torch.int16), sep.view(torch.int16))


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
def test_layer_matches_reference_golden(cuda, case):
    """The reference DiT core's gated attention output (engine/fast.py:156-174, fp32) recorded at the
    input of w_o, against this launch on the same projection rows in bf16."""
    g = load_golden(case)
    H, hd, L = int(g["H"]), int(g["hd"]), int(g["L"])
    t = lambda x, dt=torch.bfloat16: torch.as_tensor(np.ascontiguousarray(x)).to(cuda, dt).contiguous()
    out = ops.dit_attention_layer(t(g["o4"]), t(g["qk_w"], torch.float32), t(g["freqs"], torch.float32), 3, L, H, hd,
                                  float(g["qk_eps"]), t(g["ctx_k"]), t(g["ctx_v"]), t(g["bias3"]))
    assert rel_l2(out.float().cpu().numpy(), g["gated"]) < BF16_TOL


def test_layer_graph_replay(cuda):
    sh = W.c1(256)
    B, L, H, hd, S = 3, sh.L, sh.H, sh.hd, sh.S
    args = _inputs(cuda, B, L, H, hd, S, seed=21)
    out = torch.empty(B * L, H * hd, device=cuda, dtype=torch.bfloat16)
    run = lambda: ops.dit_attention_layer(args[0], args[1], args[2], B, L, H, hd, 1e-6, args[3], args[4], args[5],
                                          out=out)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        run()
    torch.cuda.current_stream().wait_stream(st)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        run()
    out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    sep = _separate(*args, B, L, H, hd, 1e-6)
    assert torch.equal(out.view(torch.int16), sep.view(torch.int16))


def test_layer_errors(cuda):
    B, L, H, hd = 1, 16, 2, 64
    o4 = torch.zeros(B * L, 4 * H * hd, device=cuda, dtype=torch.bfloat16)
    qk_w = torch.ones(2, H, hd, device=cuda)
    fr = torch.zeros(L, hd // 2, 2, device=cuda)
    qb = torch.empty(B, H, L, hd, device=cuda, dtype=torch.bfloat16)
    kb = torch.empty_like(qb)
    vb = torch.empty_like(qb)
    with pytest.raises(ValueError):
        ops.dit_attention_layer(o4.float(), qk_w, fr, B, L, H, hd, 1e-6)  # fp32 runs the separate calls
    from sokutou_b200 import _lib
    call = lambda Hh, hdd, dtype, kbuf: _lib.lib().sk_dit_attention_layer(
        o4.data_ptr(), qk_w.data_ptr(), fr.data_ptr(), 0, 0, 0, o4.data_ptr(), qb.data_ptr(), kbuf, vb.data_ptr(), B,
        Hh, L, 0, hdd, 0, 0, 1e-6, dtype, 0.0, 0)
    assert call(H, 96, 0, kb.data_ptr()) == -2   # head_dim 96: unsupported
    assert call(H, hd, 1, kb.data_ptr()) == -2   # float32
    assert call(3, hd, 0, kb.data_ptr()) == -1   # odd head count
    assert call(H, hd, 0, 0) == -1               # missing k scratch
