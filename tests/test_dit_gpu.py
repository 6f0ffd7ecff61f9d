"""DiT attention on the B200 against the CPU oracle (and the reference-made golden vectors).

Tolerances (relative L2 of the whole output):
  fp32 mode (SK_F32, CUDA-core kernel): <= 1e-5
  bf16 mode (SK_BF16, tcgen05 kernel):  <= 1e-2, compared with the float64 oracle run on the same
  bf16-rounded inputs.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2
from oracle import dit_attn_ref as D
from sokutou_b200 import dit, ops, workloads as W

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
BF16_TOL = 1e-2
DT = {"f32": torch.float32, "bf16": torch.bfloat16}


def dev(x, d, dtype):
    return torch.as_tensor(np.asarray(x)).to(device=d, dtype=dtype).contiguous()


def host(t):
    return t.float().cpu().numpy()


def tol(dt):
    return FP32_TOL if dt == torch.float32 else BF16_TOL


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
@pytest.mark.parametrize("name", ["f32", "bf16"])
def test_prologue_matches_oracle_and_golden(cuda, case, name):
    g = load_golden(case)
    dt = DT[name]
    H, hd, L = int(g["H"]), int(g["hd"]), int(g["L"])
    o4 = dev(g["o4"], cuda, dt)
    q, k, v = ops.dit_qkv_prologue(o4, dev(g["qk_w"], cuda, torch.float32), dev(g["freqs"], cuda, torch.float32),
                                   3, L, H, hd, float(g["qk_eps"]))
    qo, ko, vo = D.qkv_prologue(host(o4), g["qk_w"], g["freqs"], 3, L, H, hd, float(g["qk_eps"]), dt == torch.bfloat16)
    t = FP32_TOL if dt == torch.float32 else 2e-3
    assert rel_l2(host(q), qo) < t and rel_l2(host(k), ko) < t
    assert np.array_equal(host(v), vo)
    if dt == torch.float32:  # the reference's own q/k (engine/fast.py:156-168)
        assert rel_l2(host(q), g["q"]) < FP32_TOL
        assert rel_l2(host(k), g["k"][:, :, :L]) < FP32_TOL


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
@pytest.mark.parametrize("name", ["f32", "bf16"])
def test_attention_matches_golden(cuda, case, name):
    g = load_golden(case)
    dt = DT[name]
    L = int(g["L"])
    q = dev(g["q"], cuda, dt)
    k_lat, v_lat = dev(g["k"][:, :, :L], cuda, dt), dev(g["v"][:, :, :L], cuda, dt)
    k_ctx, v_ctx = dev(g["ctx_k"], cuda, dt), dev(g["ctx_v"], cuda, dt)
    bias = dev(D.additive_bias(g["mask"]), cuda, dt)
    y = ops.dit_attention(q, k_lat, v_lat, k_ctx, v_ctx, bias)
    ref = D.dit_attention(host(q), host(k_lat), host(v_lat), host(k_ctx)[None], host(v_ctx)[None], host(bias))
    assert rel_l2(host(y), ref) < tol(dt)
    if dt == torch.float32:
        assert rel_l2(host(y), g["y"]) < FP32_TOL
    # the SDPA drop-in (keys already concatenated per batch row, engine/fused.py:295) agrees
    yk = ops.sdpa(q, dev(g["k"], cuda, dt), dev(g["v"], cuda, dt), attn_mask=bias.reshape(3, 1, 1, -1))
    assert yk.transpose(1, 2).is_contiguous()
    assert rel_l2(host(yk.transpose(1, 2)), ref) < tol(dt)
    ym = ops.sdpa(q, dev(g["k"], cuda, dt), dev(g["v"], cuda, dt),
                  attn_mask=torch.as_tensor(g["mask"]).reshape(3, 1, 1, -1).to(cuda))
    assert torch.equal(ym, yk)


def _config_case(cuda, shape, B, dt, seed):
    x = W.dit_call_inputs(shape, B, seed, device=cuda, dtype=dt)
    qk_w = W.dit_qk_weights(shape, cuda)
    freqs = W.dit_freqs(shape.L, shape.hd, device=cuda)
    layer = dit.DitLayerAttention(B, shape.L, shape.H, shape.hd, shape.S, dt, cuda)
    bias = x["bias3"][:B].contiguous()
    y = layer.attention(x["o4"], qk_w, freqs, x["ctx_k"], x["ctx_v"], bias)
    torch.cuda.synchronize()
    ref = D.dit_attention(host(layer.q), host(layer.k), host(layer.v), host(x["ctx_k"])[None], host(x["ctx_v"])[None],
                          host(bias))
    return host(y), ref, layer, x


@pytest.mark.parametrize("shape", [W.C0, W.c1(128), W.c1(256), W.c1(512), W.C2], ids=lambda s: s.name)
@pytest.mark.parametrize("B", [3, 1])
@pytest.mark.parametrize("name", ["bf16", "f32"])
def test_baseline_configs(cuda, shape, B, name):
    dt = DT[name]
    y, ref, layer, x = _config_case(cuda, shape, B, dt, seed=7)
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) < tol(dt)


def test_full_chain_against_oracle_fp32(cuda):
    """o4 -> producer -> attention, all against the oracle's own producer (c0, fp32 mode)."""
    shape = W.C0
    y, _, layer, x = _config_case(cuda, shape, 3, torch.float32, seed=0)
    q, k, v = D.qkv_prologue(host(x["o4"]), np.ones((2, shape.H, shape.hd)), D.rope_freqs(shape.L, shape.hd), 3,
                             shape.L, shape.H, shape.hd, 1e-6, False)
    ref = D.dit_attention(q, k, v, host(x["ctx_k"])[None], host(x["ctx_v"])[None], host(x["bias3"]))
    assert rel_l2(y, ref) < FP32_TOL


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("L,Lk,S", [(1, 1, 0), (97, 97, 7), (129, 129, 200), (300, 260, 1), (128, 5, 300)])
@pytest.mark.parametrize("name", ["bf16", "f32"])
def test_ragged_shapes(cuda, hd, L, Lk, S, name):
    dt = DT[name]
    torch.manual_seed(L * 1000 + Lk + S + hd)
    B, H = 2, 3
    q = torch.randn(B, H, L, hd, device=cuda).to(dt)
    kl, vl = (torch.randn(B, H, Lk, hd, device=cuda).to(dt) for _ in range(2))
    kc, vc = ((torch.randn(S, H, hd, device=cuda).to(dt) for _ in range(2)) if S else (None, None))
    K = Lk + S
    bias = torch.zeros(B, K, device=cuda)
    bias[0, torch.rand(K, device=cuda) < 0.3] = float("-inf")
    bias[0, 0] = 0.0
    bias = bias.to(dt)
    # write into a guarded buffer: nothing past the output may change
    n = B * L * H * hd
    buf = torch.full((n + 4096,), 7.0, device=cuda, dtype=dt)
    y = ops.dit_attention(q, kl, vl, kc, vc, bias, out=buf[:n].view(B, L, H, hd))
    ref = D.dit_attention(host(q), host(kl), host(vl), None if kc is None else host(kc)[None],
                          None if vc is None else host(vc)[None], host(bias))
    assert rel_l2(host(y), ref) < tol(dt)
    assert torch.all(buf[n:] == 7.0)


@pytest.mark.parametrize("name", ["bf16", "f32"])
def test_fully_masked_row_and_no_bias(cuda, name):
    dt = DT[name]
    torch.manual_seed(3)
    B, H, L, hd, Lk, S = 3, 2, 130, 64, 140, 60
    q = torch.randn(B, H, L, hd, device=cuda).to(dt)
    kl, vl = (torch.randn(B, H, Lk, hd, device=cuda).to(dt) for _ in range(2))
    kc, vc = (torch.randn(S, H, hd, device=cuda).to(dt) for _ in range(2))
    bias = torch.zeros(B, Lk + S, device=cuda, dtype=dt)
    bias[1] = float("-inf")                        # batch row 1 sees nothing: zeros, as torch does
    y = ops.dit_attention(q, kl, vl, kc, vc, bias)
    assert torch.all(y[1] == 0)
    ref = D.dit_attention(host(q), host(kl), host(vl), host(kc)[None], host(vc)[None], host(bias))
    assert rel_l2(host(y), ref) < tol(dt)
    y0 = ops.dit_attention(q, kl, vl, kc, vc, None)
    ref0 = D.dit_attention(host(q), host(kl), host(vl), host(kc)[None], host(vc)[None], None)
    assert rel_l2(host(y0), ref0) < tol(dt)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("Lk,S", [(700, 520), (256, 1100), (8300, 200)])
def test_fully_masked_key_tiles(cuda, hd, Lk, S):
    """Key tiles past the latent ones whose every key is masked are not run by the bf16 kernel when the
    grid has more CTAs than SMs (here 6 rows x 16 heads x 2 query tiles = 192) and at most 64 key tiles
    (8300 latent keys = 65 tiles take the path without skipping): rows with dead conditioning tiles, a
    row with one live key in its last tile, a fully masked row, a row masked past its first two tiles,
    and random single-key masks that leave no tile dead. Heads are independent, so two of the 16 are
    checked against the oracle."""
    torch.manual_seed(Lk + S + hd)
    B, H, L = 6, 16, 256 if Lk < 8000 else 128
    dt = torch.bfloat16
    q = torch.randn(B, H, L, hd, device=cuda).to(dt)
    kl, vl = (torch.randn(B, H, Lk, hd, device=cuda).to(dt) for _ in range(2))
    kc, vc = (torch.randn(S, H, hd, device=cuda).to(dt) for _ in range(2))
    K = Lk + S
    bias = torch.zeros(B, K, device=cuda)
    bias[1, Lk:Lk + min(S, 128)] = float("-inf")          # row 1: the first conditioning tile ...
    for t in (2, 4):                                      # ... and more whole conditioning tiles
        bias[1, Lk + t * 128:Lk + min(S, (t + 1) * 128)] = float("-inf")
    bias[1, 300:310] = float("-inf")
    bias[2] = float("-inf")                               # row 2: one live key, in the last tile
    bias[2, K - 1] = 0.0
    bias[3] = float("-inf")                               # row 3: nothing visible -> zeros
    bias[4, 256:] = float("-inf")                         # row 4: only the first two latent tiles
    bias[5, torch.rand(K, device=cuda) < 0.5] = float("-inf")  # row 5: no tile entirely masked
    bias = bias.to(dt)
    y = ops.dit_attention(q, kl, vl, kc, vc, bias)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.all(y[3] == 0)
    hs = [0, H - 1]
    ref = D.dit_attention(host(q[:, hs]), host(kl[:, hs]), host(vl[:, hs]), host(kc[:, hs])[None],
                          host(vc[:, hs])[None], host(bias))
    got = host(y[:, :, hs])
    for r in (0, 1, 2, 4, 5):
        assert rel_l2(got[r], ref[r]) < BF16_TOL, r


@pytest.mark.parametrize("name", ["bf16", "f32"])
def test_per_batch_ctx_and_shared_bias(cuda, name):
    dt = DT[name]
    torch.manual_seed(5)
    B, H, L, hd, Lk, S = 3, 4, 128, 128, 128, 256
    q = torch.randn(B, H, L, hd, device=cuda).to(dt)
    kl, vl = (torch.randn(B, H, Lk, hd, device=cuda).to(dt) for _ in range(2))
    kc, vc = (torch.randn(B, S, H, hd, device=cuda).to(dt) for _ in range(2))
    bias = torch.zeros(Lk + S, device=cuda, dtype=dt)
    bias[Lk + 100:] = float("-inf")
    y = ops.dit_attention(q, kl, vl, kc, vc, bias)
    ref = D.dit_attention(host(q), host(kl), host(vl), host(kc), host(vc), host(bias)[None])
    assert rel_l2(host(y), ref) < tol(dt)


def test_large_scores_rescale_path(cuda):
    """Scores that grow tile by tile exercise the O rescale in TMEM."""
    torch.manual_seed(11)
    B, H, L, hd, Lk = 1, 2, 128, 64, 1024
    q = torch.randn(B, H, L, hd, device=cuda) * 3
    kl = torch.randn(B, H, Lk, hd, device=cuda) * torch.linspace(0.1, 4, Lk, device=cuda)[None, None, :, None]
    vl = torch.randn(B, H, Lk, hd, device=cuda)
    q, kl, vl = (t.to(torch.bfloat16).contiguous() for t in (q, kl, vl))
    y = ops.dit_attention(q, kl, vl)
    ref = D.dit_attention(host(q), host(kl), host(vl))
    assert rel_l2(host(y), ref) < BF16_TOL


def test_graph_capture_replays(cuda):
    shape = W.c1(256)
    x = W.dit_call_inputs(shape, 3, 1, device=cuda, dtype=torch.bfloat16)
    layer = dit.DitLayerAttention(3, shape.L, shape.H, shape.hd, shape.S, torch.bfloat16, cuda)
    args = (x["o4"], W.dit_qk_weights(shape, cuda), W.dit_freqs(shape.L, shape.hd, device=cuda), x["ctx_k"],
            x["ctx_v"], x["bias3"])
    y0 = layer.attention(*args).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.attention(*args)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.attention(*args)
    layer.y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(layer.y, y0)


def test_errors_raise(cuda):
    q = torch.zeros(1, 1, 8, 96, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        ops.dit_attention(q, q, q)
    assert ops.device_error() == 0
