"""The DiT projection GEMM (sk_dit_linear: y = x·wᵀ, F.linear at engine/fused.py:262-264) on the B200.

Bars: relative L2 <= 1e-2 (the bf16 per-layer bar) against the float64 oracle on the same bf16
inputs, and <= 3e-3 as the check of this kernel (one bf16 rounding of an fp32 accumulation is about
1e-3); the same against torch's own cuBLAS F.linear; nothing written outside y.
"""

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import dit_attn_ref as D
from sokutou_b200 import ops
from sokutou_b200._lib import SokutouError

pytestmark = pytest.mark.gpu

SHAPES = [  # M, N, K
    (1536, 3072, 768), (384, 3072, 768), (1536, 768, 768), (512, 8192, 2048), (1536, 2048, 2048),
    (128, 256, 64), (97, 200, 72), (1, 8, 8), (130, 264, 136), (300, 520, 1000), (257, 1032, 4104),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_matches_oracle(cuda, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).bfloat16()
    buf = torch.full((M * N + 4096,), 3.0, dtype=torch.bfloat16, device=cuda)
    y = ops.dit_linear(x.to(cuda), w.to(cuda), out=buf[:M * N].view(M, N))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.all(buf[M * N:] == 3.0)
    want = D.linear(x.float().numpy(), w.float().numpy(), "f32")
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    err = rel_l2(got, want)
    assert err < 1e-2 and err < 3e-3, err
    lib = torch.nn.functional.linear(x.to(cuda), w.to(cuda)).float().cpu().numpy()
    assert rel_l2(got, lib) < 3e-3


# The MLP projections around the SwiGLU (engine/fused.py:305-310): w_13 (N = 2·hidden, K = D) and w_2
# (N = D, K = hidden) at B·L = 1536 rows. The Small model's own widths D = 1280, hidden = 3680 (the
# reference's GEMM bench, ref/gemm_bench.py:26), and the same hidden/D ratio at BASELINE's c1 (D = 768)
# and c2 (D = 2048) widths.
MLP_SHAPES = [  # name, M, N, K
    ("small_w13", 1536, 7360, 1280), ("small_w2", 1536, 1280, 3680),
    ("c1_w13", 1536, 4416, 768), ("c1_w2", 1536, 768, 2208),
    ("c2_w13", 1536, 11776, 2048), ("c2_w2", 1536, 2048, 5888),
]


@pytest.mark.parametrize("name,M,N,K", MLP_SHAPES, ids=[s[0] for s in MLP_SHAPES])
def test_linear_mlp_shapes(cuda, name, M, N, K):
    """bf16 and FP8 at the MLP shapes: against torch's cuBLAS GEMM / cuBLASLt _scaled_mm on the whole
    output, and against the float64 oracle on its first 128 rows (the oracle's full product would take
    the CPU longer than the test is worth)."""
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).bfloat16()
    y = ops.dit_linear(x.to(cuda), w.to(cuda))
    lib = torch.nn.functional.linear(x.to(cuda), w.to(cuda))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert rel_l2(y.float().cpu().numpy(), lib.float().cpu().numpy()) < 3e-3
    want = D.linear(x[:128].float().numpy(), w.float().numpy(), "f32")
    assert rel_l2(y[:128].float().cpu().numpy(), want) < 3e-3
    x8, w8 = _e4m3_operands(M, N, K, M * 3 + N + K)
    inv_x, inv_w = torch.tensor([1 / 16], device=cuda), torch.tensor([1 / 64], device=cuda)
    xt, wt = torch.from_numpy(x8).to(cuda), torch.from_numpy(w8).to(cuda)
    y8 = ops.dit_linear_fp8(xt, wt, inv_x, inv_w)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert rel_l2(y8[:128].float().cpu().numpy(), D.linear_fp8(x8[:128], w8, 1 / 16, 1 / 64)) < 3e-3
    if hasattr(torch, "_scaled_mm"):
        try:
            lib8 = torch._scaled_mm(xt.view(torch.float8_e4m3fn), wt.view(torch.float8_e4m3fn).t(), inv_x, inv_w,
                                    out_dtype=torch.bfloat16)
        except RuntimeError:
            lib8 = None
        if lib8 is not None:
            assert rel_l2(y8.float().cpu().numpy(), lib8.float().cpu().numpy()) < 3e-3


@pytest.mark.parametrize("tile_n", [64, 128, 256])
@pytest.mark.parametrize("M,N,K", [(1536, 3072, 768), (97, 200, 72), (257, 1032, 4104), (640, 136, 520)])
def test_linear_every_tile_width(cuda, tile_n, M, N, K):
    g = torch.Generator().manual_seed(M + N * 3 + K + tile_n)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).bfloat16()
    y = ops.dit_linear(x.to(cuda), w.to(cuda), tile_n=tile_n)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    err = rel_l2(y.float().cpu().numpy(), D.linear(x.float().numpy(), w.float().numpy(), "f32"))
    assert err < 3e-3, err
    auto = ops.dit_linear(x.to(cuda), w.to(cuda))
    assert rel_l2(auto.float().cpu().numpy(), y.float().cpu().numpy()) < 1e-3


def test_linear_graph_replay_and_stream(cuda):
    M, N, K = 640, 1024, 512
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).bfloat16().to(cuda)
    w = (torch.randn(N, K, generator=g) * K ** -0.5).bfloat16().to(cuda)
    y = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        ops.dit_linear(x, w, out=y)
    torch.cuda.current_stream().wait_stream(st)
    ref = y.clone()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        ops.dit_linear(x, w, out=y)
    y.zero_()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_linear_errors(cuda):
    x = torch.zeros(4, 12, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(16, 12, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(SokutouError):
        ops.dit_linear(x, w)  # K = 12 is not a multiple of 8
    with pytest.raises(ValueError):
        ops.dit_linear(x.float(), w.float())  # fp32: the library GEMM
    from sokutou_b200 import _lib
    x = torch.zeros(4, 16, device=cuda, dtype=torch.bfloat16)
    y = torch.zeros(4, 16, device=cuda, dtype=torch.bfloat16)
    call = lambda M, N, K, dtype: _lib.lib().sk_dit_linear(x.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K, dtype, 0)
    assert call(4, 4, 16, 1) == -2   # float32 unsupported
    assert call(0, 8, 16, 0) == -1   # empty
    assert call(4, 12, 16, 0) == -1  # N not a multiple of 8
    assert _lib.lib().sk_dit_linear_ex(x.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 8, 16, 0, 96, 0) == -1  # tile


def _e4m3_operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x8 = D.e4m3_encode((rng.standard_normal((M, K)) * 8).astype(np.float32))
    w8 = D.e4m3_encode((rng.standard_normal((N, K)) * 32).astype(np.float32))
    return x8, w8


@pytest.mark.parametrize("M,N,K,tile_n", [(1536, 3072, 768, 0), (1536, 8192, 2048, 0), (97, 200, 80, 0),
                                          (130, 264, 144, 64), (130, 264, 144, 128), (130, 264, 144, 256),
                                          (1, 8, 16, 0), (257, 1032, 4112, 0)])
def test_linear_fp8_matches_oracle(cuda, M, N, K, tile_n):
    """The FP8 projection (torch._scaled_mm at engine/fp8.py:87-89) against the oracle's exact decode of
    the same e4m3 codes: relative L2 <= 3e-3 (one bf16 rounding); and against torch's own _scaled_mm."""
    x8, w8 = _e4m3_operands(M, N, K, M + N + K)
    inv_x = torch.tensor([1 / 16], device=cuda)
    inv_w = torch.tensor([1 / 64], device=cuda)
    xt = torch.from_numpy(x8).to(cuda)
    wt = torch.from_numpy(w8).to(cuda)
    buf = torch.full((M * N + 4096,), 3.0, dtype=torch.bfloat16, device=cuda)
    y = ops.dit_linear_fp8(xt, wt, inv_x, inv_w, out=buf[:M * N].view(M, N), tile_n=tile_n)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.all(buf[M * N:] == 3.0)
    got = y.float().cpu().numpy()
    want = D.linear_fp8(x8, w8, 1 / 16, 1 / 64)
    err = rel_l2(got, want)
    assert err < 3e-3, err
    if K % 16 == 0 and N % 16 == 0 and hasattr(torch, "_scaled_mm"):
        try:
            lib = torch._scaled_mm(xt.view(torch.float8_e4m3fn), wt.view(torch.float8_e4m3fn).t(), inv_x, inv_w,
                                   out_dtype=torch.bfloat16)
        except RuntimeError:  # a shape or build torch's FP8 GEMM does not take
            lib = None
        if lib is not None:
            assert rel_l2(got, lib.float().cpu().numpy()) < 3e-3


def test_linear_fp8_errors(cuda):
    x = torch.zeros(4, 24, device=cuda, dtype=torch.uint8)
    w = torch.zeros(8, 24, device=cuda, dtype=torch.uint8)
    one = torch.ones(1, device=cuda)
    with pytest.raises(SokutouError):
        ops.dit_linear_fp8(x, w, one, one)  # K = 24 is not a multiple of 16
    from sokutou_b200 import _lib
    x = torch.zeros(4, 32, device=cuda, dtype=torch.uint8)
    y = torch.zeros(4, 8, device=cuda, dtype=torch.bfloat16)
    assert _lib.lib().sk_dit_linear_fp8(x.data_ptr(), x.data_ptr(), y.data_ptr(), 0, one.data_ptr(), 4, 8, 32, 0,
                                        0) == -1  # missing scale
