"""The DiT `gate` consumer (engine/fused.py:182-190) on the B200 against the CPU oracle.

Bars: fp32 output relative L2 <= 1e-6 (against the reference DiT core's own golden product too);
bf16 output bit-identical to the oracle except where CUDA's expf and numpy's exp differ in the last
fp32 bit right at a bf16 rounding boundary (at most 1 bf16 step there, <= 0.1 % of elements);
the FP8 e4m3 encoder bit-exact.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2
from oracle import dit_attn_ref as D
from sokutou_b200 import ops
from sokutou_b200._lib import SokutouError

pytestmark = pytest.mark.gpu


def _bf16_steps(a, b):
    """Distance in bf16 steps between two bf16-representable float32 arrays (same sign assumed)."""
    ia = (np.asarray(a, np.float32).view(np.int32) >> 16).astype(np.int64)
    ib = (np.asarray(b, np.float32).view(np.int32) >> 16).astype(np.int64)
    return np.abs(ia - ib)


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
def test_gate_f32_matches_golden(cuda, case):
    g = load_golden(case)
    y = torch.as_tensor(g["y"]).to(cuda).contiguous()
    o4 = torch.as_tensor(g["o4"]).to(cuda).contiguous()
    out = ops.dit_gate(y, o4).cpu().numpy()
    assert rel_l2(out, g["gated"]) < 1e-6
    assert rel_l2(out, D.gate(g["y"], g["o4"], "f32")) < 1e-6


@pytest.mark.parametrize("rows,dim", [(1, 8), (97, 768), (1536, 768), (3 * 512, 2048)])
def test_gate_bf16_matches_oracle(cuda, rows, dim):
    gen = torch.Generator().manual_seed(rows + dim)
    y = (torch.randn(rows, dim, generator=gen)).bfloat16()
    o4 = (torch.randn(rows, 4 * dim, generator=gen) * 3).bfloat16()
    out = ops.dit_gate(y.to(cuda), o4.to(cuda)).float().cpu().numpy()
    want = D.gate(y.float().numpy(), o4.float().numpy(), "bf16")
    steps = _bf16_steps(out, want)
    assert steps.max() <= 1
    assert (steps > 0).mean() <= 1e-3
    assert rel_l2(out, want) < 1e-3


def test_gate_accepts_attention_layout(cuda):
    B, L, H, hd = 3, 40, 4, 64
    gen = torch.Generator().manual_seed(5)
    y = torch.randn(B, L, H, hd, generator=gen).bfloat16().to(cuda)
    o4 = torch.randn(B * L, 4 * H * hd, generator=gen).bfloat16().to(cuda)
    out = ops.dit_gate(y, o4)
    assert out.shape == (B * L, H * hd)
    want = D.gate(y.float().cpu().numpy(), o4.float().cpu().numpy(), "bf16")
    assert rel_l2(out.float().cpu().numpy(), want) < 1e-3


def test_e4m3_encoder_bit_exact(cuda):
    """gate = 100 makes sigmoid exactly 1.0f, so the output is the encoder applied to y · scale."""
    tab = D.e4m3_decode(np.arange(0x7F, dtype=np.uint8))
    mid = ((tab[1:] + tab[:-1]) / 2).astype(np.float32)
    rng = np.random.default_rng(0)
    vals = np.concatenate([tab, -tab, mid, -mid, np.nextafter(mid, np.float32(0)), np.nextafter(mid, np.float32(1e9)),
                           rng.standard_normal(40000).astype(np.float32) * 50,
                           rng.standard_normal(40000).astype(np.float32) * 1e-2,
                           np.array([0.0, -0.0, 447.9, 448.0, 449.0, 464.0, 465.0, 1e30, np.inf, -np.inf, np.nan],
                                    np.float32)]).astype(np.float32)
    n = (len(vals) + 7) // 8 * 8
    y = np.zeros(n, np.float32)
    y[: len(vals)] = vals
    rows, Dm = n // 8, 8
    o4 = np.zeros((rows, 4 * Dm), np.float32)
    o4[:, 3 * Dm:] = 100.0
    for scale in (1.0, 0.5):
        out = ops.dit_gate(torch.as_tensor(y).to(cuda), torch.as_tensor(o4).to(cuda), fp8_scale=scale)
        got = out.cpu().numpy().reshape(-1)[: len(vals)]
        want = D.e4m3_encode((vals * np.float32(scale)).astype(np.float32))
        assert np.array_equal(got, want), np.flatnonzero(got != want)[:10]


def test_gate_bf16_to_e4m3(cuda):
    gen = torch.Generator().manual_seed(9)
    y = torch.randn(256, 1024, generator=gen).bfloat16()
    o4 = torch.randn(256, 4096, generator=gen).bfloat16()
    out = ops.dit_gate(y.to(cuda), o4.to(cuda), fp8_scale=16.0).cpu().numpy()
    want = D.gate(y.float().numpy(), o4.float().numpy(), "e4m3", 16.0)
    diff = out != want
    assert diff.mean() <= 1e-3  # only where expf and numpy's exp differ in the last bit at a boundary
    if diff.any():
        assert np.abs(D.e4m3_decode(out[diff]) - D.e4m3_decode(want[diff])).max() <= \
            np.abs(D.e4m3_decode(want[diff])).max() * 0.125 + 1e-6


def test_gate_errors(cuda):
    y = torch.zeros(4, 12, device=cuda, dtype=torch.bfloat16)
    o4 = torch.zeros(4, 48, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(SokutouError):
        ops.dit_gate(y, o4)  # D = 12 is not a multiple of 8
    y = torch.zeros(0, 16, device=cuda, dtype=torch.bfloat16)
    o4 = torch.zeros(0, 64, device=cuda, dtype=torch.bfloat16)
    assert ops.dit_gate(y, o4).shape == (0, 16)
