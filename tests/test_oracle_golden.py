"""The CPU oracle against golden vectors made by the reference's own code (tests/golden/make_golden.py):
the DiT core and bias builder of the reference engine, and transformers' Qwen3 attention functions."""

import numpy as np
import pytest

from conftest import load_golden, rel_l2
from oracle import decode_attn_ref as Q
from oracle import dit_attn_ref as D

FP32_TOL = 1e-5


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
def test_qkv_prologue_matches_reference(case):
    g = load_golden(case)
    H, hd, L = int(g["H"]), int(g["hd"]), int(g["L"])
    q, k, v = D.qkv_prologue(g["o4"], g["qk_w"], g["freqs"], 3, L, H, hd, float(g["qk_eps"]), False)
    assert rel_l2(q, g["q"]) < FP32_TOL
    assert rel_l2(k, g["k"][:, :, :L]) < FP32_TOL
    assert np.array_equal(v, g["v"][:, :, :L])
    # the ctx keys follow the latent keys unchanged in every batch row (engine/fast.py:167-168)
    assert np.array_equal(g["k"][:, :, L:].transpose(0, 2, 1, 3), np.broadcast_to(g["ctx_k"], (3,) + g["ctx_k"].shape))


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
def test_attention_matches_reference_sdpa(case):
    g = load_golden(case)
    L = int(g["L"])
    y = D.dit_attention(g["q"], g["k"][:, :, :L], g["v"][:, :, :L], g["ctx_k"][None], g["ctx_v"][None],
                        D.additive_bias(g["mask"]))
    assert rel_l2(y, g["y"]) < FP32_TOL


def test_cfg_masks_match_reference():
    for case in ("dit_small", "dit_hd128"):
        g = load_golden(case)
        m = D.cfg_key_mask(int(g["L"]), int(g["Tb"]), int(g["Sp"]), int(g["seq_len"]), int(g["n_text"]))
        assert np.array_equal(m, g["mask3"])
        assert np.array_equal(D.additive_bias(m), g["bias3"])
    z = load_golden("dit_masks")
    for i in range(4):
        p = f"case{i}_"
        m = D.cfg_key_mask(*[int(z[p + k]) for k in ("lb", "tb", "n_spk", "seq_len", "n_text")])
        assert np.array_equal(m, z[p + "mask3"])
        assert np.array_equal(D.additive_bias(m), z[p + "bias3"])


def _cache_from(g):
    if str(g["cache"]) == "bf16":
        conv = lambda a: (a.astype(np.uint32) << 16).view(np.float32)
    else:
        conv = lambda a: a.astype(np.float32)
    return conv(g["Kc0"]).copy(), conv(g["Vc0"]).copy()


@pytest.mark.parametrize("case", ["decode_bf16", "decode_f32", "decode_cp"])
def test_decode_step_matches_transformers(case):
    g = load_golden(case)
    Kc, Vc = _cache_from(g)
    pos = int(g["pos"])
    out = Q.decode_step(g["qkv"], g["qn"], g["kn"], float(g["eps"]), g["rope"], Kc, Vc, pos, int(g["nq"]),
                        int(g["nkv"]), str(g["cache"]))
    assert rel_l2(out, g["out"]) < FP32_TOL
    assert rel_l2(Kc[:, pos], g["k_row"]) < FP32_TOL
    assert np.array_equal(Vc[:, pos], g["v_row"])
    f32 = Q.decode_step_f32(g["qkv"], g["qn"], g["kn"], float(g["eps"]), g["rope"], *_cache_from(g), pos,
                            int(g["nq"]), int(g["nkv"]), str(g["cache"]))
    assert rel_l2(f32, g["out"]) < FP32_TOL


def test_rope_table_matches_transformers():
    for case in ("decode_bf16", "decode_f32", "decode_cp"):
        g = load_golden(case)
        assert rel_l2(Q.rope_table(int(g["max_len"])), g["rope"]) < 1e-6


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf, -np.inf, 1e-40], np.float32)
    import torch
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(D.bf16_round(x), ref)
    assert np.isnan(D.bf16_round(np.array([np.nan], np.float32))[0])


def test_fully_masked_rows_give_zero():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 1, 3, 8))
    k = rng.standard_normal((1, 1, 5, 8))
    y = D.dit_attention(q, k, k, bias=np.full((1, 5), -np.inf))
    assert np.all(y == 0)


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
def test_gate_matches_reference(case):
    """The `gate` consumer (engine/fused.py:182-190) against the reference DiT core's own product
    y · sigmoid(gate) (engine/fast.py:174), recorded at the input of w_o."""
    g = load_golden(case)
    out = D.gate(g["y"], g["o4"], "f32")
    assert rel_l2(out, g["gated"]) < 1e-6


def test_e4m3_encoder_known_values():
    """FP8 e4m3 as the reference writes it (engine/fused.py:60-72): nearest even, ±448 saturation,
    subnormal step 2^-9, NaN -> 0x7f, signed zero kept."""
    x = np.array([0.0, -0.0, 1.0, -1.0, 1.0625, 1.1875, 448.0, 449.0, 1e6, float("inf"), float("-inf"),
                  2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -6, float("nan"), 0.3], np.float32)
    want = np.array([0x00, 0x80, 0x38, 0xB8, 0x38, 0x3A, 0x7E, 0x7E, 0x7E, 0x7E, 0xFE,
                     0x01, 0x00, 0x02, 0x08, 0x7F, 0x2A], np.uint8)
    assert np.array_equal(D.e4m3_encode(x), want)
    codes = np.arange(256, dtype=np.uint8)
    finite = (codes & 0x7F) != 0x7F
    assert np.array_equal(D.e4m3_encode(D.e4m3_decode(codes[finite])), codes[finite])  # round trip


@pytest.mark.parametrize("case", ["dit_small", "dit_hd128"])
def test_attention_layer_oracle_matches_reference(case):
    """producer -> SDPA -> gate composed (engine/fused.py:293-298) against the reference DiT core's gated
    output: float32 path within 1e-5, bf16-rounded path within the bf16 bar."""
    g = load_golden(case)
    H, hd, L = int(g["H"]), int(g["hd"]), int(g["L"])
    args = (g["o4"], g["qk_w"], g["freqs"], 3, L, H, hd, float(g["qk_eps"]), g["ctx_k"][None], g["ctx_v"][None],
            g["bias3"])
    assert rel_l2(D.attention_layer(*args, bf16=False), g["gated"]) < FP32_TOL
    assert rel_l2(D.attention_layer(*args, bf16=True), g["gated"]) < 1e-2


def test_linear_matches_torch_linear():
    """The projection restatement against torch's own F.linear (the reference's `mm`,
    engine/fused.py:262-264) in float64 on the host."""
    import torch
    rng = np.random.default_rng(4)
    x = rng.standard_normal((37, 72)).astype(np.float32)
    w = rng.standard_normal((40, 72)).astype(np.float32)
    want = torch.nn.functional.linear(torch.from_numpy(x).double(), torch.from_numpy(w).double()).numpy()
    assert rel_l2(D.linear(x, w, "f32"), want) < 1e-7
    got = D.linear(x, w, "bf16")
    ref = torch.from_numpy(want.astype(np.float32)).bfloat16().float().numpy()
    assert np.array_equal(got, ref)


def test_e4m3_decode_matches_torch_float8():
    """Every finite e4m3 code decodes to the value torch's float8_e4m3fn gives it (the operand type of
    torch._scaled_mm at engine/fp8.py:87-89), and linear_fp8 equals the float64 product of those values."""
    import torch
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)
    mine = D.e4m3_decode(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(mine, theirs)
    rng = np.random.default_rng(5)
    x8 = rng.choice(codes, size=(9, 32))
    w8 = rng.choice(codes, size=(16, 32))
    xs = torch.from_numpy(x8).view(torch.float8_e4m3fn).double()
    ws = torch.from_numpy(w8).view(torch.float8_e4m3fn).double()
    want = ((xs @ ws.T) * (np.float32(1 / 16) * np.float32(1 / 64))).float().bfloat16().float().numpy()
    assert np.array_equal(D.linear_fp8(x8, w8, 1 / 16, 1 / 64), want)
