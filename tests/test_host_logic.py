"""Host-side logic that needs no GPU: CFG bias construction, workload accounting, determinism."""

import numpy as np
import torch

from conftest import load_golden
from oracle import dit_attn_ref as D
from sokutou_b200 import dit, qwen3, workloads as W


def test_cfg_bias_matches_reference_masks():
    z = load_golden("dit_masks")
    for i in range(4):
        p = f"case{i}_"
        args = [int(z[p + k]) for k in ("lb", "tb", "n_spk", "seq_len", "n_text")]
        assert np.array_equal(dit.cfg_key_mask(*args).numpy(), z[p + "mask3"])
        b = dit.cfg_bias(*args, dtype=torch.float32).numpy()
        assert np.array_equal(b, z[p + "bias3"])


def test_flop_and_byte_accounting():
    assert W.C0.flops(3) == 1_207_959_552
    assert W.C2.flops(3) == 12_884_901_888
    # per synthesis, 10 steps B=3 + 10 steps B=1
    assert abs(W.c1(128).synthesis_flops() - 7.248e10) / 7.248e10 < 1e-3
    assert abs(W.c1(256).synthesis_flops() - 1.933e11) / 1.933e11 < 1e-3
    assert abs(W.c1(512).synthesis_flops() - 5.798e11) / 5.798e11 < 1e-3
    assert abs(W.C2.synthesis_flops() - 4.123e12) / 4.123e12 < 1e-3
    assert W.C3.layer_bytes(1120) == 4_616_192
    assert W.C3.decode_bytes() == 72_284_635_136
    assert len(W.c1(256).synthesis_calls()) == 240


def test_workload_inputs_are_seeded():
    a = W.dit_call_inputs(W.C0, 3, seed=0)
    b = W.dit_call_inputs(W.C0, 3, seed=0)
    c = W.dit_call_inputs(W.C0, 3, seed=1)
    assert torch.equal(a["o4"], b["o4"]) and not torch.equal(a["o4"], c["o4"])
    assert 16 <= a["n_text"] <= 64
    assert a["o4"].shape == (3 * 256, 4 * 12 * 64)
    assert a["bias3"].shape == (3, 512)
    # ctx keys arrive unit-RMS per head
    rms = a["ctx_k"].pow(2).mean(-1).sqrt()
    assert torch.allclose(rms, torch.ones_like(rms), atol=1e-3)


def test_freqs_table_matches_oracle():
    assert np.allclose(W.dit_freqs(300, 64).numpy(), D.rope_freqs(300, 64), atol=1e-6)


def test_qwen3_rope_table_matches_oracle():
    from oracle import decode_attn_ref as Q
    assert np.allclose(qwen3.rope_table(1200, 1e6).numpy(), Q.rope_table(1200), atol=2e-6)


def test_serving_requests_seeded():
    r = W.serving_requests(0)
    assert len(r) == 64
    assert sum(k == "dit" for k, _ in r) == 32
    assert all(96 <= s <= 384 for k, s in r if k == "dit")
    assert all(200 <= s <= 1500 for k, s in r if k == "decode")
    assert r == W.serving_requests(0)


def test_profile_module_runs_as_a_script():
    """`python -m sokutou_b200.profile` parses its arguments (no GPU needed for --help)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "sokutou_b200.profile", "--help"], cwd=root, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "--case" in r.stdout


def test_code_predictor_pair_equals_two_sequential_blocks():
    """The oracle's paired code-predictor pass (qwen3/kernels.py:600-617) and two single-position blocks
    in a row (positions 0 then 1) are the same float64 arithmetic: row 1's projection reads only its own
    residual row, and its attention sees row 0's appended key either way."""
    import numpy as np
    from oracle import decode_attn_ref as Q
    rng = np.random.default_rng(0)
    hid, nq, nkv, hd = 256, 16, 8, 128
    W = rng.standard_normal(((nq + 2 * nkv) * hd, hid)) / 16
    Wo = rng.standard_normal((hid, nq * hd)) / 45
    nw, ones = 1 + 0.1 * rng.standard_normal(hid), np.ones(hd)
    rope, h2 = Q.rope_table(16), rng.standard_normal((2, hid))
    K1, V1 = np.zeros((nkv, 16, hd)), np.zeros((nkv, 16, hd))
    K2, V2 = K1.copy(), V1.copy()
    a = Q.decode_block_pair(h2, nw, 1e-6, W, ones, ones, 1e-6, rope, K1, V1, nq, nkv, Wo, "f32")
    b = [Q.decode_block(h2[r], nw, 1e-6, W, ones, ones, 1e-6, rope, K2, V2, r, nq, nkv, Wo, "f32") for r in (0, 1)]
    for r in (0, 1):
        np.testing.assert_array_equal(a[r], b[r])
    np.testing.assert_array_equal(K1, K2)
    np.testing.assert_array_equal(V1, V2)
