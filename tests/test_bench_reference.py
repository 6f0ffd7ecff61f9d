"""bench.py's reference arm runs on the host CPU alone and prints the contract's JSON line."""

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_one_json_line():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--cpu-seconds", "2"], capture_output=True, text=True, env=env,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "dit_attn_tflops" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["cores"] >= 1


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--cpu-seconds", "1"], capture_output=True, text=True, env=env,
                         timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == ""


def test_roofline_traffic_comes_from_the_committed_single_launch_captures():
    """bench.py's roofline.traffic is the call-mix average of the per-shape one-launch captures recorded in
    the c1 profile summary; every shape of the step must have its line."""
    sys.path.insert(0, ROOT)
    import bench
    from sokutou_b200 import workloads as W
    shapes = [W.c1(L) for L in W.C1_SWEEP]
    t = bench.profile_traffic_mix("dit_attn_tc_c1.md", shapes)
    assert t is not None and t > 0
    # within a few percent of the mix's algorithmic reads (latent q/k/v per row, the shared text+speaker
    # K/V once, one bf16 bias per key and row): no re-reads
    alg = [3 * B * sh.H * sh.L * sh.hd * 2 + (sh.Tb + sh.Sp) * sh.H * sh.hd * 4 + B * (sh.L + sh.Tb + sh.Sp) * 2
           for sh in shapes for B in sh.synthesis_calls()]
    assert 1.0 <= t / (sum(alg) / len(alg)) < 1.05
