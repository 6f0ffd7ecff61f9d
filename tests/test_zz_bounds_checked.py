"""The sanitizer substitute for this pool (compute-sanitizer is unavailable): the GPU parity suites run
again against the bounds-checked library (sokutou_b200/lib/libsokutou_b200_checked.so, built with
-DSK_BOUNDS_CHECK=1), in which every guarded shared-memory, tensor-memory and global index is tested
before its access and an out-of-range one records SK_DEVERR_BOUNDS instead of touching memory. Every
test must pass and leave no such error (tests/conftest.py checks the error word after each test)."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_parity_suites_under_bounds_checks(cuda):
    from sokutou_b200 import build
    lib = build.build(checked=True)
    env = dict(os.environ, SOKUTOU_B200_LIB=lib, SOKUTOU_B200_CHECK_BOUNDS="1")
    suites = ["tests/test_dit_gpu.py", "tests/test_layer_gpu.py", "tests/test_gate_gpu.py", "tests/test_decode_gpu.py",
              "tests/test_linear_gpu.py", "tests/test_decode_block_gpu.py", "tests/test_decode_grouped_gpu.py",
              "tests/test_zz_no_alloc.py"]
    r = subprocess.run([sys.executable, "-m", "pytest", *suites, "-m", "gpu", "-q", "-x", "-p", "no:cacheprovider",
                        "-k", "not greedy"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    tail = "\n".join((r.stdout + r.stderr).strip().splitlines()[-15:])
    assert r.returncode == 0, tail
    assert " passed" in tail and "failed" not in tail, tail
