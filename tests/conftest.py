import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    n = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (n if n > 0 else 1.0))


@pytest.fixture(scope="session")
def native_lib():
    """The built shared library (builds it in-tree if needed)."""
    from sokutou_b200 import build
    build.build()
    from sokutou_b200 import _lib
    return _lib.lib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    from sokutou_b200 import build
    build.build()
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _no_bounds_error(request):
    """Under SOKUTOU_B200_CHECK_BOUNDS=1 (the bounds-checked library's run), every GPU test must leave
    no SK_DEVERR_BOUNDS in the device error word."""
    yield
    if os.environ.get("SOKUTOU_B200_CHECK_BOUNDS") == "1" and "gpu" in request.keywords:
        from sokutou_b200 import ops
        code = ops.device_error(reset=True)
        assert code != 3, f"an index out of its buffer in {request.node.name} (SK_DEVERR_BOUNDS)"
