import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def ops():
    """The drop-in module; importing it loads libsf_engine.so (no fallback)."""
    from scaffolding_b200 import _cuda_ops
    return _cuda_ops


@pytest.fixture(scope="session")
def gpu(ops):
    """Session guard for GPU tests: fail loudly (never skip) without a device."""
    n = ops.get_device_count()
    assert n > 0, "GPU tests need a CUDA device; run them with -m gpu on a B200"
    major, minor = ops.get_device_capability(0)
    assert (major, minor) == (10, 0), f"expected sm_100 (B200), got sm_{major}{minor}"
    ops.set_device(0)
    return 0
