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


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Floor audit of the per-element 16-bit checks run in this session: how
    many elements passed only through the row-RMS floor, the |A||B| floor or
    the attention rounding-flip allowance (oracle.elementwise_rel_check)."""
    try:
        from tests.gpu_util import FLOOR_AUDIT
    except Exception:  # pragma: no cover - helper import failed earlier
        return
    if not FLOOR_AUDIT:
        return
    keys = ("n", "n_row_floor", "n_absprod_floor", "n_allowance")
    tot = {k: sum(int(st.get(k, 0)) for _, st in FLOOR_AUDIT) for k in keys}
    worst = max(FLOOR_AUDIT, key=lambda t: t[1].get("max_rel_floored", 0.0))
    tr = terminalreporter
    tr.write_sep("-", "16-bit parity floor audit")
    tr.write_line(f"checks {len(FLOOR_AUDIT)}, elements {tot['n']}: passed through the row-RMS "
                  f"floor {tot['n_row_floor']}, the |A||B| floor {tot['n_absprod_floor']}, the "
                  f"rounding-flip allowance {tot['n_allowance']}")
    tr.write_line(f"largest error against the floored bar: {worst[1]['max_rel_floored']:.3e} "
                  f"({worst[0]})")
