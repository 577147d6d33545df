import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

# Tolerances for floating-point FFN outputs against the fp32 oracle.
MAX_ABS_TOL = 2e-2
REL_L2_TOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


def rel_l2(a, b):
    import numpy as np

    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_ffn_close(got, ref, max_abs=MAX_ABS_TOL, rel=REL_L2_TOL, what=""):
    import numpy as np

    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    ma = float(np.abs(got - ref).max()) if got.size else 0.0
    rl = rel_l2(got, ref) if got.size else 0.0
    assert ma <= max_abs and rl <= rel, f"{what}: max_abs={ma:.3e} (tol {max_abs}) rel_l2={rl:.3e} (tol {rel})"


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(REPO, "tests", "golden")
