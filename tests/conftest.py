import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_data.npz"

# Parity bars: max|y - y_ref| / max|y_ref| (norm-relative), per weight width.
# fp16/fp32 weights 2e-3, int8/int4 after identical dequantisation 5e-3.
TOL = {32: 2e-3, 16: 2e-3, 8: 5e-3, 4: 5e-3}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


def rel_err(y, ref) -> float:
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def assert_close(y, ref, tol, what=""):
    e = rel_err(y, ref)
    assert np.all(np.isfinite(y)), f"{what}: non-finite output"
    assert e <= tol, f"{what}: norm-relative error {e:.3e} > {tol:.1e}"
    return e
