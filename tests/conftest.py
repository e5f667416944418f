import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "vllm-grinqh-plugin_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "grinqh_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def rel_errors(y, y_ref):
    """(max |y - ref| / max |ref|, ||y - ref||_F / ||ref||_F) in float64."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(y_ref, dtype=np.float64)
    d = np.abs(y - r)
    den = max(np.abs(r).max(), 1e-30)
    fro = np.linalg.norm(y - r) / max(np.linalg.norm(r), 1e-30)
    return d.max() / den, fro


# Parity bar for floating-point outputs (bf16/fp16 outputs vs the reference's own
# implementation on identical inputs): max-normalised error and relative Frobenius.
MAX_REL_TOL = 1e-2
FRO_TOL = 2e-3
