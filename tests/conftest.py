"""Shared test set-up: import paths, the `gpu` marker, fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "quantr-in-c_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "quant_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def qr_gpu():
    """The CUDA library, initialised on device 0; fails loudly without it."""
    import quantr
    L = quantr.lib()
    rc = L.quantr_gpu_init(0)
    assert rc == 0, f"quantr_gpu_init failed: {rc}"
    L.quantr_gpu_clear_error()
    return quantr
