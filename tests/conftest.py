"""Shared fixtures.  `-m gpu` tests need a B200 and the built library;
`-m "not gpu"` tests run anywhere (oracle, golden vectors, host logic,
C-ABI load/export/argument checks)."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and libb2attn.so")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from alpacca_open_sourced_by_jt_b200 import build
    build.build()
    from alpacca_open_sourced_by_jt_b200 import _lib
    _lib.load()
    _lib.device_error(clear=True)
    return torch.device("cuda", 0)


def rel_err(a, b):
    """Max relative error, normwise: max|a - b| / max|b|.

    This is the measure the fp32 parity bar (1e-4) is stated in.  An
    elementwise ratio is not used: two float32 evaluations of the same
    softmax (even the reference's own NumPy paths) differ by a few ulps of
    the output scale, which an elementwise ratio inflates without bound on
    outputs near zero."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def max_abs_err(a, b):
    """max|a - b|: the measure of the 16-bit KV parity bar (2e-2 on
    unit-variance outputs)."""
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())
