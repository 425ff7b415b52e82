"""b2a_rmsnorm_rows (the prefill chunk's row norm, tensor.py:349-356 per
row: x * (1 / sqrt(x.x / n + eps)) * w) against NumPy on the same inputs.

The kernel sums the squares in double and rounds 1 / sqrt(mean + eps) to
f32, then forms (x * inv) * w in f32 as the reference does; the NumPy
reference does the same with a float64 sum, so f32 outputs agree to 1e-6
normwise and 16-bit outputs to one rounding of the output type.  Row
lengths cover the 16-byte-load kernel (1, 2 and 4 float4 per thread, a
ragged last float4 group) and the scalar kernel (lengths not a multiple of
4, rows longer than 4096), with padded row strides.
"""
import numpy as np
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _ref(x, w, eps):
    x64 = x.astype(np.float64)
    inv = np.float32(1.0 / np.sqrt((x64 * x64).sum(axis=1) / x.shape[1] + eps))
    return (x * inv[:, None]) * w[None, :]


@pytest.mark.parametrize("E", [1000, 2048, 3000, 4096, 257, 4098])
@pytest.mark.parametrize("dt,tol", [(torch.float32, 1e-6), (torch.float16, 2 ** -10),
                                    (torch.bfloat16, 2 ** -8)])
def test_rmsnorm_rows(cuda_dev, E, dt, tol):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    rng = np.random.default_rng(E)
    T, pad, eps = 37, 8, 1e-5
    x = (rng.standard_normal((T, E + pad)) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda_dev)
    wd = torch.from_numpy(w).to(cuda_dev)
    out = torch.zeros((T, E + pad), dtype=dt, device=cuda_dev)
    _lib.check(_lib.load().b2a_rmsnorm_rows(
        xd.data_ptr(), E + pad, wd.data_ptr(), eps, out.data_ptr(), E + pad, device._code(dt),
        T, E, None))
    torch.cuda.synchronize()
    got = out[:, :E].float().cpu().numpy()
    assert rel_err(got, _ref(x[:, :E], w, eps)) <= tol
    assert not out[:, E:].any()
