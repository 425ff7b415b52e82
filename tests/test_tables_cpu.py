"""Host-side RoPE table builder of the package vs the reference's tables.

The tables are inputs of the fused RoPE + append kernel, so they must equal
the reference's (alpaccaroo/model.py:318-323, :871-875) bit for bit: checked
against the golden tables written by the reference itself and against the
oracle's restatement for other bases, widths and frequency scales.
"""
import numpy as np
import pytest
import torch

import oracle
from alpacca_open_sourced_by_jt_b200 import device
from tests.golden import cases


def test_tables_equal_reference_golden(golden):
    g = golden("decode_config1.npz")
    cos, sin = device.rope_tables(512, 64, 500000.0, device="cpu")
    rows = g["sample_rows"]
    assert np.array_equal(cos.numpy()[rows], g["cos_tab"])
    assert np.array_equal(sin.numpy()[rows], g["sin_tab"])
    g = golden("rope_neox.npz")
    c = cases.rope_neox()
    cos, sin = device.rope_tables(c["n_ctx"], c["n_rot"], c["base"], device="cpu")
    assert np.array_equal(cos.numpy(), g["cos_tab"])
    assert np.array_equal(sin.numpy(), g["sin_tab"])


@pytest.mark.parametrize("n_ctx,n_rot,base,scale", [
    (4096, 128, 500000.0, 1.0), (300, 96, 10000.0, 1.0), (1000, 64, 1e6, 0.25),
    (33, 2, 10000.0, 1.0)])
def test_tables_equal_oracle(n_ctx, n_rot, base, scale):
    cos, sin = device.rope_tables(n_ctx, n_rot, base, scale, device="cpu")
    rc, rs = oracle.rope_tables(n_ctx, n_rot, base, scale)
    assert cos.dtype == torch.float32 and cos.shape == (n_ctx, n_rot // 2)
    assert np.array_equal(cos.numpy(), rc) and np.array_equal(sin.numpy(), rs)


def test_odd_rotary_width_rejected():
    from alpacca_open_sourced_by_jt_b200 import _lib
    with pytest.raises(_lib.B2AShapeError):
        device.rope_tables(16, 7, 10000.0, device="cpu")
