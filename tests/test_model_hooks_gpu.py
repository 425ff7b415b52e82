"""model_hooks.install on a model object: the engine-facing drop-in.

The stand-in carries exactly what the hooked methods read from an
alpaccaroo Model (alpaccaroo/model.py:299-328, 849-882): `hp` (n_head, n_kv,
head_dim, n_rot, rope_style) and the f32 `_rope_cos` / `_rope_sin` tables,
built the way the reference builds them (pinned bit for bit to the
reference's golden tables).  Its class methods are the oracle's NumPy
restatements, so uninstall() can be checked to bring them back.  The
expected values are the reference's own goldens.
"""
import math
import types

import numpy as np
import pytest

import oracle
from tests.conftest import rel_err
from tests.golden import cases

pytestmark = pytest.mark.gpu


class StandInModel:
    """The attributes and methods of alpaccaroo.model.Model that the
    hooks touch (model.py:1191-1272, 1567-1592), with NumPy bodies."""

    def __init__(self, n_head, n_kv, head_dim, n_rot, base, style, n_ctx):
        self.hp = types.SimpleNamespace(n_head=n_head, n_kv=n_kv, head_dim=head_dim,
                                        n_rot=n_rot, rope_style=style)
        self._rope_cos, self._rope_sin = oracle.rope_tables(n_ctx, n_rot, base)

    def _attention_np(self, q, K, V, group, inv_sqrt):
        return oracle.attention_decode(q, K, V, group, inv_sqrt)

    def _attention_batch_np(self, q, K, V, positions, group, inv_sqrt):
        return oracle.attention_batch(q, K, V, positions, group, inv_sqrt)

    def _attention_batch_window_np(self, q, K, V, positions, group, inv_sqrt, window=0,
                                   kv_start=0):
        return oracle.attention_batch(q, K, V, positions, group, inv_sqrt, window, kv_start)

    def _rope_np(self, vec, n_heads, pos):
        hp = self.hp
        return oracle.rope_vec(vec, n_heads, pos, self._rope_cos, self._rope_sin, hp.head_dim,
                               hp.n_rot, hp.rope_style)

    def _rope_batch_np(self, vecs, n_heads, positions):
        hp = self.hp
        return oracle.rope_batch(vecs, n_heads, positions, self._rope_cos, self._rope_sin,
                                 hp.head_dim, hp.n_rot, hp.rope_style)


def test_config1_decode_steps_through_hooks(cuda_dev, golden):
    """benchmark config 1 as the engine runs it: each cached K row rotated by
    the hooked _rope_np at its position, the query at 511, then the hooked
    _attention_np over the cache, plus a few earlier decode steps."""
    from alpacca_open_sourced_by_jt_b200 import model_hooks
    g = golden("decode_config1.npz")
    c = cases.decode_config1()
    m = StandInModel(c["H"], c["KV"], c["D"], c["D"], c["base"], "norm", c["L"])
    model_hooks.install(m)
    assert m._b2a_installed
    K = np.empty_like(c["k_raw"])
    for p in range(c["L"]):
        K[p] = m._rope_np(c["k_raw"][p].reshape(-1), c["KV"], p).reshape(c["KV"], c["D"])
    rows = g["sample_rows"]
    assert np.array_equal(K[rows], g["k_rot_rows"])  # bit-exact RoPE
    q = m._rope_np(c["q_raw"].reshape(-1), c["H"], c["L"] - 1)
    assert np.array_equal(q, g["q_rot"])
    out = m._attention_np(q, K, c["v"], c["H"] // c["KV"], 1.0 / math.sqrt(c["D"]))
    assert out.shape == (c["H"], c["D"])
    assert rel_err(out, g["out"]) < 1e-4
    # decode steps at shorter lengths, each over the cache rows [0, p]
    for p in (0, 1, 63, 300):
        qp = m._rope_np(c["q_raw"].reshape(-1), c["H"], p)
        got = m._attention_np(qp, K[:p + 1], c["v"][:p + 1], c["H"] // c["KV"], 0.125)
        want = oracle.attention_decode(qp, K[:p + 1], c["v"][:p + 1], c["H"] // c["KV"], 0.125)
        assert rel_err(got, want) < 1e-4
    model_hooks.uninstall(m)
    assert not m._b2a_installed
    assert m._attention_np.__func__ is StandInModel._attention_np


def test_neox_batch_rope_through_hooks(cuda_dev, golden):
    from alpacca_open_sourced_by_jt_b200 import model_hooks
    g = golden("rope_neox.npz")
    c = cases.rope_neox()
    m = StandInModel(c["H"], c["KV"], c["D"], c["n_rot"], c["base"], "neox", c["n_ctx"])
    model_hooks.install(m)
    k = m._rope_batch_np(c["k"].reshape(len(c["positions"]), -1), c["KV"], c["positions"])
    assert np.array_equal(k, g["k_rot"])
    q = np.stack([m._rope_np(c["q"][i].reshape(-1), c["H"], int(p))
                  for i, p in enumerate(c["positions"])])
    assert np.array_equal(q, g["q_rot"])


def test_prefill_hooks_including_head_dim_256(cuda_dev, golden):
    """The prefill hooks on the reference's goldens, among them gemma3's
    window variant at head_dim 256, which the reference's GPU tier declines
    and the hooks now serve on the GPU at the fp32 bar."""
    from alpacca_open_sourced_by_jt_b200 import model_hooks
    g = golden("prefill_small.npz")
    c = cases.prefill_small()
    m = StandInModel(c["H"], c["KV"], c["D"], c["D"], 10000.0, "norm", 64)
    model_hooks.install(m)
    out = m._attention_batch_np(c["q"], c["k"], c["v"], c["positions"], c["H"] // c["KV"],
                                1.0 / math.sqrt(c["D"]))
    assert rel_err(out, g["out"]) < 1e-4
    w = cases.prefill_window()
    outw = m._attention_batch_window_np(w["q"], w["k"], w["v"], w["positions"],
                                        w["H"] // w["KV"], 1.0 / math.sqrt(w["D"]),
                                        w["window"], w["kv_start"])
    assert rel_err(outw, g["out_window"]) < 1e-4
    gm = golden("prefill_more.npz")
    d = cases.prefill_gemma3_window_d256()
    m256 = StandInModel(d["H"], d["KV"], d["D"], d["D"], 10000.0, "norm", 128)
    model_hooks.install(m256)
    out = m256._attention_batch_window_np(d["q"], d["k"], d["v"], d["positions"],
                                          d["H"] // d["KV"], 1.0 / math.sqrt(d["D"]),
                                          d["window"], d["kv_start"])
    assert rel_err(out, gm["window_d256"]) < 1e-4
    # a head_dim no kernel serves (6: not a multiple of 4) is declined by
    # cuda.attention_batch, as the reference's GPU tier declines, and the
    # model's own (class) method answers, as it does in the reference
    m6 = StandInModel(2, 1, 6, 6, 10000.0, "norm", 8)
    model_hooks.install(m6)
    rng = np.random.default_rng(6)
    args = (rng.standard_normal((2, 2, 6)).astype(np.float32),
            rng.standard_normal((2, 1, 6)).astype(np.float32),
            rng.standard_normal((2, 1, 6)).astype(np.float32), np.array([0, 1], np.int32), 2, 0.4)
    from alpacca_open_sourced_by_jt_b200 import cuda as b200_cuda
    assert b200_cuda.attention_batch(*args) is None
    got = m6._attention_batch_np(*args)
    assert np.array_equal(got, StandInModel._attention_batch_np(m6, *args))
    gotw = m6._attention_batch_window_np(*args, 1, 0)
    assert np.array_equal(gotw, StandInModel._attention_batch_window_np(m6, *args, 1, 0))
