"""Fused RoPE + KV append vs the oracle (the reference's NumPy rotation and
cache-row stores).  fp32 results are required bit-identical; 16-bit cache
rows must equal the fp32 result rounded to nearest (torch's cast)."""
import numpy as np
import pytest
import torch

import oracle
from tests.golden import cases

pytestmark = pytest.mark.gpu


def _tab(n_ctx, n_rot, base, dev):
    cos, sin = oracle.rope_tables(n_ctx, n_rot, base)
    return cos, sin, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)


def test_rope_decode_dropin_bit_exact_config1(cuda_dev, golden):
    from alpacca_open_sourced_by_jt_b200 import kernels
    g = golden("decode_config1.npz")
    c = cases.decode_config1()
    cos, sin = oracle.rope_tables(c["L"], c["D"], c["base"])
    q = kernels.rope_decode(c["q_raw"].reshape(-1), cos[c["L"] - 1], sin[c["L"] - 1], c["H"],
                            c["D"], c["D"], "norm")
    assert np.array_equal(q, g["q_rot"])
    for i, p in enumerate(g["sample_rows"]):
        k = kernels.rope_decode(c["k_raw"][p].reshape(-1), cos[p], sin[p], c["KV"], c["D"],
                                c["D"], "norm")
        assert np.array_equal(k.reshape(c["KV"], c["D"]), g["k_rot_rows"][i])


def test_rope_neox_partial_bit_exact(cuda_dev, golden):
    from alpacca_open_sourced_by_jt_b200 import kernels
    g = golden("rope_neox.npz")
    c = cases.rope_neox()
    for i, p in enumerate(c["positions"]):
        out = kernels.rope_decode(c["q"][i].reshape(-1), g["cos_tab"][p], g["sin_tab"][p], c["H"],
                                  c["D"], c["n_rot"], "neox")
        assert np.array_equal(out, g["q_rot"][i])


@pytest.mark.parametrize("style", ["norm", "neox"])
@pytest.mark.parametrize("kv", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("per_sequence", [False, True])
def test_rope_append_fused(cuda_dev, style, kv, per_sequence):
    from alpacca_open_sourced_by_jt_b200 import device
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[kv]
    rng = np.random.default_rng(3)
    n, H, KV, D, n_rot, n_ctx = 6, 8, 2, 128, 96, 300
    cos, sin, ct, st = _tab(n_ctx, n_rot, 500000.0, cuda_dev)
    q = rng.standard_normal((n, H, D), dtype=np.float32)
    k = rng.standard_normal((n, KV, D), dtype=np.float32)
    v = rng.standard_normal((n, KV, D), dtype=np.float32)
    bq = rng.standard_normal(H * D, dtype=np.float32)
    bk = rng.standard_normal(KV * D, dtype=np.float32)
    bv = rng.standard_normal(KV * D, dtype=np.float32)
    pos = np.array([0, 1, 17, 100, 298, 299], np.int32)
    S = n if per_sequence else 1
    kc = torch.zeros((S, n_ctx, KV, D), dtype=tdt, device=cuda_dev)
    vc = torch.zeros_like(kc)
    qd = torch.from_numpy(q).to(cuda_dev)
    device.rope_append(qd, torch.from_numpy(k).to(cuda_dev), torch.from_numpy(v).to(cuda_dev),
                       torch.from_numpy(pos).to(cuda_dev), ct, st, k_cache=kc, v_cache=vc,
                       n_rot=n_rot, style=style, per_sequence=per_sequence,
                       bq=torch.from_numpy(bq).to(cuda_dev), bk=torch.from_numpy(bk).to(cuda_dev),
                       bv=torch.from_numpy(bv).to(cuda_dev))
    kref = np.zeros((S, n_ctx, KV, D), np.float32)
    vref = np.zeros_like(kref)
    qref = oracle.rope_append(q, k, v, pos, kref, vref, cos, sin, n_rot, style, bq, bk, bv,
                              seq_of_token=np.arange(n) if per_sequence else None)
    assert np.array_equal(qd.cpu().numpy(), qref)
    want_k = torch.from_numpy(kref).to(tdt)
    want_v = torch.from_numpy(vref).to(tdt)
    assert torch.equal(kc.cpu(), want_k)
    assert torch.equal(vc.cpu(), want_v)


def test_rope_append_packed_qk_in_place(cuda_dev):
    """The reference's packed qk row (q heads then k heads, cuda.py:723-786):
    q rotated in place inside the packed buffer, k taken from the same rows."""
    from alpacca_open_sourced_by_jt_b200 import _lib, device  # noqa: F401
    rng = np.random.default_rng(8)
    n, H, KV, D, n_ctx = 3, 4, 2, 64, 64
    cos, sin, ct, st = _tab(n_ctx, D, 10000.0, cuda_dev)
    qk = rng.standard_normal((n, (H + KV) * D), dtype=np.float32)
    v = rng.standard_normal((n, KV * D), dtype=np.float32)
    pos = np.array([5, 6, 7], np.int32)
    qkd = torch.from_numpy(qk).to(cuda_dev)
    kc = torch.zeros((1, n_ctx, KV, D), device=cuda_dev)
    vc = torch.zeros_like(kc)
    q_view = qkd.as_strided((n, H, D), ((H + KV) * D, D, 1))
    k_view = qkd.as_strided((n, KV, D), ((H + KV) * D, D, 1), H * D)
    device.rope_append(q_view, k_view, torch.from_numpy(v).to(cuda_dev).view(n, KV, D),
                       torch.from_numpy(pos).to(cuda_dev), ct, st, k_cache=kc, v_cache=vc)
    kref = np.zeros((1, n_ctx, KV, D), np.float32)
    vref = np.zeros_like(kref)
    qref = oracle.rope_append(qk[:, :H * D].reshape(n, H, D), qk[:, H * D:].reshape(n, KV, D),
                              v.reshape(n, KV, D), pos, kref, vref, cos, sin, D, "norm")
    got = qkd.cpu().numpy()
    assert np.array_equal(got[:, :H * D].reshape(n, H, D), qref)
    assert np.array_equal(got[:, H * D:], qk[:, H * D:])  # k part of the row untouched
    assert np.array_equal(kc.cpu().numpy(), kref)
    assert np.array_equal(vc.cpu().numpy(), vref)


def test_rope_append_bf16_q_out(cuda_dev):
    """Prefill-chunk form: rotated q written to a separate bf16 buffer."""
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(10)
    n, H, KV, D, n_ctx = 130, 8, 2, 128, 200
    cos, sin, ct, st = _tab(n_ctx, D, 500000.0, cuda_dev)
    q = rng.standard_normal((n, H, D), dtype=np.float32)
    k = rng.standard_normal((n, KV, D), dtype=np.float32)
    v = rng.standard_normal((n, KV, D), dtype=np.float32)
    pos = np.arange(50, 50 + n, dtype=np.int32)
    kc = torch.zeros((n_ctx, KV, D), dtype=torch.bfloat16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    qo = torch.empty((n, H, D), dtype=torch.bfloat16, device=cuda_dev)
    qd = torch.from_numpy(q).to(cuda_dev)
    device.rope_append(qd, torch.from_numpy(k).to(cuda_dev), torch.from_numpy(v).to(cuda_dev),
                       torch.from_numpy(pos).to(cuda_dev), ct, st, k_cache=kc, v_cache=vc,
                       q_out=qo)
    kref = np.zeros((1, n_ctx, KV, D), np.float32)
    vref = np.zeros_like(kref)
    qref = oracle.rope_append(q, k, v, pos, kref, vref, cos, sin, D, "norm")
    assert torch.equal(qo.cpu(), torch.from_numpy(qref).to(torch.bfloat16))
    assert np.array_equal(qd.cpu().numpy(), q)  # input q untouched
    assert torch.equal(kc.cpu(), torch.from_numpy(kref[0]).to(torch.bfloat16))


def test_imrope_append_matches_reference(cuda_dev, golden):
    from alpacca_open_sourced_by_jt_b200 import device
    g = golden("qwen35.npz")
    r = cases.imrope_case()
    x = r["x"]  # 3 tokens x 3 heads x 128
    n, H, D = x.shape
    # heads 0,1 as q, head 2 as a single KV head
    q = torch.from_numpy(np.ascontiguousarray(x[:, :2])).to(cuda_dev)
    k = torch.from_numpy(np.ascontiguousarray(x[:, 2:])).to(cuda_dev)
    v = torch.from_numpy(np.ascontiguousarray(x[:, 2:] * 2)).to(cuda_dev)
    kc = torch.zeros((1, 32, 1, D), device=cuda_dev)
    vc = torch.zeros_like(kc)
    pos = torch.tensor([0, 17, 5], dtype=torch.int32, device=cuda_dev)
    qo = device.imrope_append(q, k, v, torch.from_numpy(r["lanes"]).to(cuda_dev), pos,
                              r["sections"], k_cache=kc, v_cache=vc, freq_base=r["base"])
    want = g["imrope_out"].astype(np.float32)  # reference in double, rounded to f32
    got_q = qo.cpu().numpy()
    got_k = kc.cpu().numpy()[0, [0, 17, 5], 0]
    assert np.abs(got_q - want[:, :2]).max() <= 1e-6 * np.abs(want).max()
    assert np.abs(got_k - want[:, 2]).max() <= 1e-6 * np.abs(want).max()
    assert np.array_equal(vc.cpu().numpy()[0, [0, 17, 5], 0], x[:, 2] * 2)


def test_position_outside_cache_writes_nothing(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    _lib.device_error(clear=True)
    n_ctx, KV, D = 16, 2, 64
    cos, sin, ct, st = _tab(n_ctx, D, 10000.0, cuda_dev)
    q = torch.randn((2, 4, D), device=cuda_dev)
    k = torch.randn((2, KV, D), device=cuda_dev)
    v = torch.randn((2, KV, D), device=cuda_dev)
    kc = torch.zeros((1, n_ctx, KV, D), device=cuda_dev)
    vc = torch.zeros_like(kc)
    pos = torch.tensor([3, n_ctx], dtype=torch.int32, device=cuda_dev)  # second is out of range
    device.rope_append(q, k, v, pos, ct, st, k_cache=kc, v_cache=vc)
    code, aux = _lib.device_error(clear=True)
    assert code == _lib.ERR_POSITION and aux == 1
    assert kc[0, 3].abs().sum().item() > 0  # the valid token was stored
    assert kc[0, 4:].abs().sum().item() == 0 and vc[0, 4:].abs().sum().item() == 0
