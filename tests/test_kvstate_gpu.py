"""KV state boundary on the GPU.

* b2a_kv_convert against torch's host conversions, bit for bit: exact
  widening, round-to-nearest-even narrowing, every dtype pair, counts that
  are not a multiple of the vector width, misaligned views, and special
  values.
* DeviceAttentionState snapshots against the bytes the reference's own
  FullAttentionState produced (tests/golden/kv_state.npz), truncate, and
  snapshot -> restore round trips for 16-bit caches.
* DeviceMirror: valid_upto, invalidate, sync and fetch with the semantics
  of the reference's chain mirror (alpaccaroo/cuda.py:1875-1900, 2046-2061).
"""
import numpy as np
import pytest
import torch

from tests.golden import cases

pytestmark = pytest.mark.gpu

DTS = [torch.float32, torch.float16, torch.bfloat16]


def _special(n, rng):
    x = rng.standard_normal(n).astype(np.float32) * 3
    sp = np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 1e-8, -1e-8, 3.0e38, 6e-5,
                   1.0 + 2 ** -9, 1.0 + 3 * 2 ** -9], np.float32)
    k = min(n, sp.size)
    x[:k] = sp[:k]
    return x


@pytest.mark.parametrize("src_dt", DTS)
@pytest.mark.parametrize("dst_dt", DTS)
@pytest.mark.parametrize("n,off", [(1, 0), (8 * 1000 + 5, 0), (4097, 1), (100003, 3)])
def test_kv_convert_bit_exact(cuda_dev, src_dt, dst_dt, n, off):
    from alpacca_open_sourced_by_jt_b200.kvstate import convert
    rng = np.random.default_rng(n + off)
    src_host = torch.from_numpy(_special(n + off, rng)).to(src_dt)
    src = src_host.to(cuda_dev)[off:]
    dst = torch.full((n + off,), 7.0, dtype=dst_dt, device=cuda_dev)[off:]
    convert(src, dst)
    torch.cuda.synchronize()
    want = src_host[off:].to(torch.float32).to(dst_dt) if src_dt != torch.float32 else \
        src_host[off:].to(dst_dt)
    got = dst.cpu()
    assert torch.equal(got.view(torch.int16 if dst_dt != torch.float32 else torch.int32),
                       want.view(torch.int16 if dst_dt != torch.float32 else torch.int32))


def test_kv_convert_rejects_overlap_and_bad_dtype(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib
    lib = _lib.load()
    buf = torch.zeros(64, dtype=torch.float32, device=cuda_dev)
    assert lib.b2a_kv_convert(buf.data_ptr(), _lib.F32, buf.data_ptr() + 16, _lib.F32, 32,
                              None) == _lib.ERR_ARG
    assert lib.b2a_kv_convert(buf.data_ptr(), 9, buf[32:].data_ptr(), _lib.F32, 8,
                              None) == _lib.ERR_DTYPE


def _state_from_case(dtype, dev, n_ctx=64):
    from alpacca_open_sourced_by_jt_b200.kvstate import DeviceAttentionState
    c = cases.kv_state_case()
    st = DeviceAttentionState(c["layer_index"], c["KV"], c["D"], c["D"], n_ctx, dtype, dev)
    for p in range(c["L"]):  # one row at a time, as the reference appends
        st.append(c["k"][p].ravel(), c["v"][p].ravel())
    return st, c


def test_f32_snapshot_equals_reference_bytes(cuda_dev, golden):
    g = golden("kv_state.npz")
    st, c = _state_from_case(torch.float32, cuda_dev)
    s = st.snapshot()
    assert s.logical_length == int(g["length"]) and s.dtype == str(g["dtype"])
    assert s.key == g["key"].tobytes() and s.value == g["value"].tobytes()
    assert st.memory_bytes() == int(g["memory_bytes"]) == s.memory_bytes()
    st.truncate(c["truncate"])
    s = st.snapshot()
    assert s.logical_length == int(g["length_cut"])
    assert s.key == g["key_cut"].tobytes() and s.value == g["value_cut"].tobytes()
    assert st.memory_bytes() == int(g["memory_bytes_cut"])
    with pytest.raises(ValueError):
        st.truncate(c["truncate"] + 1)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_16bit_snapshot_widens_and_round_trips(cuda_dev, golden, dtype):
    from alpacca_open_sourced_by_jt_b200.kvstate import DeviceAttentionState
    g = golden("kv_state.npz")
    st, c = _state_from_case(dtype, cuda_dev)
    s = st.snapshot()
    # the snapshot holds the stored 16-bit rows widened exactly to f32
    k16 = torch.from_numpy(c["k"]).to(dtype).to(torch.float32).numpy()
    assert s.key == k16.astype("<f4").tobytes()
    # restoring the reference's own f32 record narrows it the same way
    ref = type(s)(layer_index=c["layer_index"], logical_length=int(g["length"]),
                  kv_heads=c["KV"], key_dim=c["D"], value_dim=c["D"],
                  key=g["key"].tobytes(), value=g["value"].tobytes())
    back = DeviceAttentionState.from_snapshot(ref, 64, dtype, cuda_dev)
    assert torch.equal(back.key[:c["L"]], st.key[:c["L"]])
    assert torch.equal(back.value[:c["L"]], st.value[:c["L"]])
    # and a 16-bit snapshot restores bit-exactly
    again = DeviceAttentionState.from_snapshot(s, 64, dtype, cuda_dev)
    assert again.snapshot() == s
    cl = st.clone()
    assert cl.snapshot() == s


def test_mirror_sync_invalidate_fetch(cuda_dev):
    from alpacca_open_sourced_by_jt_b200.kvstate import DeviceMirror
    rng = np.random.default_rng(5)
    n_ctx, KV, D, layers = 40, 2, 32, 3
    hk = [rng.standard_normal((n_ctx, KV, D), dtype=np.float32) for _ in range(layers)]
    hv = [rng.standard_normal((n_ctx, KV, D), dtype=np.float32) for _ in range(layers)]
    m = DeviceMirror(hk, hv, torch.bfloat16, cuda_dev)

    def rounded(a):
        return torch.from_numpy(a).to(torch.bfloat16)

    m.sync(10)
    assert m.valid_upto == 10
    for li in range(layers):
        assert torch.equal(m.k[li][:10].cpu(), rounded(hk[li][:10]))
        assert torch.equal(m.v[li][:10].cpu(), rounded(hv[li][:10]))
    old = m.k[0][:5].clone()
    for li in range(layers):  # a host mutation of rows 5.. (e.g. a prefix restart)
        hk[li][5:12] += 1.0
    m.invalidate(5)
    assert m.valid_upto == 5
    m.invalidate(30)  # beyond the mirrored prefix: no change
    assert m.valid_upto == 5
    m.sync(12)
    assert m.valid_upto == 12
    assert torch.equal(m.k[0][:5], old)
    for li in range(layers):
        assert torch.equal(m.k[li][:12].cpu(), rounded(hk[li][:12]))
    # rows computed on the device come home widened
    for li in range(layers):
        m.k[li][12:20] = torch.randn((8, KV, D), device=cuda_dev).to(torch.bfloat16)
    m.fetch(12, 20)
    for li in range(layers):
        assert np.array_equal(hk[li][12:20], m.k[li][12:20].float().cpu().numpy())
