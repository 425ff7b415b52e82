"""tcgen05 causal prefill vs the oracle (the reference's NumPy einsum path).

The kernel takes 16-bit q/K/V and accumulates in fp32 (P is rounded to 16
bits for the second MMA).  The oracle runs in fp32 on the same 16-bit
inputs; the bar is 2e-2 max abs error on unit-variance outputs.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import max_abs_err, rel_err
from tests.golden import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["head", "pair", "single"])
def kernel(request, monkeypatch):
    """Run a test on every prefill kernel: the paired-head persistent kernel
    (default for even GQA groups), the one-head persistent kernel (default
    for odd groups) and the non-persistent one-tile kernel."""
    if request.param == "pair":
        monkeypatch.delenv("B2ATTN_PREFILL", raising=False)
    else:
        monkeypatch.setenv("B2ATTN_PREFILL", request.param)
    return request.param


def _run(T, t_kv, H, KV, D, dt, dev, positions=None, window=0, kv_start=0, out_dtype=None,
         seed=0):
    from alpacca_open_sourced_by_jt_b200 import device
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((T, H, D), generator=g).to(dt)
    k = torch.randn((t_kv, KV, D), generator=g).to(dt)
    v = torch.randn((t_kv, KV, D), generator=g).to(dt)
    if positions is None:
        positions = np.arange(kv_start + t_kv - T, kv_start + t_kv, dtype=np.int32)
    pos = torch.from_numpy(np.asarray(positions, np.int32))
    out = device.prefill(q.to(dev), k.to(dev), v.to(dev), pos.to(dev), window=window,
                         kv_start=kv_start, out_dtype=out_dtype or torch.float32)
    torch.cuda.synchronize()
    ref = oracle.attention_batch(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                 np.asarray(positions, np.int32), H // KV, 1 / math.sqrt(D),
                                 window, kv_start)
    return out.float().cpu().numpy().reshape(T, -1), ref


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("T", [1, 77, 128, 300])
def test_causal_from_zero(cuda_dev, kernel, dt, D, T):
    out, ref = _run(T, T, 8, 2, D, dt, cuda_dev, seed=T)
    assert max_abs_err(out, ref) < 2e-2


@pytest.mark.parametrize("group", [1, 2, 3, 4, 8])
def test_gqa_groups_with_prefix(cuda_dev, kernel, group):
    # a 200-token chunk after a 333-token prefix: 533 keys, queries at 333..532
    out, ref = _run(200, 533, 2 * group, 2, 128, torch.bfloat16, cuda_dev, seed=group)
    assert max_abs_err(out, ref) < 2e-2


def test_window_and_kv_start(cuda_dev, kernel):
    out, ref = _run(150, 260, 8, 2, 64, torch.bfloat16, cuda_dev,
                    positions=np.arange(200, 350, dtype=np.int32), window=64, kv_start=100)
    assert max_abs_err(out, ref) < 2e-2


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_16bit_output(cuda_dev, kernel, out_dtype):
    out, ref = _run(256, 256, 4, 1, 128, torch.bfloat16, cuda_dev, out_dtype=out_dtype)
    assert max_abs_err(out, ref) < 2e-2


def test_config2_shape(cuda_dev, kernel):
    """benchmark config 2 geometry (S=2048, 32/8 heads, D=128, bf16, bf16 out)
    against the oracle on a subset of heads' rows (the oracle's fp32 einsum
    over all 32 heads x 2048^2 scores is too slow for a unit test)."""
    from alpacca_open_sourced_by_jt_b200 import device
    S, H, KV, D = 2048, 32, 8, 128
    g = torch.Generator().manual_seed(1)
    q = torch.randn((S, H, D), generator=g).to(torch.bfloat16)
    k = torch.randn((S, KV, D), generator=g).to(torch.bfloat16)
    v = torch.randn((S, KV, D), generator=g).to(torch.bfloat16)
    pos = torch.arange(S, dtype=torch.int32)
    out = device.prefill(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), pos.to(cuda_dev))
    out = out.float().cpu().numpy()
    rows = np.r_[0:3, 127:130, 1000:1003, 2040:2048]
    kvh = 3
    ref = oracle.attention_batch(q[rows][:, kvh * 4:(kvh + 1) * 4].float().numpy(),
                                 k[:, kvh:kvh + 1].float().numpy(), v[:, kvh:kvh + 1].float().numpy(),
                                 rows.astype(np.int32), 4, 1 / math.sqrt(D))
    got = out[rows][:, kvh * 4:(kvh + 1) * 4].reshape(len(rows), -1)
    assert max_abs_err(got, ref) < 2e-2


def test_determinism(cuda_dev, kernel):
    from alpacca_open_sourced_by_jt_b200 import device
    q = torch.randn((384, 8, 128), device=cuda_dev, dtype=torch.bfloat16)
    k = torch.randn((384, 2, 128), device=cuda_dev, dtype=torch.bfloat16)
    v = torch.randn((384, 2, 128), device=cuda_dev, dtype=torch.bfloat16)
    pos = torch.arange(384, dtype=torch.int32, device=cuda_dev)
    a = device.prefill(q, k, v, pos)
    b = device.prefill(q, k, v, pos)
    assert torch.equal(a, b)


def test_golden_through_attention_batch_dropin(cuda_dev, golden):
    """The reference's cuda.attention_batch signature on the reference's own
    golden cases: fp32 host inputs run the fp32 kernel and meet the fp32 bar
    (1e-4 max relative error, normwise)."""
    from alpacca_open_sourced_by_jt_b200 import cuda
    g = golden("prefill_small.npz")
    c = cases.prefill_small()
    out = cuda.attention_batch(c["q"], c["k"], c["v"], c["positions"], c["H"] // c["KV"],
                               1 / math.sqrt(c["D"]))
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < 1e-4
    w = cases.prefill_window()
    outw = cuda.attention_batch(w["q"], w["k"], w["v"], w["positions"], w["H"] // w["KV"],
                                1 / math.sqrt(w["D"]), w["window"], w["kv_start"])
    assert rel_err(outw, g["out_window"]) < 1e-4
    # a geometry outside the kernels' set is declined like the reference
    # (None: the caller keeps its own path), not faked
    for hd in (260, 6):
        assert cuda.attention_batch(np.zeros((2, 2, hd), np.float32),
                                    np.zeros((2, 1, hd), np.float32),
                                    np.zeros((2, 1, hd), np.float32),
                                    np.array([0, 1], np.int32), 2, 0.0625) is None


def test_golden_more_through_dropins(cuda_dev, golden):
    """Reference-run goldens: gemma3's window variant at head_dim 256, rows
    with no visible key (the NumPy path's mean of V), and fp32 values beyond
    fp16's range, all at the fp32 bar."""
    from alpacca_open_sourced_by_jt_b200 import cuda
    g = golden("prefill_more.npz")
    for name, case in (("window_d256", cases.prefill_gemma3_window_d256()),
                       ("empty_rows", cases.prefill_empty_rows())):
        assert case["sha256"] == str(g[name + "_sha256"])
        out = cuda.attention_batch(case["q"], case["k"], case["v"], case["positions"],
                                   case["H"] // case["KV"], 1 / math.sqrt(case["D"]),
                                   case["window"], case["kv_start"])
        assert rel_err(out, g[name]) < 1e-4, name
    b = cases.prefill_large_magnitude()
    out = cuda.attention_batch(b["q"], b["k"], b["v"], b["positions"], b["H"] // b["KV"],
                               1 / math.sqrt(b["D"]))
    assert np.isfinite(out).all()
    assert rel_err(out, g["large"]) < 1e-4


def test_qwen35_dropins(cuda_dev, golden):
    from alpacca_open_sourced_by_jt_b200 import qwen35_kernels as q35
    g = golden("qwen35.npz")
    c = cases.qwen35_decode()
    assert rel_err(q35.qwen35_full_attention_decode(c["q"], c["k"], c["v"]), g["decode_out"]) < 1e-4
    p = cases.qwen35_prefill()
    out = q35.qwen35_full_attention_prefill(p["q"], p["k"], p["v"], p["prefix"])
    assert rel_err(out, g["prefill_out"]) < 1e-4
    # Qwen35's key_length 256 with a prefix (the reference serves any head_dim)
    m = golden("prefill_more.npz")
    d = cases.prefill_qwen35_d256()
    out = q35.qwen35_full_attention_prefill(d["q"], d["k"], d["v"], d["prefix"])
    assert out.shape == m["qwen35_d256"].shape
    assert rel_err(out, m["qwen35_d256"]) < 1e-4


# ---------------------------------------------------------------------------
# fp32 kernel (fp32 inputs): the fp32 bar, any head_dim multiple of 4 <= 256
# ---------------------------------------------------------------------------

def _run_f32(T, t_kv, H, KV, D, dev, positions=None, window=0, kv_start=0, seed=0, scale_q=1.0,
             out_dtype=torch.float32):
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(seed)
    q = (scale_q * rng.standard_normal((T, H, D))).astype(np.float32)
    k = rng.standard_normal((t_kv, KV, D), dtype=np.float32)
    v = rng.standard_normal((t_kv, KV, D), dtype=np.float32)
    if positions is None:
        positions = np.arange(kv_start + t_kv - T, kv_start + t_kv, dtype=np.int32)
    positions = np.asarray(positions, np.int32)
    out = device.prefill(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                         torch.from_numpy(v).to(dev), torch.from_numpy(positions).to(dev),
                         window=window, kv_start=kv_start, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = oracle.attention_batch(q, k, v, positions, H // KV, 1 / math.sqrt(D), window, kv_start)
    return out.float().cpu().numpy().reshape(T, -1), ref


@pytest.mark.parametrize("D", [4, 36, 64, 80, 96, 128, 200, 256])
@pytest.mark.parametrize("T", [1, 63, 130])
def test_f32_causal_head_dims(cuda_dev, D, T):
    out, ref = _run_f32(T, T + 17, 8, 2, D, cuda_dev, seed=D + T)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("group", [1, 3, 4, 8])
def test_f32_gqa_window_kv_start(cuda_dev, group):
    out, ref = _run_f32(150, 260, 2 * group, 2, 128, cuda_dev,
                        positions=np.arange(200, 350, dtype=np.int32), window=64, kv_start=100,
                        seed=group)
    assert rel_err(out, ref) < 1e-4


def test_f32_any_position_order(cuda_dev):
    """The fp32 kernel takes a tile's key range from its rows' minimum and
    maximum positions, so positions need no order."""
    pos = np.random.default_rng(3).permutation(300).astype(np.int32)[:100]
    out, ref = _run_f32(100, 300, 8, 2, 64, cuda_dev, positions=pos, seed=3)
    assert rel_err(out, ref) < 1e-4


def test_f32_peaked_softmax(cuda_dev):
    """Large scores (q scaled by 40): online-softmax rescaling in fp32."""
    out, ref = _run_f32(200, 400, 4, 2, 128, cuda_dev, seed=9, scale_q=40.0)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_f32_16bit_output(cuda_dev, out_dtype):
    out, ref = _run_f32(96, 96, 4, 1, 256, cuda_dev, out_dtype=out_dtype, seed=5)
    assert max_abs_err(out, ref) < 2e-2


def test_f32_empty_rows_mean_of_v(cuda_dev):
    """Rows before every cached key get the mean of the value rows, like
    the NumPy path (a longer case than the golden one: several key tiles)."""
    out, ref = _run_f32(80, 150, 4, 2, 64, cuda_dev,
                        positions=np.arange(60, 140, dtype=np.int32), kv_start=100, seed=11)
    assert rel_err(out, ref) < 1e-4


# ---------------------------------------------------------------------------
# head_dim 256 on the tensor cores (one-head kernel, 64-key tiles)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [1, 100, 128, 300])
def test_d256_causal(cuda_dev, dt, T):
    out, ref = _run(T, T, 8, 2, 256, dt, cuda_dev, seed=T + 1)
    assert max_abs_err(out, ref) < 2e-2


@pytest.mark.parametrize("group", [1, 2, 4, 8])
def test_d256_gqa_with_prefix(cuda_dev, group):
    out, ref = _run(200, 533, 2 * group, 2, 256, torch.bfloat16, cuda_dev, seed=group)
    assert max_abs_err(out, ref) < 2e-2


def test_d256_window_kv_start(cuda_dev):
    out, ref = _run(150, 260, 8, 2, 256, torch.bfloat16, cuda_dev,
                    positions=np.arange(200, 350, dtype=np.int32), window=64, kv_start=100)
    assert max_abs_err(out, ref) < 2e-2


def test_d256_many_items(cuda_dev):
    """More work items than SMs: 16/2 heads (Qwen35's full-attention
    geometry) over a 1500-row chunk after a 500-row prefix."""
    out, ref = _run(1500, 2000, 16, 2, 256, torch.bfloat16, cuda_dev, seed=12)
    assert max_abs_err(out, ref) < 2e-2


@pytest.mark.parametrize("D", [64, 128, 256])
def test_empty_rows_mean_of_v_16bit(cuda_dev, kernel, D):
    """Rows with no visible key get the mean of the value rows on the tensor
    -core kernels too: a whole tile before kv_start (rows 0..127) and a
    ragged tile whose first rows precede it."""
    out, ref = _run(300, 200, 8, 2, D, torch.bfloat16, cuda_dev,
                    positions=np.arange(50, 350, dtype=np.int32), kv_start=200, seed=D)
    assert max_abs_err(out, ref) < 2e-2


def test_long_prefix_multi_item_per_cta(cuda_dev, kernel):
    """More work items than SMs (several items per persistent CTA), a long
    prefix and a ragged last tile."""
    out, ref = _run(1000, 3000, 32, 8, 128, torch.bfloat16, cuda_dev, seed=7)
    assert max_abs_err(out, ref) < 2e-2


def test_out_of_order_positions_are_reported(cuda_dev, kernel):
    """The persistent kernels take a tile's key range from its first and
    last query; positions that decrease inside a tile are outside that
    contract and must be reported, not silently mis-masked (the one-tile
    kernel computes the exact range and serves them correctly)."""
    if kernel == "single":
        pytest.skip("the one-tile kernel computes the exact key range")
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    _lib.device_error(clear=True)
    T, H, KV, D = 128, 8, 2, 64
    q = torch.randn((T, H, D), device=cuda_dev, dtype=torch.bfloat16)
    k = torch.randn((400, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    v = torch.randn((400, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int32, device=cuda_dev)
    pos[5] = 399  # a row that sees keys past the tile's last position
    device.prefill(q, k, v, pos)
    code, aux = _lib.device_error(clear=True)
    assert code == _lib.ERR_POSITION and aux == 5
