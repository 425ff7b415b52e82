"""Split-KV decode kernels vs the oracle (the reference's NumPy decode).

Tolerances: fp32 caches 1e-4 max relative error (normwise, see
conftest.rel_err); f16/bf16 caches 2e-2 max abs error on unit-variance
outputs, against the oracle evaluated in fp32 on the same 16-bit-rounded
K/V (the kernel additionally rounds q and the softmax weights to 16 bits
for the tensor cores; fp32 accumulation throughout).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import max_abs_err, rel_err
from tests.golden import cases

pytestmark = pytest.mark.gpu

TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _caches(rng, B, n_ctx, KV, D, dt, dev, pad=0):
    """Random caches with `pad` extra rows of stride per sequence."""
    k = rng.standard_normal((B, n_ctx + pad, KV, D), dtype=np.float32)
    v = rng.standard_normal((B, n_ctx + pad, KV, D), dtype=np.float32)
    kt = torch.from_numpy(k).to(dev).to(TDT[dt])[:, :n_ctx]
    vt = torch.from_numpy(v).to(dev).to(TDT[dt])[:, :n_ctx]
    # the oracle sees exactly the values the kernel reads
    return kt, vt, kt.float().cpu().numpy(), vt.float().cpu().numpy()


def _run(B, H, KV, D, lens, dt, dev, split_rows=0, n_ctx=None, pad=0, seed=0, lse=False):
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(seed)
    n_ctx = n_ctx or max(max(lens), 1)
    kt, vt, kh, vh = _caches(rng, B, n_ctx, KV, D, dt, dev, pad)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    qt = torch.from_numpy(q).to(dev)
    lt = torch.tensor(lens, dtype=torch.int32, device=dev)
    lse_t = torch.empty((B, H), dtype=torch.float32, device=dev) if lse else None
    out = device.decode(qt, kt, vt, lt, max_len=n_ctx, split_rows=split_rows, lse=lse_t)
    torch.cuda.synchronize()
    ref = np.zeros((B, H, D), np.float32)
    for b in range(B):
        if lens[b] > 0:
            ref[b] = oracle.attention_decode(q[b], kh[b, :lens[b]], vh[b, :lens[b]], H // KV,
                                             1.0 / math.sqrt(D))
    return out.cpu().numpy(), ref, (q, kh, vh), lse_t


def test_config1_golden_through_dropin(cuda_dev, golden):
    """benchmark config 1 end to end through kernels.attention_decode (the
    reference's kernels.py signature) against the reference's own output."""
    from alpacca_open_sourced_by_jt_b200 import kernels
    g = golden("decode_config1.npz")
    c = cases.decode_config1()
    cos, sin = oracle.rope_tables(c["L"], c["D"], c["base"])
    K = np.stack([oracle.rope_vec(c["k_raw"][p].reshape(-1), c["KV"], p, cos, sin, c["D"],
                                  c["D"], "norm").reshape(c["KV"], c["D"]) for p in range(c["L"])])
    out = kernels.attention_decode(g["q_rot"], K, c["v"], c["H"] // c["KV"],
                                   1.0 / math.sqrt(c["D"]))
    assert out.shape == (32, 64) and out.dtype == np.float32
    assert rel_err(out, g["out"]) < 1e-4


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("group", [1, 4, 8, 16])
def test_fp32_cache(cuda_dev, D, group):
    out, ref, _, _ = _run(2, 2 * group, 2, D, [300, 77], "f32", cuda_dev, split_rows=128)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("group", [1, 4, 8, 16])
def test_16bit_cache_shapes(cuda_dev, dt, D, group):
    out, ref, _, _ = _run(2, 2 * group, 2, D, [517, 64], dt, cuda_dev, split_rows=256)
    assert max_abs_err(out, ref) < 2e-2
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("lens", [[1], [5, 63, 64, 65], [127, 128, 129, 1000], [4097, 1, 2048]])
@pytest.mark.parametrize("split_rows", [64, 192, 0])
def test_ragged_lengths_and_splits(cuda_dev, dt, lens, split_rows):
    out, ref, _, _ = _run(len(lens), 32, 8, 128, lens, dt, cuda_dev, split_rows=split_rows,
                          n_ctx=4160, seed=len(lens))
    assert max_abs_err(out, ref) < 2e-2


def test_sequence_stride_padding(cuda_dev):
    """Sequences live `seq_stride` elements apart (padding rows between)."""
    out, ref, _, _ = _run(3, 32, 8, 128, [700, 9, 1024], "bf16", cuda_dev, n_ctx=1024, pad=37)
    assert max_abs_err(out, ref) < 2e-2


def test_zero_length_and_lse(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device  # noqa: F401
    out, ref, (q, kh, vh), lse = _run(3, 8, 2, 64, [0, 50, 333], "f32", cuda_dev, lse=True)
    assert np.all(out[0] == 0.0)
    lse = lse.cpu().numpy()
    assert np.all(np.isneginf(lse[0]))
    for b in (1, 2):
        L = [0, 50, 333][b]
        s = np.einsum("khd,tkd->kht", q[b].reshape(2, 4, 64).astype(np.float64),
                      kh[b, :L].astype(np.float64)) / 8.0
        ref_lse = np.log(np.exp(s - s.max(-1, keepdims=True)).sum(-1)) + s.max(-1)
        assert np.abs(lse[b] - ref_lse.reshape(-1)).max() < 1e-4
    assert rel_err(out[1:], ref[1:]) < 1e-4


def test_never_written_rows_do_not_leak(cuda_dev):
    """Rows past a sequence's length (NaN/Inf garbage here) never reach the
    output, including inside a partially filled tile."""
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(9)
    B, H, KV, D, n_ctx = 2, 32, 8, 128, 512
    k = torch.full((B, n_ctx, KV, D), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
    v = torch.full((B, n_ctx, KV, D), float("inf"), dtype=torch.bfloat16, device=cuda_dev)
    lens = [70, 129]
    kv_h = []
    for b, L in enumerate(lens):
        kk = torch.from_numpy(rng.standard_normal((L, KV, D), dtype=np.float32)).to(cuda_dev)
        vv = torch.from_numpy(rng.standard_normal((L, KV, D), dtype=np.float32)).to(cuda_dev)
        k[b, :L] = kk.to(torch.bfloat16)
        v[b, :L] = vv.to(torch.bfloat16)
        kv_h.append((k[b, :L].float().cpu().numpy(), v[b, :L].float().cpu().numpy()))
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    out = device.decode(torch.from_numpy(q).to(cuda_dev), k, v,
                        torch.tensor(lens, dtype=torch.int32, device=cuda_dev), split_rows=64)
    out = out.cpu().numpy()
    assert np.isfinite(out).all()
    for b in range(B):
        ref = oracle.attention_decode(q[b], kv_h[b][0], kv_h[b][1], 4, 1 / math.sqrt(D))
        assert max_abs_err(out[b], ref) < 2e-2


def test_split_size_invariance_and_determinism(cuda_dev):
    """Size-independent properties at a long context: different KV splits
    agree to fp32 rounding, and a rerun is bit-identical."""
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(4)
    B, H, KV, D, L = 2, 32, 8, 128, 32768
    k = torch.randn((B, L, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    v = torch.randn((B, L, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    q = torch.from_numpy(rng.standard_normal((B, H, D), dtype=np.float32)).to(cuda_dev)
    lens = torch.tensor([L, L - 1000], dtype=torch.int32, device=cuda_dev)
    a = device.decode(q, k, v, lens, split_rows=512)
    b = device.decode(q, k, v, lens, split_rows=2048)
    c = device.decode(q, k, v, lens, split_rows=512)
    assert torch.equal(a, c)
    # different split boundaries round the softmax weights to bf16 against
    # different running maxima: agreement to ~1e-4 of unit-scale outputs
    assert (a - b).abs().max().item() < 1e-3
    # and against the oracle at full 32K length for the first sequence
    ref = oracle.attention_decode(q[0].cpu().numpy(), k[0].float().cpu().numpy(),
                                  v[0].float().cpu().numpy(), 4, 1 / math.sqrt(D))
    assert max_abs_err(a[0].cpu().numpy(), ref) < 2e-2


def test_lse_combine_kernel_matches_oracle(cuda_dev):
    """Shard a context three ways (one shard empty), decode each shard with
    lse, merge with b2a_lse_combine: equals the unsharded decode."""
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(12)
    H, KV, D, L = 64, 8, 128, 3000
    k = torch.randn((1, L, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    v = torch.randn((1, L, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    q = torch.from_numpy(rng.standard_normal((1, H, D), dtype=np.float32)).to(cuda_dev)
    bounds = [0, 1234, 1234, L]
    os_, ls_ = [], []
    for g in range(3):
        a, b = bounds[g], bounds[g + 1]
        n = max(b - a, 1)
        lse = torch.empty((1, H), device=cuda_dev)
        lens = torch.tensor([b - a], dtype=torch.int32, device=cuda_dev)
        o = device.decode(q, k[:, a:a + n].contiguous(), v[:, a:a + n].contiguous(), lens,
                          lse=lse, max_len=n)
        os_.append(o.reshape(H, D))
        ls_.append(lse.reshape(H))
    merged = device.lse_combine(torch.stack(os_), torch.stack(ls_))
    full = device.decode(q, k, v, torch.tensor([L], dtype=torch.int32, device=cuda_dev))
    # shard boundaries change where P is rounded to bf16 (see above)
    assert (merged - full.reshape(H, D)).abs().max().item() < 1e-3
