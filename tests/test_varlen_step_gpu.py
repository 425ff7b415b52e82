"""Batched variable-length decode step (the config-3 path) vs the oracle.

One token of every sequence per step: the fused RoPE + append kernel rotates
q and k at the sequence's own position and stores k/v into a fp16 cache,
then the split-KV decode attends over the sequence's rows.  The oracle runs
the reference's per-sequence loop (alpaccaroo/model.py:1418-1440: rope,
cache store, _attention_np over cache[:pos+1]) on the same fp16-rounded
rows.  Several steps in a row check that appended rows are the ones later
steps read.  Tolerances: the rotated q and the stored rows bit-exact; the
attention output 2e-2 max abs error (fp16 K/V, 16-bit q and softmax weights
on the tensor cores, fp32 accumulation).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import max_abs_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_varlen_decode_steps_with_fused_append(cuda_dev, dt):
    from alpacca_open_sourced_by_jt_b200 import device
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[dt]
    rng = np.random.default_rng(2)
    B, H, KV, D, n_ctx, n_steps = 12, 32, 8, 128, 1600, 3
    lens0 = rng.integers(1, 1500, size=B)
    lens0[0], lens0[1] = 0, 1500 - 1      # an empty history and a near-full one
    kc = torch.from_numpy(rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)).to(
        cuda_dev).to(tdt)
    vc = torch.from_numpy(rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)).to(
        cuda_dev).to(tdt)
    kref = kc.float().cpu().numpy()
    vref = vc.float().cpu().numpy()
    cos, sin = oracle.rope_tables(n_ctx, D, 500000.0)
    ct, st = device.rope_tables(n_ctx, D, 500000.0, device=cuda_dev)
    split = device.decode_split_rows(B, KV, n_ctx, tdt)
    ws = device.decode_workspace(B, H, D, n_ctx, split, cuda_dev)
    for s in range(n_steps):
        pos = (lens0 + s).astype(np.int32)
        q = rng.standard_normal((B, H, D), dtype=np.float32)
        k = rng.standard_normal((B, KV, D), dtype=np.float32)
        v = rng.standard_normal((B, KV, D), dtype=np.float32)
        qr = torch.empty((B, H, D), dtype=torch.float32, device=cuda_dev)
        pd = torch.from_numpy(pos).to(cuda_dev)
        device.rope_append(torch.from_numpy(q).to(cuda_dev), torch.from_numpy(k).to(cuda_dev),
                           torch.from_numpy(v).to(cuda_dev), pd, ct, st, k_cache=kc,
                           v_cache=vc, per_sequence=True, q_out=qr)
        out = device.decode(qr, kc, vc, pd + 1, workspace=ws, split_rows=split, max_len=n_ctx)
        torch.cuda.synchronize()
        # oracle: rope + store in fp32, rows rounded as the cache dtype stores them
        kst = np.zeros((B, n_ctx, KV, D), np.float32)
        vst = np.zeros_like(kst)
        qref = oracle.rope_append(q, k, v, pos, kst, vst, cos, sin, D, "norm",
                                  seq_of_token=np.arange(B))
        for b in range(B):
            rk = torch.from_numpy(kst[b, pos[b]]).to(tdt).float().numpy()
            rv = torch.from_numpy(vst[b, pos[b]]).to(tdt).float().numpy()
            kref[b, pos[b]], vref[b, pos[b]] = rk, rv
        assert np.array_equal(qr.cpu().numpy(), qref)
        kd, vd = kc.float().cpu().numpy(), vc.float().cpu().numpy()
        for b in range(B):
            assert np.array_equal(kd[b, pos[b]], kref[b, pos[b]])
            assert np.array_equal(vd[b, pos[b]], vref[b, pos[b]])
        ref = oracle.attention_decode_varlen(qref, kref, vref, pos + 1, H // KV,
                                             1.0 / math.sqrt(D))
        assert max_abs_err(out.cpu().numpy(), ref) < 2e-2
