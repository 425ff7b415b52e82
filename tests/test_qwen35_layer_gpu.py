"""Qwen35 full-attention layer on the device vs the reference's own layer.

tests/golden/qwen35_layer.npz holds the reference's trace boundaries
(Qcur_normed, Kcur_normed, attn_pregate, attn_gated) for one token after 40
cached rows (alpaccaroo/qwen35_runtime.py:597-664).  Tolerances: q and k
after RMSNorm + IMROPE within 1e-6 of the largest value (double evaluation
rounded to f32, as the IMROPE test); with an f32 cache the attention output
and the gated output within 1e-4 normwise (f32 GQA vs the reference's
math.fsum); with 16-bit caches 2e-2 max abs error.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.conftest import max_abs_err, rel_err
from tests.golden import cases

pytestmark = pytest.mark.gpu


def _layer(c, dtype, dev, batch=1, n_ctx=64):
    from alpacca_open_sourced_by_jt_b200.qwen35_layer import Qwen35AttentionLayer
    return Qwen35AttentionLayer(query_heads=c["H"], kv_heads=c["KV"], head_dim=c["D"],
                                rms_epsilon=c["eps"], rope_freq_base=c["base"],
                                sections=c["sections"], query_norm=c["q_norm"],
                                key_norm=c["k_norm"], n_ctx=n_ctx, batch=batch,
                                kv_dtype=dtype, device_=dev)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_layer_matches_reference_trace(cuda_dev, golden, dtype):
    g = golden("qwen35_layer.npz")
    c = cases.qwen35_layer_case()
    L = c["L"]
    lay = _layer(c, dtype, cuda_dev)
    lay.k_cache[0, :L] = torch.from_numpy(c["k_prev"]).to(cuda_dev).to(dtype)
    lay.v_cache[0, :L] = torch.from_numpy(c["v_prev"]).to(cuda_dev).to(dtype)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev).reshape(1, -1)
    out = lay.step(dev(c["query_gate"]), dev(c["key"]), dev(c["value"]),
                   torch.tensor([L], dtype=torch.int32, device=cuda_dev))
    torch.cuda.synchronize()
    q = lay.q.cpu().numpy().ravel()
    k = lay.k_cache[0, L].float().cpu().numpy().ravel()
    v = lay.v_cache[0, L].float().cpu().numpy().ravel()
    tol = 1e-6 * np.abs(g["q_normed"]).max()
    assert np.abs(q - g["q_normed"]).max() <= tol
    if dtype == torch.float32:
        assert np.abs(k - g["k_normed"]).max() <= 1e-6 * np.abs(g["k_normed"]).max()
        assert np.array_equal(v, g["appended_value"])
        assert rel_err(lay.attended.cpu().numpy().ravel(), g["pregate"]) < 1e-4
        assert rel_err(out.cpu().numpy().ravel(), g["gated"]) < 1e-4
    else:
        # the stored row is the f32 result rounded to the cache type
        assert max_abs_err(k, g["k_normed"]) < 2e-2
        assert np.array_equal(v, torch.from_numpy(g["appended_value"]).to(dtype).float().numpy())
        assert max_abs_err(out.cpu().numpy().ravel(), g["gated"]) < 2e-2


def test_layer_batch_of_sequences_at_different_positions(cuda_dev):
    c = cases.qwen35_layer_case()
    rng = np.random.default_rng(4)
    B, H, KV, D, n_ctx = 3, c["H"], c["KV"], c["D"], 80
    lay = _layer(c, torch.float32, cuda_dev, batch=B, n_ctx=n_ctx)
    pos = np.array([0, 17, 63], np.int32)
    prev_k = rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)
    prev_v = rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)
    lay.k_cache.copy_(torch.from_numpy(prev_k))
    lay.v_cache.copy_(torch.from_numpy(prev_v))
    qg = rng.standard_normal((B, H * 2 * D), dtype=np.float32)
    k = rng.standard_normal((B, KV * D), dtype=np.float32)
    v = rng.standard_normal((B, KV * D), dtype=np.float32)
    out = lay.step(torch.from_numpy(qg).to(cuda_dev), torch.from_numpy(k).to(cuda_dev),
                   torch.from_numpy(v).to(cuda_dev), torch.from_numpy(pos).to(cuda_dev))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        p = int(pos[b])
        _, _, _, gated = oracle.qwen35_attention_layer(
            qg[b], k[b], v[b], c["q_norm"], c["k_norm"], c["eps"], c["sections"], c["base"], p,
            prev_k[b, :p], prev_v[b, :p])
        assert rel_err(got[b], gated) < 1e-4
