"""Whole-token decode on the device (decode_chain.py) vs the reference.

* b2a_q8_gemv in its three input modes and with the residual epilogue vs
  the oracle's restatement of the reference's Q8_0 matvec
  (alpaccaroo/qmatrix.py:312-320) with its RMSNorm / SwiGLU inputs:
  1e-5 normwise (f32 accumulation in a different order).
* b2a_q8_embed vs the reference's dequantized row: exact.
* DecodeChain on a small Q8_0 llama model vs the logits of the reference's
  own Model._forward_np (tests/golden/llama_q8.npz, six tokens): 1e-4
  normwise with an f32 KV cache, 1e-2 with f16 (the cache rounding).
"""
import numpy as np
import pytest
import torch

import oracle
from oracle import llama_q8 as L
from tests.conftest import rel_err
from tests.golden import cases

pytestmark = pytest.mark.gpu


def _q8(rng, rows, cols):
    return L.quantize_q8_0(rng.normal(0.0, 0.02, (rows, cols)).astype(np.float32))


@pytest.mark.parametrize("rows,cols", [(1, 32), (3, 96), (300, 2048), (257, 8192), (37, 6144),
                                       (64, 4096), (17, 512), (2000, 256)])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_q8_gemv_modes(cuda_dev, rows, cols, mode):
    from alpacca_open_sourced_by_jt_b200.decode_chain import Q8Matrix
    rng = np.random.default_rng(rows * 7 + cols + mode)
    data = _q8(rng, rows, cols)
    w = Q8Matrix.from_q8_0(data, rows, cols, cuda_dev)
    xin = rng.standard_normal(2 * cols if mode == 2 else cols).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    if mode == 0:
        xv = xin
    elif mode == 1:
        xv = L.rmsnorm(xin, nw, 1e-5)
    else:
        g, u = xin[:cols], xin[cols:]
        xv = g / (np.float32(1.0) + np.exp(-g)) * u
    want = L.q8_0_matvec(data, rows, cols, xv)
    x = torch.from_numpy(xin).to(cuda_dev)
    out = torch.zeros(rows, dtype=torch.float32, device=cuda_dev)
    w.gemv(x, out, mode=mode, aux=torch.from_numpy(nw).to(cuda_dev), eps=1e-5)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), want) < 1e-5
    base = rng.standard_normal(rows).astype(np.float32)
    out.copy_(torch.from_numpy(base))
    w.gemv(x, out, mode=mode, aux=torch.from_numpy(nw).to(cuda_dev), eps=1e-5, flags=1 | 4)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), base + want) < 1e-5


@pytest.mark.parametrize("rows,cols", [(8, 64), (512, 2048), (40, 8192)])
def test_q8_gemv_swiglu_epilogue(cuda_dev, rows, cols):
    from alpacca_open_sourced_by_jt_b200.decode_chain import Q8Matrix
    rng = np.random.default_rng(rows + cols)
    dg, du = _q8(rng, rows, cols), _q8(rng, rows, cols)
    w = Q8Matrix.interleave(Q8Matrix.from_q8_0(dg, rows, cols, cuda_dev),
                            Q8Matrix.from_q8_0(du, rows, cols, cuda_dev))
    xin = rng.standard_normal(cols).astype(np.float32)
    gate = L.q8_0_matvec(dg, rows, cols, xin)
    up = L.q8_0_matvec(du, rows, cols, xin)
    want = gate / (np.float32(1.0) + np.exp(-gate)) * up
    out = torch.zeros(rows, dtype=torch.float32, device=cuda_dev)
    w.gemv(torch.from_numpy(xin).to(cuda_dev), out, flags=2)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), want) < 1e-5


def test_q8_embed_row(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib
    from alpacca_open_sourced_by_jt_b200.decode_chain import Q8Matrix
    rng = np.random.default_rng(2)
    rows, cols = 50, 256
    data = _q8(rng, rows, cols)
    w = Q8Matrix.from_q8_0(data, rows, cols, cuda_dev)
    out = torch.zeros(cols, dtype=torch.float32, device=cuda_dev)
    for t in (0, 17, 49):
        tok = torch.tensor([t], dtype=torch.int32, device=cuda_dev)
        _lib.check(_lib.load().b2a_q8_embed(w.codes.data_ptr(), w.scales.data_ptr(), rows, cols,
                                            tok.data_ptr(), 1, out.data_ptr(), None))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), L.q8_0_row(data, rows, cols, t))


@pytest.mark.parametrize("kv_dtype,tol", [(torch.float32, 1e-4), (torch.float16, 1e-2)])
def test_chain_matches_reference_logits(cuda_dev, golden, kv_dtype, tol):
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    g = golden("llama_q8.npz")
    c = cases.llama_q8_case()
    assert c["sha256"] == str(g["weights_sha256"])
    model = LlamaQ8.from_spec(c, cuda_dev)
    chain = DecodeChain(model, c["n_ctx"], kv_dtype)
    for pos, tok in enumerate(c["tokens"]):
        logits = chain(tok, pos).numpy()
        assert rel_err(logits, g["logits"][pos]) < tol, pos
    assert chain.launches == 2 + 6 * c["n_layer"]


@pytest.mark.parametrize("kv_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,KV,D,cols", [(32, 8, 64, 2048), (2, 1, 64, 8192), (4, 2, 128, 256)])
def test_qkv_rope_epilogue_matches_two_launches(cuda_dev, kv_dtype, H, KV, D, cols):
    """b2a_q8_gemv_qkv_rope against the GEMV (RMSNorm mode) followed by
    b2a_rope_append: the same products, rotation and stores, so q and the
    cache rows must agree bit for bit; the other cache rows stay untouched."""
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.decode_chain import Q8Matrix
    rng = np.random.default_rng(H * D + cols)
    rows, n_ctx = (H + 2 * KV) * D, 64
    w = Q8Matrix.from_q8_0(_q8(rng, rows, cols), rows, cols, cuda_dev)
    x = torch.from_numpy(rng.standard_normal(cols).astype(np.float32)).to(cuda_dev)
    nw = torch.from_numpy((1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)).to(cuda_dev)
    ct, st = device.rope_tables(n_ctx, D, 500000.0, device=cuda_dev)
    pos = torch.tensor([37], dtype=torch.int32, device=cuda_dev)
    base = torch.from_numpy(rng.standard_normal((1, n_ctx, KV, D)).astype(np.float32)).to(
        cuda_dev).to(kv_dtype)
    k_ref, v_ref, k_got, v_got = base.clone(), base.clone(), base.clone(), base.clone()
    qkv = torch.zeros(rows, dtype=torch.float32, device=cuda_dev)
    w.gemv(x, qkv, mode=1, aux=nw, eps=1e-5)
    qd, kd = H * D, KV * D
    device.rope_append(qkv[:qd].view(1, H, D), qkv[qd:qd + kd].view(1, KV, D),
                       qkv[qd + kd:].view(1, KV, D), pos, ct, st, k_cache=k_ref, v_cache=v_ref)
    q_got = torch.zeros(rows, dtype=torch.float32, device=cuda_dev)
    w.gemv_qkv_rope(x, nw, 1e-5, q_got, ct, st, pos, k_got, v_got, H, KV, D, flags=4)
    torch.cuda.synchronize()
    assert torch.equal(q_got[:qd], qkv[:qd])
    assert torch.equal(k_got, k_ref) and torch.equal(v_got, v_ref)
