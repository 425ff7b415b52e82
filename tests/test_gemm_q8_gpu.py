"""b2a_gemm_q8 / b2a_gemm_qkv_rope_q8: the chunk GEMMs reading Q8_0 weights
(int8 codes, an f16 scale per 32 codes) and decoding them inside the kernel.

The converter warps write d * code, rounded once to the operand type, into
the tensor cores' shared-memory tiles, so every product must equal
b2a_gemm's on the dequantized matrix (the 16-bit copy the reference-shaped
host code would make: codes.float() * scales.float(), rounded) bit for bit.
The one exception is the in-place residual on the stream-K schedule, whose
partial sums are added in an order that changes between runs; it is held to
1e-6 normwise.  Codes cover the whole int8 range (-128 .. 127) and scales
include f16 subnormals, so the in-register dequantization is checked at its
edges.
"""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _q8(N, K, dev, seed, subnormal=False):
    g = torch.Generator(device=dev).manual_seed(seed)
    codes = torch.randint(-128, 128, (N, K), device=dev, generator=g, dtype=torch.int32).to(torch.int8)
    scales = (0.0005 + 0.002 * torch.rand((N, K // 32), device=dev, generator=g))
    if subnormal:  # every 7th scale below the f16 normal range (6.1e-5)
        scales.view(-1)[::7] = 3e-6
    return codes, scales.to(torch.float16)


def _dequant(codes, scales, dt):
    N, K = codes.shape
    w = codes.float().view(N, K // 32, 32) * scales.float()[:, :, None]
    return w.reshape(N, K).to(dt)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (77, 100, 96), (300, 520, 224),
                                   (1000, 3072, 512), (2048, 2048, 2048)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_q8_equals_gemm_on_dequantized(cuda_dev, M, N, K, dt):
    from alpacca_open_sourced_by_jt_b200 import device
    codes, scales = _q8(N, K, cuda_dev, M + N + K, subnormal=True)
    g = torch.Generator(device=cuda_dev).manual_seed(K)
    a = torch.randn((M, K), device=cuda_dev, generator=g).to(dt)
    got = device.gemm_q8(a, (codes, scales))
    want = device.gemm(a, _dequant(codes, scales, dt))
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_gemm_q8_16bit_out(cuda_dev, out_dtype):
    from alpacca_open_sourced_by_jt_b200 import device
    M, N, K = 333, 768, 320
    codes, scales = _q8(N, K, cuda_dev, 9)
    a = torch.randn((M, K), device=cuda_dev).to(torch.float16)
    got = device.gemm_q8(a, (codes, scales), out_dtype=out_dtype)
    want = device.gemm(a, _dequant(codes, scales, torch.float16), out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 8192), (130, 200, 512), (400, 2048, 2048)])
def test_gemm_q8_residual_in_place(cuda_dev, M, N, K):
    from alpacca_open_sourced_by_jt_b200 import device
    codes, scales = _q8(N, K, cuda_dev, 17)
    g = torch.Generator(device=cuda_dev).manual_seed(18)
    a = torch.randn((M, K), device=cuda_dev, generator=g).to(torch.float16)
    x = torch.randn((M, N), device=cuda_dev, generator=g)
    x1, x2 = x.clone(), x.clone()
    device.gemm_q8(a, (codes, scales), out=x1, c_in=x1)
    device.gemm(a, _dequant(codes, scales, torch.float16), out=x2, c_in=x2)
    torch.cuda.synchronize()
    assert rel_err(x1.cpu().numpy(), x2.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("M", [5, 130, 2048])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_q8_swiglu_halves(cuda_dev, M, dt):
    """GEMM_SWIGLU (256-row groups of 128 gate then 128 up rows)."""
    from alpacca_open_sourced_by_jt_b200 import device
    F, K = 512, 256
    codes, scales = _q8(2 * F, K, cuda_dev, M)
    a = torch.randn((M, K), device=cuda_dev).to(dt)
    got = device.gemm_q8(a, (codes, scales), epilogue=device.GEMM_SWIGLU, out_dtype=dt)
    want = device.gemm(a, _dequant(codes, scales, dt), epilogue=device.GEMM_SWIGLU, out_dtype=dt)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("M,F,K", [(5, 256, 256), (130, 1024, 512), (2048, 8192, 2048),
                                   (77, 200, 128)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_q8_swiglu8_interleave(cuda_dev, M, F, K, dt):
    """GEMM_SWIGLU8: the decode GEMV's layout (16-row groups of 8 gate rows
    then their 8 up rows); against the same product to f32 with SwiGLU in
    torch (the kernel's exponential may differ from torch's by an ulp)."""
    from alpacca_open_sourced_by_jt_b200 import device
    codes, scales = _q8(2 * F, K, cuda_dev, M + F)
    a = torch.randn((M, K), device=cuda_dev).to(dt)
    got = device.gemm_q8(a, (codes, scales), epilogue=device.GEMM_SWIGLU8)
    s = device.gemm_q8(a, (codes, scales)).view(M, F // 8, 2, 8)
    gate, up = s[:, :, 0].reshape(M, F), s[:, :, 1].reshape(M, F)
    want = gate / (1 + torch.exp(-gate)) * up
    torch.cuda.synchronize()
    assert got.shape == (M, F)
    assert rel_err(got.cpu().numpy(), want.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("T,E,H,KV,D,pos0", [(200, 512, 8, 2, 128, 37), (77, 320, 4, 4, 64, 0),
                                             (2048, 2048, 32, 8, 64, 5)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_qkv_rope_q8_equals_dequantized(cuda_dev, T, E, H, KV, D, pos0, dt):
    from alpacca_open_sourced_by_jt_b200 import device
    n_ctx = pos0 + T + 5
    codes, scales = _q8((H + 2 * KV) * D, E, cuda_dev, T + E)
    a = torch.randn((T, E), device=cuda_dev).to(dt)
    cos, sin = device.rope_tables(n_ctx, D, 500000.0, device=cuda_dev)
    pos = torch.arange(pos0, pos0 + T, dtype=torch.int32, device=cuda_dev)
    outs = []
    for w in ((codes, scales), _dequant(codes, scales, dt)):
        kc = torch.zeros((n_ctx, KV, D), device=cuda_dev, dtype=dt)
        vc = torch.zeros_like(kc)
        q = torch.zeros((T, H, D), device=cuda_dev, dtype=dt)
        device.gemm_qkv_rope(a, w, pos, cos, sin, H=H, KV=KV, k_cache=kc, v_cache=vc, q_out=q)
        outs.append((q, kc, vc))
    torch.cuda.synchronize()
    for x, y in zip(*outs):
        assert torch.equal(x, y)


@pytest.mark.parametrize("rows,cols", [(16, 32), (300, 224), (4096, 2048), (3, 8192)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_q8_dequant_equals_host_dequantization(cuda_dev, rows, cols, dt):
    """b2a_q8_dequant: d * code rounded once, bit for bit, into a strided view."""
    from alpacca_open_sourced_by_jt_b200 import device
    codes, scales = _q8(rows, cols, cuda_dev, rows + cols, subnormal=True)
    big = torch.full((rows, cols + 24), 7.0, device=cuda_dev, dtype=dt)
    got = device.q8_dequant((codes, scales), out=big[:, 8:8 + cols])
    torch.cuda.synchronize()
    assert torch.equal(got, _dequant(codes, scales, dt))
    assert (big[:, :8] == 7).all() and (big[:, 8 + cols:] == 7).all()


@pytest.mark.parametrize("M,F,K", [(130, 1024, 512), (2048, 8192, 2048)])
def test_gemm_swiglu8_on_16bit_weights_equals_q8(cuda_dev, M, F, K):
    """b2a_gemm with GEMM_SWIGLU8 on the dequantized rows gives what b2a_gemm_q8
    gives on the codes."""
    from alpacca_open_sourced_by_jt_b200 import device
    codes, scales = _q8(2 * F, K, cuda_dev, M)
    a = torch.randn((M, K), device=cuda_dev).to(torch.float16)
    got = device.gemm(a, device.q8_dequant((codes, scales)), epilogue=device.GEMM_SWIGLU8,
                      out_dtype=torch.float16)
    want = device.gemm_q8(a, (codes, scales), epilogue=device.GEMM_SWIGLU8,
                          out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_gemm_q8_rejects_bad_arguments(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    a = torch.zeros((16, 96), device=cuda_dev, dtype=torch.float16)
    codes = torch.zeros((64, 96), device=cuda_dev, dtype=torch.int8)
    scales = torch.zeros((64, 3), device=cuda_dev, dtype=torch.float16)
    lib = _lib.load()
    out = torch.zeros((16, 64), device=cuda_dev)
    # K not a multiple of 32
    rc = lib.b2a_gemm_q8(a.data_ptr(), 96, codes.data_ptr(), 96, scales.data_ptr(), 3,
                         _lib.F16, None, 0, out.data_ptr(), 64, _lib.F32, 16, 64, 80, 0, None)
    assert rc == _lib.ERR_SHAPE
    # code rows not a multiple of 16 bytes apart
    rc = lib.b2a_gemm_q8(a.data_ptr(), 96, codes.data_ptr(), 88, scales.data_ptr(), 3,
                         _lib.F16, None, 0, out.data_ptr(), 64, _lib.F32, 16, 64, 64, 0, None)
    assert rc == _lib.ERR_ALIGN
    # SWIGLU8 with rows not a multiple of 16
    rc = lib.b2a_gemm_q8(a.data_ptr(), 96, codes.data_ptr(), 96, scales.data_ptr(), 3,
                         _lib.F16, None, 0, out.data_ptr(), 64, _lib.F32, 16, 40, 96, 2, None)
    assert rc == _lib.ERR_SHAPE
    with pytest.raises(_lib.B2AShapeError):
        device.gemm_q8(a, (codes[:, :64], scales))
