"""b2a_gemm (tcgen05 + TMEM + TMA) against a PyTorch product of the same
16-bit inputs.

The kernel multiplies 16-bit operands exactly and accumulates in fp32; the
tensor core's fp32 accumulation over K/16 chained MMAs rounds differently
from a sequential fp32 sum, and the difference grows with K.  So fp32
outputs are measured against an fp64 product (normwise, max |a-b| / max |b|)
and must be within twice the error of PyTorch's own 16-bit GEMM with fp32
accumulation (cuBLAS) on the same inputs, or within 1e-6; 16-bit outputs
within one rounding of the output type (2^-8 relative for bf16, 2^-10 for
f16).
Shapes cover tails in M, N and K, several tiles per CTA (the persistent
loop and both TMEM accumulators), the in-place residual and the SwiGLU
epilogue of the prefill chunk's gate/up projection.
"""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _ref(a, w):
    return a.float() @ w.float().t()


def _check(got, a, w, add=None, swiglu=False):
    """got within max(2 x cuBLAS's error, 1e-6) of the fp64 product."""
    ref = a.double() @ w.double().t()
    lib = torch.mm(a, w.t(), out_dtype=torch.float32).double()
    if swiglu:
        F = w.shape[0] // 2
        def act(s):
            g = s.view(-1, F // 128, 2, 128)[:, :, 0].reshape(-1, F)
            u = s.view(-1, F // 128, 2, 128)[:, :, 1].reshape(-1, F)
            return g / (1 + torch.exp(-g)) * u
        ref, lib = act(ref), act(lib)
    if add is not None:
        ref, lib = ref + add.double(), lib + add.double()
    ref_np = ref.cpu().numpy()
    err = rel_err(got.double().cpu().numpy(), ref_np)
    bar = max(2 * rel_err(lib.cpu().numpy(), ref_np), 1e-6)
    assert err <= bar, (err, bar)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (77, 100, 72), (300, 520, 200),
                                   (1000, 3072, 512), (2048, 2048, 8192)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_store(cuda_dev, M, N, K, dt):
    from alpacca_open_sourced_by_jt_b200 import device
    g = torch.Generator(device=cuda_dev).manual_seed(M + N + K)
    a = torch.randn((M, K), device=cuda_dev, generator=g).to(dt)
    w = (0.05 * torch.randn((N, K), device=cuda_dev, generator=g)).to(dt)
    out = device.gemm(a, w)
    torch.cuda.synchronize()
    _check(out, a, w)


@pytest.mark.parametrize("out_dtype,tol", [(torch.bfloat16, 2 ** -8), (torch.float16, 2 ** -10)])
def test_gemm_16bit_out_and_strides(cuda_dev, out_dtype, tol):
    from alpacca_open_sourced_by_jt_b200 import device
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    M, N, K = 333, 768, 320
    big = torch.randn((M, K + 64), device=cuda_dev, generator=g).to(torch.bfloat16)
    a = big[:, 32:32 + K]  # row stride K + 64, 64-byte offset
    w = (0.05 * torch.randn((N, K), device=cuda_dev, generator=g)).to(torch.bfloat16)
    out_big = torch.zeros((M, N + 8), device=cuda_dev, dtype=out_dtype)
    device.gemm(a, w, out=out_big[:, :N])
    torch.cuda.synchronize()
    assert rel_err(out_big[:, :N].float().cpu().numpy(), _ref(a, w).cpu().numpy()) < tol
    assert not out_big[:, N:].any()


@pytest.mark.parametrize("M,N,K", [(400, 2048, 2048), (2048, 2048, 8192), (130, 200, 520),
                                   (2048, 2048, 2048)])
def test_gemm_residual_in_place(cuda_dev, M, N, K):
    """x += a . w^T in place.  These shapes take the stream-K schedule (fewer
    than two full waves of tiles): K ranges split across CTAs, each adding
    its partial sum into x; (130, 200, 520) has a ragged tile edge and a
    ragged last K block."""
    from alpacca_open_sourced_by_jt_b200 import device
    g = torch.Generator(device=cuda_dev).manual_seed(6)
    a = torch.randn((M, K), device=cuda_dev, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn((N, K), device=cuda_dev, generator=g)).to(torch.bfloat16)
    x = torch.randn((M, N), device=cuda_dev, generator=g)
    x0 = x.clone()
    device.gemm(a, w, out=x, c_in=x)
    torch.cuda.synchronize()
    _check(x, a, w, add=x0)


@pytest.mark.parametrize("M", [5, 130, 2048])
def test_gemm_swiglu(cuda_dev, M):
    from alpacca_open_sourced_by_jt_b200 import device
    g = torch.Generator(device=cuda_dev).manual_seed(M)
    F, K = 512, 256
    a = torch.randn((M, K), device=cuda_dev, generator=g).to(torch.bfloat16)
    wg = (0.1 * torch.randn((F, K), device=cuda_dev, generator=g)).to(torch.bfloat16)
    wu = (0.1 * torch.randn((F, K), device=cuda_dev, generator=g)).to(torch.bfloat16)
    # 256-row groups: 128 gate rows, then the matching 128 up rows
    w = torch.cat([wg.view(F // 128, 128, K), wu.view(F // 128, 128, K)], 1).reshape(2 * F, K)
    out = device.gemm(a, w, epilogue=device.GEMM_SWIGLU)
    torch.cuda.synchronize()
    _check(out, a, w, swiglu=True)


def test_gemm_rejects_bad_arguments(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    a = torch.zeros((16, 64), device=cuda_dev, dtype=torch.bfloat16)
    w = torch.zeros((256, 64), device=cuda_dev, dtype=torch.bfloat16)
    with pytest.raises(_lib.B2AError):
        device.gemm(a, w[:100], epilogue=device.GEMM_SWIGLU)  # N % 256
    with pytest.raises(_lib.B2AError):
        device.gemm(a, w[:40], epilogue=device.GEMM_SWIGLU8)  # N % 16
    with pytest.raises(_lib.B2AError):
        device.gemm(a, w.to(torch.float16))  # mixed operand types
    lib = _lib.load()
    assert lib.b2a_gemm(a.data_ptr(), 60, w.data_ptr(), 64, _lib.BF16, None, 0,
                        a.data_ptr(), 64, _lib.F32, 16, 256, 64, 0, None) == _lib.ERR_ALIGN


# the 148-SM wave model takes 192-column tiles for the first three and
# 256-column tiles for the last (148 tiles of 256 against 222 of 192)
@pytest.mark.parametrize("T,E,H,KV,D,pos0", [(200, 512, 8, 2, 128, 37), (77, 320, 4, 4, 64, 0),
                                             (256, 4096, 32, 8, 128, 1000),
                                             (4736, 128, 8, 4, 64, 3)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_qkv_rope_equals_gemm_then_rope(cuda_dev, T, E, H, KV, D, pos0, dt):
    """The fused epilogue gives what the two launches give, bit for bit: the
    same fp32 accumulator, rotated with the same rounded products and stored
    with the same rounding."""
    from alpacca_open_sourced_by_jt_b200 import device
    g = torch.Generator(device=cuda_dev).manual_seed(T + E)
    n_ctx = pos0 + T + 5
    a = torch.randn((T, E), device=cuda_dev, generator=g).to(dt)
    w = (0.05 * torch.randn(((H + 2 * KV) * D, E), device=cuda_dev, generator=g)).to(dt)
    cos, sin = device.rope_tables(n_ctx, D, 10000.0, device=cuda_dev)
    pos = torch.arange(pos0, pos0 + T, dtype=torch.int32, device=cuda_dev)
    kc0, vc0 = (torch.zeros((1, n_ctx, KV, D), device=cuda_dev, dtype=dt) for _ in range(2))
    q0 = torch.zeros((T, H, D), device=cuda_dev, dtype=dt)
    qkv = device.gemm(a, w)
    qd, kd = H * D, KV * D
    device.rope_append(qkv[:, :qd].view(T, H, D), qkv[:, qd:qd + kd].view(T, KV, D),
                       qkv[:, qd + kd:].view(T, KV, D), pos, cos, sin, k_cache=kc0,
                       v_cache=vc0, q_out=q0)
    kc1, vc1 = torch.zeros_like(kc0), torch.zeros_like(vc0)
    q1 = torch.zeros_like(q0)
    device.gemm_qkv_rope(a, w, pos, cos, sin, H=H, KV=KV, k_cache=kc1, v_cache=vc1, q_out=q1)
    torch.cuda.synchronize()
    assert torch.equal(q1, q0)
    assert torch.equal(kc1, kc0) and torch.equal(vc1, vc0)
    assert kc1[0, pos0 + T:].abs().sum().item() == 0


def test_gemm_qkv_rope_position_outside_cache(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    _lib.device_error(clear=True)
    n_ctx, H, KV, D, E = 16, 2, 1, 64, 128
    a = torch.randn((2, E), device=cuda_dev).to(torch.bfloat16)
    w = torch.randn(((H + 2 * KV) * D, E), device=cuda_dev).to(torch.bfloat16)
    cos, sin = device.rope_tables(n_ctx, D, 10000.0, device=cuda_dev)
    kc = torch.zeros((n_ctx, KV, D), device=cuda_dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = torch.zeros((2, H, D), device=cuda_dev, dtype=torch.bfloat16)
    pos = torch.tensor([3, n_ctx], dtype=torch.int32, device=cuda_dev)  # second is out of range
    device.gemm_qkv_rope(a, w, pos, cos, sin, H=H, KV=KV, k_cache=kc, v_cache=vc, q_out=q)
    code, aux = _lib.device_error(clear=True)
    assert code == _lib.ERR_POSITION and aux == 1
    assert kc[3].abs().sum().item() > 0 and q[0].abs().sum().item() > 0
    assert q[1].abs().sum().item() == 0
    assert kc[4:].abs().sum().item() == 0 and vc[4:].abs().sum().item() == 0
