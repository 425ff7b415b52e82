"""the benchmark's 16-bit configurations at full size against a plain PyTorch fp32
reference of the same attention, computed on the GPU.

The CPU oracle would take minutes at these sizes; the fp32 reference here
is the textbook formula (the reference's NumPy algorithm, model.py:1231-1272:
scores = q . K^T * scale, causal mask, softmax, . V) evaluated by torch in
fp32 on the same 16-bit inputs, with K/V heads expanded for GQA.  Bar: the
16-bit KV bar of north_star, max abs error < 2e-2 on unit-variance inputs
(P is rounded to 16 bits in the kernels; the observed errors are ~1e-3).

* config 2: causal prefill, S=2048, 32 q / 8 KV heads, D=128, bf16 in and
  out, every query row and head (the paired-head and one-head kernels);
* head_dim 256 (Qwen35 full-attention geometry), S=2048, 16 q / 2 KV heads;
* config 4: one decode step of 4 sequences x 131072 rows, 64 q / 8 KV heads,
  D=128, bf16 (the unsharded decode, the N=1 point of the split);
* config 3: 64 sequences with lengths uniform in [1024, 8192] (seed 2), fp16.
"""
import math

import numpy as np
import pytest
import torch

from tests.conftest import max_abs_err

pytestmark = pytest.mark.gpu


def _prefill_ref(q, k, v, scale):
    """fp32 causal attention, q (S, H, D), k/v (S, KV, D) -> (S, H, D)."""
    S, H, D = q.shape
    KV = k.shape[1]
    g = H // KV
    qf = q.float().permute(1, 0, 2)                                  # (H, S, D)
    kf = k.float().permute(1, 0, 2).repeat_interleave(g, dim=0)      # (H, S, D)
    vf = v.float().permute(1, 0, 2).repeat_interleave(g, dim=0)
    out = torch.empty((H, S, D), dtype=torch.float32, device=q.device)
    mask = torch.ones((S, S), dtype=torch.bool, device=q.device).tril()
    for h0 in range(0, H, 8):  # 8 heads at a time keeps the scores at 128 MB
        s = torch.matmul(qf[h0:h0 + 8], kf[h0:h0 + 8].transpose(1, 2)) * scale
        s = s.masked_fill(~mask, float("-inf"))
        out[h0:h0 + 8] = torch.matmul(torch.softmax(s, dim=-1), vf[h0:h0 + 8])
    return out.permute(1, 0, 2)


def _decode_ref(q, k, v, lens, scale):
    """fp32 decode, q (B, H, D) f32, k/v (B, n_ctx, KV, D) -> (B, H, D)."""
    B, H, D = q.shape
    KV = k.shape[2]
    g = H // KV
    out = torch.empty((B, H, D), dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(lens[b])
        kf = k[b, :L].float()                                        # (L, KV, D)
        vf = v[b, :L].float()
        qg = q[b].view(KV, g, D)
        s = torch.einsum("kgd,lkd->kgl", qg, kf) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("kgl,lkd->kgd", p, vf).reshape(H, D)
    return out


@pytest.mark.parametrize("kernel", ["pair", "head"])
def test_config2_prefill_every_row_vs_fp32(cuda_dev, monkeypatch, kernel):
    from alpacca_open_sourced_by_jt_b200 import device
    monkeypatch.setenv("B2ATTN_PREFILL", kernel)
    S, H, KV, D = 2048, 32, 8, 128
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    q = torch.randn((S, H, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    k = torch.randn((S, KV, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    v = torch.randn((S, KV, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    pos = torch.arange(S, dtype=torch.int32, device=cuda_dev)
    out = device.prefill(q, k, v, pos)
    ref = _prefill_ref(q, k, v, 1.0 / math.sqrt(D))
    assert out.dtype == torch.bfloat16
    assert max_abs_err(out.float().cpu().numpy(), ref.cpu().numpy()) < 2e-2


def test_head_dim_256_prefill_every_row_vs_fp32(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    S, H, KV, D = 2048, 16, 2, 256
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    q = torch.randn((S, H, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    k = torch.randn((S, KV, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    v = torch.randn((S, KV, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    pos = torch.arange(S, dtype=torch.int32, device=cuda_dev)
    out = device.prefill(q, k, v, pos, out_dtype=torch.float32)
    ref = _prefill_ref(q, k, v, 1.0 / math.sqrt(D))
    assert max_abs_err(out.cpu().numpy(), ref.cpu().numpy()) < 2e-2


def test_config4_decode_vs_fp32(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    B, L, H, KV, D = 4, 131072, 64, 8, 128
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    k = torch.randn((B, L, KV, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    v = torch.randn((B, L, KV, D), device=cuda_dev, generator=g).to(torch.bfloat16)
    q = torch.randn((B, H, D), device=cuda_dev, generator=g)
    lens = torch.full((B,), L, dtype=torch.int32, device=cuda_dev)
    out = device.decode(q, k, v, lens)
    ref = _decode_ref(q, k, v, lens.cpu().tolist(), 1.0 / math.sqrt(D))
    assert max_abs_err(out.cpu().numpy(), ref.cpu().numpy()) < 2e-2


def test_config3_ragged_decode_vs_fp32(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    B, H, KV, D = 64, 32, 8, 128
    Ls = np.random.default_rng(2).integers(1024, 8192 + 1, size=B)
    n_ctx = 8192
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    k = torch.randn((B, n_ctx, KV, D), device=cuda_dev, generator=g).to(torch.float16)
    v = torch.randn((B, n_ctx, KV, D), device=cuda_dev, generator=g).to(torch.float16)
    q = torch.randn((B, H, D), device=cuda_dev, generator=g)
    lens = torch.from_numpy(Ls.astype(np.int32)).to(cuda_dev)
    out = device.decode(q, k, v, lens, max_len=n_ctx)
    ref = _decode_ref(q, k, v, Ls.tolist(), 1.0 / math.sqrt(D))
    assert max_abs_err(out.cpu().numpy(), ref.cpu().numpy()) < 2e-2
