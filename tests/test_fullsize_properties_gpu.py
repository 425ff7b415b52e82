"""Decode at the benchmark's full sizes, checked through properties that hold at
any size (the oracle's NumPy einsum would take minutes there):

* the headline workload (16 sequences x 32768 rows, 32 q / 8 KV heads,
  head_dim 128, bf16): decoding the two halves of the cache and merging them
  by their log-sum-exp (b2a_lse_combine, the merge of cuda.py:674-694) gives
  the full decode to 1e-5 normwise.  Every call uses the full decode's split
  size and the halves start on split boundaries, so each split's partial
  (its own max, and P rounded to 16 bits against it) is the same; only the
  fp32 merge is grouped differently;
  and with every V row of a KV head equal to one vector c, the output is c
  to within the 16-bit rounding of P (2^-9 relative), because the softmax
  weights sum to one;
* config 4 (4 sequences x 131072 rows, 64 q / 8 KV heads): four row shards
  merged equal the unsharded decode to 1e-5 normwise, the single-GPU
  statement of the multi-GPU split;
* config 3 (64 sequences, lengths uniform in [1024, 8192] from seed 2, fp16
  cache): every sequence of the batch equals that sequence decoded alone
  with the same split size, bit for bit (no cross-sequence state);
* config 2 (causal prefill, 2048 tokens, 32 q / 8 KV heads, head_dim 128,
  bf16): the chunk in two halves (the second over the whole key range,
  split on a 128-row query tile) equals the single call bit for bit, for the
  paired-head and the one-head kernels, since every query tile visits the
  same key tiles in the same order either way.
"""
import numpy as np
import pytest
import torch

from tests.conftest import max_abs_err, rel_err

pytestmark = pytest.mark.gpu


def _rand(shape, dt, dev, g):
    return torch.randn(shape, device=dev, generator=g).to(dt)


def _shard_decode(device, q, k, v, L, n_shards, split):
    """Decode each of n_shards row ranges with its lse, then merge."""
    B, H, D = q.shape
    rows = L // n_shards
    assert rows % split == 0
    outs, lses = [], []
    for i in range(n_shards):
        sl = slice(i * rows, (i + 1) * rows)
        lens = torch.full((B,), rows, dtype=torch.int32, device=q.device)
        lse = torch.empty((B, H), device=q.device)
        outs.append(device.decode(q, k[:, sl], v[:, sl], lens, lse=lse, split_rows=split))
        lses.append(lse)
    o = torch.stack([x.view(B * H, D) for x in outs])
    ls = torch.stack([x.view(B * H) for x in lses])
    return device.lse_combine(o, ls).view(B, H, D)


def test_headline_halves_and_constant_values(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    B, L, H, KV, D = 16, 32768, 32, 8, 128
    g = torch.Generator(device=cuda_dev).manual_seed(4)
    q = torch.randn((B, H, D), device=cuda_dev, generator=g)
    k = _rand((B, L, KV, D), torch.bfloat16, cuda_dev, g)
    v = _rand((B, L, KV, D), torch.bfloat16, cuda_dev, g)
    lens = torch.full((B,), L, dtype=torch.int32, device=cuda_dev)
    split = device.decode_split_rows(B, KV, L, torch.bfloat16)
    full = device.decode(q, k, v, lens, split_rows=split)
    merged = _shard_decode(device, q, k, v, L, 2, split)
    torch.cuda.synchronize()
    assert rel_err(merged.cpu().numpy(), full.cpu().numpy()) < 1e-5
    # every V row of a (sequence, KV head) equal to one vector c
    c = _rand((B, 1, KV, D), torch.bfloat16, cuda_dev, g)
    v.copy_(c.expand(B, L, KV, D))
    out = device.decode(q, k, v, lens)
    torch.cuda.synchronize()
    want = c.float().squeeze(1).repeat_interleave(H // KV, dim=1)  # (B, H, D)
    scale = float(want.abs().max())
    assert max_abs_err(out.cpu().numpy(), want.cpu().numpy()) < 2 ** -9 * scale * 2


def test_config4_shards_merge_to_full(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    B, L, H, KV, D = 4, 131072, 64, 8, 128
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    q = torch.randn((B, H, D), device=cuda_dev, generator=g)
    k = _rand((B, L, KV, D), torch.bfloat16, cuda_dev, g)
    v = _rand((B, L, KV, D), torch.bfloat16, cuda_dev, g)
    lens = torch.full((B,), L, dtype=torch.int32, device=cuda_dev)
    split = device.decode_split_rows(B, KV, L, torch.bfloat16)
    full = device.decode(q, k, v, lens, split_rows=split)
    merged = _shard_decode(device, q, k, v, L, 4, split)
    torch.cuda.synchronize()
    assert rel_err(merged.cpu().numpy(), full.cpu().numpy()) < 1e-5


def test_config3_batch_equals_each_sequence_alone(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    B, Lmax, H, KV, D = 64, 8192, 32, 8, 128
    lens_np = np.random.default_rng(2).integers(1024, 8193, size=B).astype(np.int32)
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    q = torch.randn((B, H, D), device=cuda_dev, generator=g)
    k = _rand((B, Lmax, KV, D), torch.float16, cuda_dev, g)
    v = _rand((B, Lmax, KV, D), torch.float16, cuda_dev, g)
    lens = torch.from_numpy(lens_np).to(cuda_dev)
    split = device.decode_split_rows(B, KV, Lmax, torch.float16)
    batch = device.decode(q, k, v, lens, split_rows=split, max_len=Lmax)
    for b in range(B):
        one = device.decode(q[b:b + 1].contiguous(), k[b:b + 1], v[b:b + 1], lens[b:b + 1],
                            split_rows=split, max_len=Lmax)
        assert torch.equal(one[0], batch[b]), b


@pytest.mark.parametrize("kernel", ["pair", "head"])
def test_config2_prefill_in_two_chunks_is_bit_identical(cuda_dev, monkeypatch, kernel):
    from alpacca_open_sourced_by_jt_b200 import device
    if kernel == "head":
        monkeypatch.setenv("B2ATTN_PREFILL", "head")
    else:
        monkeypatch.delenv("B2ATTN_PREFILL", raising=False)
    S, H, KV, D = 2048, 32, 8, 128
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    q = _rand((S, H, D), torch.bfloat16, cuda_dev, g)
    k = _rand((S, KV, D), torch.bfloat16, cuda_dev, g)
    v = _rand((S, KV, D), torch.bfloat16, cuda_dev, g)
    pos = torch.arange(S, dtype=torch.int32, device=cuda_dev)
    full = device.prefill(q, k, v, pos)
    h = S // 2
    first = device.prefill(q[:h].contiguous(), k[:h].contiguous(), v[:h].contiguous(), pos[:h].contiguous())
    second = device.prefill(q[h:].contiguous(), k, v, pos[h:].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([first, second]), full)

