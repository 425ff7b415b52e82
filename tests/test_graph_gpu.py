"""CUDA-graph capture of the hot path: a decode step (fused RoPE+append then
split-KV decode) and a prefill chunk (RoPE+append to a bf16 q buffer then
the tcgen05 prefill) are captured once and replayed with new tokens,
positions and lengths written into the same device buffers between replays
(the capturability the qwen35_cuda_graph wiring needs: no host scalars that
change per token)."""
import math

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_decode_step_graph_replays_with_new_positions(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(50)
    B, H, KV, D, n_ctx = 4, 32, 8, 128, 2048
    cos, sin = oracle.rope_tables(n_ctx, D, 500000.0)
    ct, st = torch.from_numpy(cos).to(cuda_dev), torch.from_numpy(sin).to(cuda_dev)
    kc = torch.randn((B, n_ctx, KV, D), device=cuda_dev).to(torch.bfloat16)
    vc = torch.randn((B, n_ctx, KV, D), device=cuda_dev).to(torch.bfloat16)
    q_in = torch.zeros((B, H, D), device=cuda_dev)
    k_in = torch.zeros((B, KV, D), device=cuda_dev)
    v_in = torch.zeros((B, KV, D), device=cuda_dev)
    pos = torch.zeros(B, dtype=torch.int32, device=cuda_dev)
    lens = torch.ones(B, dtype=torch.int32, device=cuda_dev)
    out = torch.empty((B, H, D), device=cuda_dev)
    split = 256
    ws = device.decode_workspace(B, H, D, n_ctx, split, cuda_dev)

    def step():
        device.rope_append(q_in, k_in, v_in, pos, ct, st, k_cache=kc, v_cache=vc,
                           per_sequence=True)
        device.decode(q_in, kc, vc, lens, out=out, workspace=ws, split_rows=split, max_len=n_ctx)

    step()  # eager warm-up (kernel attributes, tensor maps); appends a zero row 0
    torch.cuda.synchronize()
    k_host = kc.float().cpu().numpy()  # host mirror of the caches from here on
    v_host = vc.float().cpu().numpy()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for it in range(3):
        p = rng.integers(0, n_ctx, size=B).astype(np.int32)
        q = rng.standard_normal((B, H, D), dtype=np.float32)
        k = rng.standard_normal((B, KV, D), dtype=np.float32)
        v = rng.standard_normal((B, KV, D), dtype=np.float32)
        q_in.copy_(torch.from_numpy(q))
        k_in.copy_(torch.from_numpy(k))
        v_in.copy_(torch.from_numpy(v))
        pos.copy_(torch.from_numpy(p))
        lens.copy_(torch.from_numpy(p + 1))
        g.replay()
        torch.cuda.synchronize()
        # reference: same append into host caches (rows cast to bf16), then decode
        kr = np.zeros((B, n_ctx, KV, D), np.float32)
        vr = np.zeros_like(kr)
        qr = oracle.rope_append(q, k, v, p, kr, vr, cos, sin, D, "norm",
                                seq_of_token=np.arange(B))
        for b in range(B):
            k_host[b, p[b]] = torch.from_numpy(kr[b, p[b]]).to(torch.bfloat16).float().numpy()
            v_host[b, p[b]] = torch.from_numpy(vr[b, p[b]]).to(torch.bfloat16).float().numpy()
        assert np.array_equal(q_in.cpu().numpy(), qr)
        got = out.cpu().numpy()
        for b in range(B):
            n = int(p[b]) + 1
            ref = oracle.attention_decode(qr[b], k_host[b, :n], v_host[b, :n], H // KV,
                                          1 / math.sqrt(D))
            assert np.abs(got[b] - ref).max() < 2e-2, (it, b)


def test_prefill_chunk_graph_replays_with_new_offsets(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    rng = np.random.default_rng(51)
    T, H, KV, D, n_ctx = 192, 16, 4, 128, 1024
    cos, sin = oracle.rope_tables(n_ctx, D, 500000.0)
    ct, st = torch.from_numpy(cos).to(cuda_dev), torch.from_numpy(sin).to(cuda_dev)
    # a zero-initialised cache: rows past the written positions hold finite values
    kc = torch.zeros((n_ctx, KV, D), dtype=torch.bfloat16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    q_in = torch.zeros((T, H, D), device=cuda_dev)
    k_in = torch.zeros((T, KV, D), device=cuda_dev)
    v_in = torch.zeros((T, KV, D), device=cuda_dev)
    pos = torch.zeros(T, dtype=torch.int32, device=cuda_dev)
    q16 = torch.empty((T, H, D), dtype=torch.bfloat16, device=cuda_dev)
    out = torch.empty((T, H, D), dtype=torch.float32, device=cuda_dev)

    def chunk():
        device.rope_append(q_in, k_in, v_in, pos, ct, st, k_cache=kc, v_cache=vc, q_out=q16)
        # t_kv is the cache capacity: the positions decide what each query sees
        device.prefill(q16, kc, vc, pos, out=out)

    chunk()
    torch.cuda.synchronize()
    kc.zero_()
    vc.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chunk()
    k_host = np.zeros((1, n_ctx, KV, D), np.float32)
    v_host = np.zeros_like(k_host)
    for start in (0, T, 2 * T + 17):
        q = rng.standard_normal((T, H, D), dtype=np.float32)
        k = rng.standard_normal((T, KV, D), dtype=np.float32)
        v = rng.standard_normal((T, KV, D), dtype=np.float32)
        p = np.arange(start, start + T, dtype=np.int32)
        q_in.copy_(torch.from_numpy(q))
        k_in.copy_(torch.from_numpy(k))
        v_in.copy_(torch.from_numpy(v))
        pos.copy_(torch.from_numpy(p))
        g.replay()
        torch.cuda.synchronize()
        kr = np.zeros_like(k_host)
        vr = np.zeros_like(v_host)
        qr = oracle.rope_append(q, k, v, p, kr, vr, cos, sin, D, "norm")
        k_host[0, p] = torch.from_numpy(kr[0, p]).to(torch.bfloat16).float().numpy()
        v_host[0, p] = torch.from_numpy(vr[0, p]).to(torch.bfloat16).float().numpy()
        q16_ref = torch.from_numpy(qr).to(torch.bfloat16).float().numpy()
        ref = oracle.attention_batch(q16_ref, k_host[0, :start + T], v_host[0, :start + T], p,
                                     H // KV, 1 / math.sqrt(D))
        got = out.cpu().numpy().reshape(T, -1)
        assert np.abs(got - ref).max() < 2e-2, start
