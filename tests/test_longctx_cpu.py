"""Host logic of the multi-GPU decode on CPU ranks (gloo, world size 2 and
3), with the NumPy oracle standing in for the device kernels: the
long-context split (row sharding, the gather and the merge order) and the
ragged batch sharded by whole sequences (placement and the ordered gather).
Also a failure case: a rank that never joins makes the others fail with a
timeout instead of hanging."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from alpacca_open_sourced_by_jt_b200.longctx import (LongContextDecoder, gather_placed,
                                                     place_sequences, shard_lengths, shard_rows)


def test_shard_rows_cover_exactly():
    for L in (0, 1, 7, 131072, 131073):
        for world in (1, 2, 3, 8):
            ranges = [shard_rows(L, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == L
            for (a0, b0), (a1, _) in zip(ranges, ranges[1:]):
                assert b0 == a1
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    assert shard_lengths([10, 3], 1, 4) == [3, 1]
    with pytest.raises(ValueError):
        shard_rows(5, 2, 2)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_place_sequences_balances_rows(world):
    lens = np.random.default_rng(2).integers(1024, 8192 + 1, size=64)
    placed = place_sequences(lens, world)
    assert len(placed) == world
    assert sorted(i for p in placed for i in p) == list(range(64))  # each sequence once
    counts = [len(p) for p in placed]
    assert max(counts) - min(counts) <= 1
    assert all(p == sorted(p) for p in placed)
    loads = [int(lens[p].sum()) for p in placed]
    dealt = [int(lens[r::world].sum()) for r in range(world)]
    assert max(loads) <= max(dealt)
    # within one sequence's length of a perfect split
    assert max(loads) - lens.sum() / world <= lens.max()
    if world == 8:
        assert max(loads) / (lens.sum() / world) < 1.02


def test_place_sequences_edges():
    assert place_sequences([], 4) == [[], [], [], []]
    assert place_sequences([5], 3) == [[0], [], []]
    assert place_sequences([1, 9, 9, 1], 2) == [[0, 1], [2, 3]]
    with pytest.raises(ValueError):
        place_sequences([3], 0)
    with pytest.raises(ValueError):
        place_sequences([-1], 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _np_partial(q, k, v, lens, scale, max_len, out, lse):
    """Oracle stand-in for b2a_decode with lse_out, writing into the views."""
    q = q.numpy()
    B, H, D = q.shape
    KV = k.shape[2]
    o = np.zeros((B, H, D))
    ls = np.full((B, H), -np.inf)
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            continue
        pm, pl, pacc = oracle.split_decode_partials(q[b], k[b, :n].numpy(), v[b, :n].numpy(),
                                                    H // KV, scale, 10 ** 9)
        o[b] = pacc[:, 0] / pl[:, :1]
        ls[b] = pm[:, 0] + np.log(pl[:, 0])
    out.copy_(torch.from_numpy(o))
    lse.copy_(torch.from_numpy(ls))


def _np_combine(o_all, lse_all, out):
    res, _ = oracle.lse_combine(o_all.numpy(), lse_all.numpy())
    out.copy_(torch.from_numpy(res))


def _worker(rank, world, port, q, K, V, lengths, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        dec = LongContextDecoder(partial_fn=_np_partial, combine_fn=_np_combine)
        B, L = K.shape[0], K.shape[1]
        a, b = dec.rows(L)
        lens = torch.tensor(shard_lengths(lengths, rank, world))
        # this rank's rows of every sequence, re-based at 0 (a shard's local cache)
        ks = torch.zeros((B, max(b - a, 1)) + K.shape[2:])
        vs = torch.zeros_like(ks)
        for s in range(B):
            sa, sb = shard_rows(int(lengths[s]), rank, world)
            ks[s, :sb - sa] = K[s, sa:sb]
            vs[s, :sb - sa] = V[s, sa:sb]
        out = dec.decode(q, ks, vs, lens, scale=0.125)
        result_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_decode_on_gloo_ranks_matches_unsharded(world):
    rng = np.random.default_rng(40 + world)
    B, H, KV, D, L = 3, 8, 2, 16, 50
    q = torch.from_numpy(rng.standard_normal((B, H, D), dtype=np.float32))
    K = torch.from_numpy(rng.standard_normal((B, L, KV, D), dtype=np.float32))
    V = torch.from_numpy(rng.standard_normal((B, L, KV, D), dtype=np.float32))
    lengths = [50, 1, 29]  # sequence 1 leaves every rank but rank 0 empty
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, K, V, lengths, rq))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(rq.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for b in range(B):
        ref = oracle.attention_decode(q[b].numpy(), K[b, :lengths[b]].numpy(),
                                      V[b, :lengths[b]].numpy(), H // KV, 0.125)
        for r in range(world):
            assert np.abs(results[r][b] - ref).max() < 1e-5


def _placed_worker(rank, world, port, q, K, V, lengths, result_q):
    """Config 3's layout: each rank decodes whole sequences (the oracle in
    place of the device decode), then gathers the batch in order."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        placed = place_sequences(lengths, world)
        H, KV = q.shape[1], K.shape[2]
        mine = [oracle.attention_decode(q[b].numpy(), K[b, :lengths[b]].numpy(),
                                        V[b, :lengths[b]].numpy(), H // KV, 0.125)
                for b in placed[rank]]
        local = torch.from_numpy(np.stack(mine)) if mine else torch.zeros((0,) + q.shape[1:])
        result_q.put((rank, gather_placed(local, placed).numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_placed_batch_on_gloo_ranks_matches_unsharded(world):
    rng = np.random.default_rng(60 + world)
    B, H, KV, D, L = 7, 8, 2, 16, 40
    q = torch.from_numpy(rng.standard_normal((B, H, D), dtype=np.float32))
    K = torch.from_numpy(rng.standard_normal((B, L, KV, D), dtype=np.float32))
    V = torch.from_numpy(rng.standard_normal((B, L, KV, D), dtype=np.float32))
    lengths = [40, 3, 17, 29, 1, 33, 8]
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_placed_worker, args=(r, world, port, q, K, V, lengths, rq))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(rq.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for b in range(B):
        ref = oracle.attention_decode(q[b].numpy(), K[b, :lengths[b]].numpy(),
                                      V[b, :lengths[b]].numpy(), H // KV, 0.125)
        for r in range(world):
            assert np.array_equal(results[r][b], ref.astype(np.float32))


def _lonely_worker(port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    try:
        # world size 2, but rank 1 never starts: rendezvous must time out
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        result_q.put("joined")
    except Exception as e:  # noqa: BLE001
        result_q.put(type(e).__name__)


def test_missing_rank_fails_with_timeout_not_hang():
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(_free_port(), rq))
    p.start()
    res = rq.get(timeout=120)
    p.join(timeout=30)
    assert res != "joined"
