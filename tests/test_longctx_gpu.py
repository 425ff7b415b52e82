"""Long-context split decode across GPUs (one process per GPU).

Each rank decodes its share of the KV rows; the parts meet either through
the fused peer-memory kernel (b2a_decode_sharded: split merge, NVLink peer
stores of every rank's (o, lse) rows, bounded flag waits, LSE merge) or
through an NCCL all-gather and the LSE-combine kernel.  Both must match the
unsharded decode.  The multi-GPU tests are skipped on a box with fewer GPUs;
the one-rank tests run the same kernel with G = 1, and the timeout test
makes a wait run out on a flag that no rank sets.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shards(dev, B, L, KV, D, lengths, a, b, seed=3):
    g = torch.Generator(device=dev).manual_seed(seed)  # the same full cache on every rank
    K = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    V = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    ks = K[:, a:b].contiguous()
    vs = V[:, a:b].contiguous()
    lens = torch.tensor([max(0, min(n, b) - a) for n in lengths], dtype=torch.int32, device=dev)
    return K, V, ks, vs, lens


def test_p2p_one_rank_matches_decode(cuda_dev):
    """G = 1: the fused kernel publishes to and waits on its own buffer;
    several steps in a row alternate the exchange slots."""
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.longctx import LongContextDecoder
    B, H, KV, D, L = 3, 32, 8, 128, 5000
    lengths = [L, 4097, 0]
    K, V, ks, vs, lens = _shards(cuda_dev, B, L, KV, D, lengths, 0, L)
    dec = LongContextDecoder(exchange="p2p")
    full_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_dev)
    for step in range(5):
        q = torch.randn((B, H, D), device=cuda_dev)
        out = dec.decode(q, ks, vs, lens, max_len=L)
        want = device.decode(q, K, V, full_lens)
        torch.cuda.synchronize()
        assert (out - want).abs().max().item() < 1e-5, step
    from alpacca_open_sourced_by_jt_b200 import _lib
    assert _lib.device_error(clear=True) == (0, 0)


def test_p2p_graph_replay_one_rank(cuda_dev):
    """The captured step replays for new queries and new lengths."""
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.longctx import LongContextDecoder
    B, H, KV, D, L = 2, 16, 2, 256, 3000
    K, V, ks, vs, lens = _shards(cuda_dev, B, L, KV, D, [L, L], 0, L, seed=5)
    q = torch.randn((B, H, D), device=cuda_dev)
    dec = LongContextDecoder(exchange="p2p")
    replay, out = dec.graph(q, ks, vs, lens, max_len=L)
    for n0, n1 in ((3000, 1), (17, 2999), (1500, 64)):
        q.copy_(torch.randn((B, H, D), device=cuda_dev))
        lens.copy_(torch.tensor([n0, n1], dtype=torch.int32))
        replay()
        want = device.decode(q, K, V, lens.clone(), max_len=L)
        torch.cuda.synchronize()
        assert (out - want).abs().max().item() < 1e-5


def test_p2p_wait_times_out_and_reports(cuda_dev):
    """A rank whose peer never arrives: one process calls with G = 2 and a
    peer table of two local buffers, so no one sets the second rank's
    flags.  The bounded wait runs out (about two seconds), the kernel
    records B2A_ERR_TIMEOUT and returns, and the context stays usable."""
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    _lib.device_error(clear=True)
    B, H, KV, D, L = 1, 8, 2, 64, 300
    K, V, ks, vs, lens = _shards(cuda_dev, B, L, KV, D, [L], 0, L)
    n = int(_lib.load().b2a_shard_exchange_bytes(B, H, D, 2))
    bufs = [torch.zeros(n, dtype=torch.uint8, device=cuda_dev) for _ in range(2)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda_dev)
    q = torch.randn((B, H, D), device=cuda_dev)
    device.decode_sharded(q, ks, vs, lens, table, 0, 2, max_len=L)
    code, aux = _lib.device_error(clear=True)
    assert code == _lib.ERR_TIMEOUT and (aux & 0xF0000) == 0x50000
    out = device.decode(q, K, V, torch.tensor([L], dtype=torch.int32, device=cuda_dev))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert _lib.device_error(clear=True) == (0, 0)


def _worker(rank, world, port, rq):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    errs = {}
    graphs = []
    try:
        from alpacca_open_sourced_by_jt_b200 import _lib, device
        from alpacca_open_sourced_by_jt_b200.longctx import LongContextDecoder
        B, H, KV, D, L = 2, 64, 8, 128, 10000
        lengths = [L, 7777]
        full_lens = torch.tensor(lengths, dtype=torch.int32, device=dev)
        for mode in ("nccl", "p2p"):
            dec = LongContextDecoder(exchange=mode)
            a, b = dec.rows(L)
            K, V, ks, vs, lens = _shards(dev, B, L, KV, D, lengths, a, b)
            worst = 0.0
            for step in range(4):
                gq = torch.Generator(device=dev).manual_seed(100 + step)  # same q on every rank
                q = torch.randn((B, H, D), device=dev, generator=gq)
                out = dec.decode(q, ks, vs, lens, max_len=b - a)
                full = device.decode(q, K, V, full_lens)
                torch.cuda.synchronize()
                worst = max(worst, (out - full).abs().max().item())
            if mode == "p2p":
                replay, gout = dec.graph(q, ks, vs, lens, max_len=b - a)
                graphs.append(replay)
                for step in range(3):
                    gq = torch.Generator(device=dev).manual_seed(200 + step)
                    q.copy_(torch.randn((B, H, D), device=dev, generator=gq))
                    replay()
                    full = device.decode(q, K, V, full_lens)
                    torch.cuda.synchronize()
                    worst = max(worst, (gout - full).abs().max().item())
                dec.close()
            errs[mode] = worst
        errs["device_error"] = _lib.device_error(clear=True)
        rq.put((rank, errs))
    finally:
        graphs.clear()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_split_decode_matches_unsharded(cuda_dev, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(rq.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, errs in res.items():
        assert errs["device_error"] == (0, 0), (r, errs)
        assert errs["nccl"] < 1e-3, (r, errs)
        assert errs["p2p"] < 1e-3, (r, errs)
