"""Long-context split decode across 2 GPUs (NCCL, one process per GPU):
each rank decodes its half of the KV rows with the B200 kernel, the parts
are gathered and merged by the LSE-combine kernel; the result must match
the unsharded decode.  Skipped on a 1-GPU box."""
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


def _worker(rank, world, port, rq):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from alpacca_open_sourced_by_jt_b200 import device
        from alpacca_open_sourced_by_jt_b200.longctx import LongContextDecoder, shard_rows
        B, H, KV, D, L = 2, 64, 8, 128, 10000
        g = torch.Generator(device=dev).manual_seed(3)  # same full cache on every rank
        K = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
        V = torch.randn((B, L, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
        q = torch.randn((B, H, D), device=dev, generator=g)
        lengths = [L, 7777]
        dec = LongContextDecoder()
        a, b = dec.rows(L)
        ks = K[:, a:b].contiguous()
        vs = V[:, a:b].contiguous()
        lens = torch.tensor([max(0, min(n, b) - a) for n in lengths], dtype=torch.int32,
                            device=dev)
        out = dec.decode(q, ks, vs, lens, max_len=b - a)
        full = device.decode(q, K, V, torch.tensor(lengths, dtype=torch.int32, device=dev))
        err = (out - full).abs().max().item()
        rq.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_split_decode_matches_unsharded(cuda_dev):
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, rq)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(rq.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, err in res.items():
        assert err < 1e-3, (r, err)
