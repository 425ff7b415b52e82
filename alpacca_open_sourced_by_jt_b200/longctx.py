"""Long-context decode split across GPUs (one process per GPU).

The KV sequence of every sequence in the batch is cut into `world`
contiguous row ranges.  Rank r holds rows [start_r, stop_r) of each
sequence's cache and decodes its range with `lse_out` set.  The per-rank
normalised outputs and natural-log log-sum-exps are then all-gathered (NCCL
over NVLink on B200) and merged by the log-sum-exp combine kernel:

    out = sum_r exp(lse_r - L) * o_r,   L = log sum_r exp(lse_r)

That is the algebra of the reference's split combine
(alpaccaroo/cuda.py:674-694) lifted from CTAs to GPUs.  A rank whose range is
empty for a sequence contributes lse = -inf and weight 0.  The exchange is
B*H*(D+1)*4 bytes per rank (133 KB for 4 sequences x 64 heads x 128), so the
step is latency-bound, not bandwidth-bound.

The host logic (row ranges, gather, ordering) is independent of the device
kernels: `partial_fn` and `combine_fn` default to the B200 kernels and can be
replaced (the CPU tests run it on gloo ranks with the NumPy oracle).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_rows(length: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced row range [start, stop) of `length` rows for
    `rank` of `world` (the first length % world ranks get one extra row)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if length < 0:
        raise ValueError("length must be non-negative")
    base, extra = divmod(length, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_lengths(lengths, rank: int, world: int) -> list[int]:
    """Per-sequence number of rows rank `rank` holds."""
    out = []
    for L in lengths:
        a, b = shard_rows(int(L), rank, world)
        out.append(b - a)
    return out


def _gpu_partial(q, k_shard, v_shard, lens_shard, scale, max_len, out, lse):
    from . import device
    device.decode(q, k_shard, v_shard, lens_shard, scale=scale, max_len=max_len, out=out, lse=lse)


def _gpu_combine(o_all, lse_all, out):
    from . import device
    device.lse_combine(o_all, lse_all, out=out)


class LongContextDecoder:
    """Decode one query token per sequence over a KV cache whose rows are
    sharded across the ranks of `group`.

    Each rank's decode writes its normalised output and its lse into one
    packed f32 buffer [B*H*D | B*H]; a single all_gather_into_tensor moves
    every rank's packed buffer (one collective per step), and the combine
    kernel reads the gathered parts in place through their strides."""

    def __init__(self, group=None, partial_fn: Callable | None = None,
                 combine_fn: Callable | None = None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
        else:  # single process: one shard holding every row
            self.rank, self.world = 0, 1
        self.partial_fn = partial_fn or _gpu_partial
        self.combine_fn = combine_fn or _gpu_combine
        self._bufs = {}

    def rows(self, length: int) -> tuple[int, int]:
        return shard_rows(length, self.rank, self.world)

    def buffers(self, B: int, H: int, D: int, device) -> tuple:
        """(packed, gathered, out) for this shape, allocated once and reused
        so repeated steps (and a captured graph) see the same memory."""
        key = (B, H, D, str(device))
        bufs = self._bufs.get(key)
        if bufs is None:
            R = B * H
            packed = torch.empty(R * (D + 1), dtype=torch.float32, device=device)
            gathered = torch.empty((self.world, R * (D + 1)), dtype=torch.float32,
                                   device=device)
            out = torch.empty((B, H, D), dtype=torch.float32, device=device)
            bufs = self._bufs[key] = (packed, gathered, out)
        return bufs

    def decode(self, q, k_shard, v_shard, lens_shard, *, scale=None, max_len=None):
        """q (B, H, D) identical on every rank; k_shard/v_shard this rank's rows
        (B, n_local, KV, D); lens_shard (B,) int32 rows held here.  Returns the
        merged (B, H, D) f32 output (the same values on every rank)."""
        B, H, D = q.shape
        R = B * H
        if scale is None:
            scale = D ** -0.5
        packed, gathered, out = self.buffers(B, H, D, q.device)
        self.partial_fn(q, k_shard, v_shard, lens_shard, scale, max_len,
                        packed[:R * D].view(B, H, D), packed[R * D:].view(B, H))
        if self.world == 1:
            gathered[0].copy_(packed)
        elif dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(gathered, packed, group=self.group)
        else:  # gloo (CPU ranks) has no single-tensor all-gather
            dist.all_gather(list(gathered.unbind(0)), packed, group=self.group)
        o_all = gathered[:, :R * D].view(self.world, R, D)
        lse_all = gathered[:, R * D:]
        self.combine_fn(o_all, lse_all, out.view(R, D))
        return out
