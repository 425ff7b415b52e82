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

Two exchanges are provided:
  "p2p"   (default on GPUs) one fused kernel (b2a_decode_sharded) merges the
          rank's split partials, stores its (o, lse) rows straight into
          every rank's exchange buffer over NVLink (plain peer stores through
          CUDA-IPC mappings set up once by PeerExchange), waits for the
          other ranks' rows and merges them: no collective call, one launch
          after the split kernel, and the step can be replayed as a CUDA
          graph (`graph()`).
  "nccl"  the decode with lse, one NCCL all_gather_into_tensor of the
          packed parts, and the LSE-combine kernel.
The host logic (row ranges, gather, ordering) is independent of the device
kernels: `partial_fn` and `combine_fn` default to the B200 kernels and can be
replaced (the CPU tests run the "nccl" exchange on gloo ranks with the NumPy
oracle).

A ragged batch of many shorter sequences is sharded by whole sequences
instead (no exchange at all): `place_sequences` balances the ranks' rows and
`gather_placed` brings the outputs back in batch order where a caller wants
them in one place.
"""
from __future__ import annotations

import ctypes
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


def place_sequences(lengths, world: int) -> list[list[int]]:
    """Whole sequences of a ragged batch placed on `world` ranks, for a batch
    sharded by sequence (each rank decodes its sequences alone, no exchange).

    A decode step reads every cached row once, so a rank's time follows the
    sum of its sequences' lengths and the step waits for the busiest rank.
    Sequences are taken longest first and each goes to the rank with the
    fewest rows so far among the ranks that still hold fewer than
    ceil(B / world) sequences (the batch shapes stay equal to within one
    sequence).  Ties go to the lower rank; each rank's list is returned in
    ascending batch order.  For 64 lengths uniform in [1024, 8192] the
    busiest of 8 ranks holds 1.01x the mean rows; dealing sequences out
    round-robin gives 1.22x."""
    if world <= 0:
        raise ValueError(f"bad world size {world}")
    lens = [int(L) for L in lengths]
    if any(L < 0 for L in lens):
        raise ValueError("lengths must be non-negative")
    cap = -(-len(lens) // world)
    loads = [0] * world
    placed: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        r = min((r for r in range(world) if len(placed[r]) < cap), key=lambda r: (loads[r], r))
        placed[r].append(i)
        loads[r] += lens[i]
    return [sorted(p) for p in placed]


def gather_placed(out_local: torch.Tensor, placed: list[list[int]], group=None) -> torch.Tensor:
    """A batch decoded by whole sequences per rank (place_sequences), back in
    batch order on every rank.

    out_local holds this rank's outputs, one row per sequence of
    placed[rank] in that order.  Returns (B, ...) where row i is sequence i's
    output.  One all_gather of equal-size blocks (each rank's rows padded to
    the largest count); the decode itself needs no exchange, this is only for
    callers that want every output in one place."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if len(placed) != world:
        raise ValueError(f"placement for {len(placed)} ranks, group of {world}")
    mine = placed[rank]
    if out_local.shape[0] != len(mine):
        raise ValueError(f"{out_local.shape[0]} output rows for {len(mine)} sequences")
    cap = max(1, max(len(p) for p in placed))
    buf = out_local.new_zeros((cap,) + tuple(out_local.shape[1:]))
    buf[:len(mine)] = out_local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    out = out_local.new_empty((sum(len(p) for p in placed),) + tuple(out_local.shape[1:]))
    for r, idx in enumerate(placed):
        if idx:
            out[torch.tensor(idx, device=out.device)] = parts[r][:len(idx)]
    return out


def _gpu_partial(q, k_shard, v_shard, lens_shard, scale, max_len, out, lse):
    from . import device
    device.decode(q, k_shard, v_shard, lens_shard, scale=scale, max_len=max_len, out=out, lse=lse)


def _gpu_combine(o_all, lse_all, out):
    from . import device
    device.lse_combine(o_all, lse_all, out=out)


class PeerExchange:
    """Every rank's exchange buffer for b2a_decode_sharded, mapped into this
    process.  Each rank allocates its buffer (b2a_shard_exchange_bytes,
    zeroed), publishes its CUDA-IPC handle with one all-gather, opens the
    others' handles (peer access over NVLink) and keeps a device table of
    the G buffer addresses.  Construction is collective: every rank of
    `group` must build one with the same (B, H, D), and a barrier at the end
    makes sure every buffer is zeroed and mapped before any rank's first
    step writes into it."""

    def __init__(self, B: int, H: int, D: int, group=None, device=None):
        from . import _lib
        lib = _lib.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.shape = (B, H, D)
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = int(lib.b2a_shard_exchange_bytes(B, H, D, self.world))
        if nbytes <= 0:
            raise ValueError("bad exchange shape")
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_longlong(0)
        _lib.check(lib.b2a_ipc_handle(self.buf.data_ptr(), handle, ctypes.byref(offset)))
        rec = bytes(handle) + int(offset.value).to_bytes(8, "little", signed=True)
        mine = torch.frombuffer(bytearray(rec), dtype=torch.uint8).to(dev)
        every = torch.empty((self.world, len(rec)), dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().numpy()
        self._bases = []
        addrs = []
        for g in range(self.world):
            if g == self.rank:
                addrs.append(self.buf.data_ptr())
                continue
            h = bytes(every[g, :64])
            off = int.from_bytes(bytes(every[g, 64:72]), "little", signed=True)
            base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(lib.b2a_ipc_open(h, off, ctypes.byref(base), ctypes.byref(ptr)))
            self._bases.append(base.value)
            addrs.append(ptr.value)
        self.table = torch.tensor(addrs, dtype=torch.int64, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the peers' buffers (collective: no rank may still be
        stepping)."""
        from . import _lib
        lib = _lib.load()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for b in self._bases:
            _lib.check(lib.b2a_ipc_close(b))
        self._bases = []


class LongContextDecoder:
    """Decode one query token per sequence over a KV cache whose rows are
    sharded across the ranks of `group`.

    Each rank's decode writes its normalised output and its lse into one
    packed f32 buffer [B*H*D | B*H]; a single all_gather_into_tensor moves
    every rank's packed buffer (one collective per step), and the combine
    kernel reads the gathered parts in place through their strides."""

    def __init__(self, group=None, partial_fn: Callable | None = None,
                 combine_fn: Callable | None = None, exchange: str = "nccl"):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
        else:  # single process: one shard holding every row
            self.rank, self.world = 0, 1
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', not {exchange!r}")
        if exchange == "p2p" and (partial_fn or combine_fn):
            raise ValueError("the p2p exchange runs the fused device kernel only")
        if exchange == "p2p" and self.world > 1 and dist.get_backend(group) != "nccl":
            raise ValueError("the p2p exchange needs GPU ranks (an nccl process group)")
        self.exchange = exchange
        self.partial_fn = partial_fn or _gpu_partial
        self.combine_fn = combine_fn or _gpu_combine
        self._bufs = {}
        self._peers = {}
        self._ws = {}

    def peers(self, B: int, H: int, D: int, device) -> "PeerExchange | None":
        """The exchange buffers for this shape (built collectively on first
        use; every rank must reach this call)."""
        key = (B, H, D, str(device))
        px = self._peers.get(key)
        if px is None:
            if self.world == 1:
                px = _SoloExchange(B, H, D, device)
            else:
                px = PeerExchange(B, H, D, group=self.group, device=device)
            self._peers[key] = px
        return px

    def close(self) -> None:
        for px in self._peers.values():
            px.close()
        self._peers = {}

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
        if self.exchange == "p2p":
            from . import device as _device
            px = self.peers(B, H, D, q.device)
            out = self.buffers(B, H, D, q.device)[2]
            ws = self._workspace(B, H, D, k_shard, max_len)
            return _device.decode_sharded(q, k_shard, v_shard, lens_shard, px.table, self.rank,
                                          self.world, scale=scale, max_len=max_len, out=out,
                                          workspace=ws)
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

    def _workspace(self, B, H, D, k_shard, max_len):
        from . import device as _device
        n_ctx = k_shard.shape[-3]
        ml = n_ctx if max_len is None else int(max_len)
        KV = k_shard.shape[-2]
        key = (B, H, D, KV, ml, k_shard.dtype, str(k_shard.device))
        ws = self._ws.get(key)
        if ws is None:
            split = _device.decode_split_rows(B, KV, ml, k_shard.dtype)
            ws = self._ws[key] = _device.decode_workspace(B, H, D, ml, split, k_shard.device)
        return ws

    def graph(self, q, k_shard, v_shard, lens_shard, *, scale=None, max_len=None):
        """Capture one decode step (p2p exchange) as a CUDA graph and return
        (replay, out): replay() reruns the step on the current contents of
        q, the shards and lens_shard (lengths are read on the device), and
        out holds the merged rows.  Collective like decode(): every rank
        captures, and replays, the same steps in the same order.  The
        capture runs one step (warm-up) eagerly first."""
        if self.exchange != "p2p":
            raise ValueError("graph() captures the p2p exchange (no collective in the graph)")
        out = self.decode(q, k_shard, v_shard, lens_shard, scale=scale, max_len=max_len)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.decode(q, k_shard, v_shard, lens_shard, scale=scale, max_len=max_len)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        return g.replay, out


class _SoloExchange:
    """The one-rank case of PeerExchange: this process's own buffer only."""

    def __init__(self, B, H, D, device):
        from . import _lib
        n = int(_lib.load().b2a_shard_exchange_bytes(B, H, D, 1))
        self.buf = torch.zeros(n, dtype=torch.uint8, device=device)
        self.table = torch.tensor([self.buf.data_ptr()], dtype=torch.int64, device=device)

    def close(self) -> None:
        pass
