"""A batched decode-attention step replayed as one CUDA graph.

The reference runs a decode token on the GPU as a fixed sequence of launches
(alpaccaroo/cuda.py:2082-2159, DecodeChain.step: per layer the rope/store
kernel, then the split attention kernels, cuda.py:2106-2127), and its Qwen35
runtime replays a whole token as one captured graph
(qwen35_cuda_graph.py:781-851).  DecodeStep does that for the attention part
of a step, from host memory to host memory:

    pinned host [q | k | v] (f32)  and  [positions | lengths] (int32)
      -> one H2D copy each
      -> fused bias-free RoPE + KV append at each sequence's own position
         (b2a_rope_append, per_sequence)
      -> split-KV decode over positions + 1 rows (b2a_decode)
      -> one D2H copy of the output into pinned host memory

Each call writes the step's inputs into the pinned staging buffers, replays
the graph (one launch) and waits for the output.  The caches stay resident;
the caller owns them and may read them between calls.  Nothing is allocated
per call.

Construction runs every kernel once on small private buffers (first-launch
set-up stays out of the capture) and then captures the step; it never
writes to the caller's caches.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib, device


class DecodeStep:
    """One decode token for a batch of sequences, as a replayable graph.

    k_cache/v_cache: (B, n_ctx, KV, D) f32/f16/bf16 CUDA tensors, one
    sequence per batch row (the reference's per-sequence cache layout,
    model.py:867-870).  cos_tab/sin_tab: the model's RoPE tables
    (device.rope_tables).  n_heads: query heads H (a multiple of KV).
    """

    def __init__(self, k_cache: torch.Tensor, v_cache: torch.Tensor, cos_tab: torch.Tensor,
                 sin_tab: torch.Tensor, n_heads: int, *, style: str = "norm",
                 scale: float | None = None, max_len: int | None = None):
        _lib.load()
        if k_cache.dim() != 4 or k_cache.shape != v_cache.shape or not k_cache.is_cuda:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, "caches must be CUDA (B, n_ctx, KV, D)")
        B, n_ctx, KV, D = k_cache.shape
        H = int(n_heads)
        if H % KV:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, f"n_heads {H} not a multiple of {KV}")
        self.B, self.H, self.KV, self.D, self.n_ctx = B, H, KV, D, n_ctx
        self.max_len = int(max_len or n_ctx)
        dev = k_cache.device
        self._kc, self._vc, self._ct, self._st = k_cache, v_cache, cos_tab, sin_tab
        self._style, self._scale = style, scale
        nq, nk = B * H * D, B * KV * D
        # pinned staging: [q | k | v] f32 and [positions | lengths] int32
        self._h_f = torch.zeros(nq + 2 * nk, dtype=torch.float32).pin_memory()
        self._h_i = torch.zeros(2 * B, dtype=torch.int32).pin_memory()
        self._h_out = torch.zeros((B, H, D), dtype=torch.float32).pin_memory()
        self._d_f = torch.zeros(nq + 2 * nk, dtype=torch.float32, device=dev)
        self._d_i = torch.zeros(2 * B, dtype=torch.int32, device=dev)
        self._out = torch.zeros((B, H, D), dtype=torch.float32, device=dev)
        self.q = self._h_f[:nq].view(B, H, D)
        self.k = self._h_f[nq:nq + nk].view(B, KV, D)
        self.v = self._h_f[nq + nk:].view(B, KV, D)
        self.positions = self._h_i[:B]
        self._pos_np = self._h_i[:B].numpy()   # numpy views of the pinned staging
        self._lens_np = self._h_i[B:].numpy()
        self._limit = min(n_ctx, self.max_len)
        self._split = device.decode_split_rows(B, KV, self.max_len, k_cache.dtype)
        self._ws = device.decode_workspace(B, H, D, self.max_len, self._split, dev)
        self._warm_up(dev, k_cache.dtype)
        self._stream = torch.cuda.Stream(device=dev)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=self._stream):
            self._body()

    # -- the captured body ---------------------------------------------------
    def _body(self):
        B, H, KV, D = self.B, self.H, self.KV, self.D
        nq, nk = B * H * D, B * KV * D
        self._d_f.copy_(self._h_f, non_blocking=True)
        self._d_i.copy_(self._h_i, non_blocking=True)
        q = self._d_f[:nq].view(B, H, D)
        k = self._d_f[nq:nq + nk].view(B, KV, D)
        v = self._d_f[nq + nk:].view(B, KV, D)
        device.rope_append(q, k, v, self._d_i[:B], self._ct, self._st, k_cache=self._kc,
                           v_cache=self._vc, style=self._style, per_sequence=True)
        device.decode(q, self._kc, self._vc, self._d_i[B:], scale=self._scale,
                      max_len=self.max_len, out=self._out, workspace=self._ws,
                      split_rows=self._split)
        self._h_out.copy_(self._out, non_blocking=True)

    def _warm_up(self, dev, dt):
        """Run each kernel once outside the capture, on private buffers."""
        H, KV, D = self.H, self.KV, self.D
        kc = torch.zeros((1, 1, KV, D), dtype=dt, device=dev)
        vc = torch.zeros_like(kc)
        q = torch.zeros((1, H, D), dtype=torch.float32, device=dev)
        kv = torch.zeros((1, KV, D), dtype=torch.float32, device=dev)
        p = torch.zeros(1, dtype=torch.int32, device=dev)
        device.rope_append(q, kv, kv, p, self._ct, self._st, k_cache=kc, v_cache=vc,
                           style=self._style, per_sequence=True)
        device.decode(q, kc, vc, p + 1, max_len=1)
        torch.cuda.synchronize(dev)
        _lib.raise_device_error()

    # -- per token ---------------------------------------------------------------
    def __call__(self, q=None, k=None, v=None, positions=None) -> torch.Tensor:
        """One step.  q (B, H, D), k/v (B, KV, D) f32 and positions (B,) int
        are copied into the pinned staging buffers when given (or written
        there directly through .q/.k/.v/.positions beforehand); sequence b's
        new row goes to cache row positions[b] and attention covers rows
        0..positions[b].  Returns the pinned (B, H, D) f32 output, valid
        until the next call."""
        for dst, src in ((self.q, q), (self.k, k), (self.v, v), (self.positions, positions)):
            if src is not None:
                dst.copy_(src if torch.is_tensor(src) else torch.as_tensor(np.asarray(src)))
        pos = self._pos_np
        if pos.min() < 0 or pos.max() >= self._limit:
            raise _lib.B2AError(_lib.ERR_POSITION, f"positions must lie in [0, {self._limit})")
        np.add(pos, 1, out=self._lens_np)
        self._graph.replay()   # on the caller's current stream
        torch.cuda.current_stream().synchronize()
        return self._h_out
