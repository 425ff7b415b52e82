"""The device half of a Qwen35 full-attention layer, for a batch of
sequences decoding one token each.

Between the layer's projections and its output projection the reference
runs (alpaccaroo/qwen35_runtime.py:597-664; device graph
qwen35_cuda_graph.py:781-851): split each head's interleaved
[query | gate] row, per-head RMSNorm of q and k, IMROPE at lanes [p,p,p,0],
append k and v to the cache, one-token GQA over the cache, and
out = attended * sigmoid(gate).  Here that is three launches:

  b2a_qwen35_attn_prep  split + RMSNorm + IMROPE + append (one CTA per head)
  b2a_decode            split-KV GQA decode over positions + 1 rows
  b2a_sigmoid_gate      the output gate, reading the gates in place

All buffers are preallocated, so a step can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib, device


class Qwen35AttentionLayer:
    """One full-attention layer's device state and step.

    query_norm/key_norm: the layer's (head_dim,) RMSNorm weights.  The cache
    is (batch, n_ctx, kv_heads, head_dim) of kv_dtype, one sequence per row
    (key_length == value_length, as the reference's GQA path requires,
    qwen35_runtime.py:115-116)."""

    def __init__(self, *, query_heads: int, kv_heads: int, head_dim: int, rms_epsilon: float,
                 rope_freq_base: float, sections, query_norm, key_norm, n_ctx: int,
                 batch: int = 1, kv_dtype: torch.dtype = torch.bfloat16, device_=None):
        _lib.load()
        H, KV, D = int(query_heads), int(kv_heads), int(head_dim)
        if KV <= 0 or H % KV:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, f"{H} query heads over {KV} KV heads")
        self.H, self.KV, self.D, self.B, self.n_ctx = H, KV, D, int(batch), int(n_ctx)
        self.eps, self.base = float(rms_epsilon), float(rope_freq_base)
        self.sections = (ctypes.c_int * 4)(*[int(x) for x in sections])
        dev = torch.device(device_) if device_ is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.device = dev
        self.q_norm = torch.as_tensor(query_norm, dtype=torch.float32).to(dev).contiguous()
        self.k_norm = torch.as_tensor(key_norm, dtype=torch.float32).to(dev).contiguous()
        if self.q_norm.numel() != D or self.k_norm.numel() != D:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, "norm weights must have head_dim values")
        self.k_cache = torch.zeros((self.B, self.n_ctx, KV, D), dtype=kv_dtype, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.q = torch.zeros((self.B, H, D), dtype=torch.float32, device=dev)
        self.attended = torch.zeros_like(self.q)
        self.out = torch.zeros_like(self.q)
        self.lanes = torch.zeros((self.B, 4), dtype=torch.int32, device=dev)
        self.lens = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self._split = device.decode_split_rows(self.B, KV, self.n_ctx, kv_dtype)
        self._ws = device.decode_workspace(self.B, H, D, self.n_ctx, self._split, dev)
        self.scale = 1.0 / math.sqrt(D)

    def step(self, query_gate: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
             positions: torch.Tensor, stream=None) -> torch.Tensor:
        """One token per sequence.  query_gate (B, H*2*D), key/value (B, KV*D)
        f32 CUDA rows as the projections produce them; positions (B,) int32
        cache rows (text lanes [p,p,p,0]).  Returns self.out, (B, H, D) f32:
        the gated attention output, the input of the output projection."""
        B, H, KV, D = self.B, self.H, self.KV, self.D
        for name, t, n in (("query_gate", query_gate, H * 2 * D), ("key", key, KV * D),
                           ("value", value, KV * D)):
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                    and t.numel() == B * n):
                raise _lib.B2AShapeError(_lib.ERR_SHAPE, f"{name} must be CUDA f32 ({B}, {n})")
        if not (positions.is_cuda and positions.dtype == torch.int32 and positions.numel() == B):
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, "positions must be CUDA int32 (B,)")
        st = device._stream(stream)
        self.lanes[:, :3] = positions.view(B, 1)
        torch.add(positions, 1, out=self.lens)
        lib = _lib.load()
        _lib.check(lib.b2a_qwen35_attn_prep(
            query_gate.data_ptr(), H * 2 * D, key.data_ptr(), KV * D, value.data_ptr(), KV * D,
            self.q_norm.data_ptr(), self.k_norm.data_ptr(), self.eps, self.lanes.data_ptr(),
            self.sections, self.base, 1.0, positions.data_ptr(), 1, self.k_cache.data_ptr(),
            self.v_cache.data_ptr(), self.k_cache.stride(0), self.n_ctx,
            device._code(self.k_cache.dtype), self.q.data_ptr(), _lib.F32, B, H, KV, D, st))
        device.decode(self.q, self.k_cache, self.v_cache, self.lens, scale=self.scale,
                      max_len=self.n_ctx, out=self.attended, workspace=self._ws,
                      split_rows=self._split, stream=stream)
        _lib.check(lib.b2a_sigmoid_gate(
            self.attended.data_ptr(), D, query_gate.data_ptr() + 4 * D, 2 * D,
            self.out.data_ptr(), D, B * H, D, st))
        return self.out
