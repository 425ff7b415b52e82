"""Drop-in for the batched-attention entry point of alpaccaroo/cuda.py.

`attention_batch(q, K, V, positions, group, inv_sqrt, window=0, kv_start=0)`
keeps the reference's signature and contract (cuda.py:1186-1242): host
float32 q (t_q, n_head, hd), K/V (t_kv, n_kv, hd), int32 absolute
positions; returns (t_q, n_head*hd) float32, or None for a geometry the
kernel does not serve (the reference declines head_dim > 128 the same way
and its caller keeps the NumPy einsum).  The work runs on the tcgen05 flash
prefill kernel with 16-bit operands and fp32 accumulation: operands are
rounded to fp16 (bf16 when a value exceeds fp16's range), so results agree
with the fp32 NumPy path to ~1e-3, not bit-for-bit.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from . import device as _dev
from ._hostio import to_device, to_host

_FP16_MAX = 60000.0


def available() -> bool:
    """True when a CUDA device is visible and libb2attn.so loads."""
    try:
        _lib.load()
    except ImportError:
        return False
    return torch.cuda.is_available()


def status() -> str:
    if not available():
        return "b2attn unavailable (no CUDA device or library)"
    return (f"b2attn abi {_lib.load().b2a_version()} on "
            f"{torch.cuda.get_device_name(torch.cuda.current_device())}")


def _operand_dtype(*arrays) -> torch.dtype:
    big = max(float(np.abs(a).max()) if a.size else 0.0 for a in arrays)
    return torch.float16 if big < _FP16_MAX else torch.bfloat16


def attention_batch(q, K, V, positions, group: int, inv_sqrt: float, window: int = 0,
                    kv_start: int = 0):
    """Batched causal GQA for the prefill path (cuda.py:1186-1242)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    if q.ndim != 3 or K.ndim != 3 or K.shape != V.shape:
        return None
    t_q, n_head, hd = q.shape
    t_kv, n_kv, hd_k = K.shape
    if (hd != hd_k or hd not in (64, 128) or t_q == 0 or t_kv == 0 or group < 1
            or n_kv * group != n_head or pos.shape != (t_q,)):
        return None
    dt = _operand_dtype(q, K, V)
    qd = to_device(q).to(dt)
    Kd = to_device(K).to(dt)
    Vd = to_device(V).to(dt)
    pd = to_device(pos)
    out = _dev.prefill(qd, Kd, Vd, pd, scale=float(inv_sqrt), window=int(window),
                       kv_start=int(kv_start), out_dtype=torch.float32)
    return to_host(out).reshape(t_q, n_head * hd)
