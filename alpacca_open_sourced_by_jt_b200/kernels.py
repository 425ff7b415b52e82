"""Drop-in for the attention/RoPE entry points of alpaccaroo/kernels.py.

Same names, arguments, shapes and dtypes as the reference's
`attention_decode` (kernels.py:1183-1200) and `rope_decode`
(kernels.py:1172-1180): host NumPy float32 in, fresh host NumPy float32 out.
Each call uploads its operands, runs the B200 kernel and downloads the
result; device-resident callers use `device.decode` / `device.rope_append`
directly and skip the copies.  There is no CPU fallback: a missing GPU or
library raises.
"""
from __future__ import annotations

import numpy as np
import torch

from . import device as _dev
from ._hostio import to_device, to_host


def attention_decode(q, K, V, group, inv_sqrt):
    """Single-token grouped-query attention over the KV cache.

    q f32 (n_head*head_dim,), K/V f32 (t, n_kv, head_dim); returns
    (n_head, head_dim) float32 = softmax(q.K^T * inv_sqrt).V with query
    head h reading KV head h // group (kernels.py:1183-1200).  Runs the
    fp32 split-KV kernel, so results match the NumPy path to ~1e-6.
    """
    K = np.asarray(K)
    V = np.asarray(V)
    if K.ndim != 3 or K.shape != V.shape:
        raise ValueError("K and V must both be (t, n_kv, head_dim)")
    t, n_kv, hd = K.shape
    if t == 0:
        raise ValueError("attention over an empty KV cache")
    n_head = n_kv * int(group)
    qd = to_device(np.ascontiguousarray(q, dtype=np.float32).reshape(1, n_head, hd))
    Kd = to_device(np.ascontiguousarray(K, dtype=np.float32))
    Vd = to_device(np.ascontiguousarray(V, dtype=np.float32))
    lens = torch.tensor([t], dtype=torch.int32, device=qd.device)
    out = _dev.decode(qd, Kd, Vd, lens, scale=float(inv_sqrt), max_len=t)
    return to_host(out).reshape(n_head, hd)


def rope_decode(v, cos_row, sin_row, n_heads, hd, n_rot, style):
    """Rotate one token's q or k vector: returns a fresh (n_heads*hd,)
    float32 array, bit-identical to the NumPy slicing path
    (kernels.py:1172-1180, model.py:1191-1209)."""
    vec = np.ascontiguousarray(v, dtype=np.float32).reshape(1, n_heads, hd)
    half = n_rot // 2
    cos = np.ascontiguousarray(cos_row, dtype=np.float32)[:half].reshape(1, half)
    sin = np.ascontiguousarray(sin_row, dtype=np.float32)[:half].reshape(1, half)
    vd = to_device(vec)
    pos = torch.zeros(1, dtype=torch.int32, device=vd.device)
    _dev.rope_append(vd, None, None, pos, to_device(cos), to_device(sin), n_rot=n_rot,
                     style=style)
    return to_host(vd).reshape(-1)
