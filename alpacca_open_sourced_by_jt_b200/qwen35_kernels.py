"""Drop-in for the Qwen35 full-attention entry points of
alpaccaroo/qwen35_kernels.py (:363-411).

`qwen35_full_attention_decode(queries, keys, values)`: queries (H, Dk),
keys (T, KV, Dk), values (T, KV, Dv) -> (H, Dv) float32, scale 1/sqrt(Dk),
contiguous grouping; runs the fp32 split-KV kernel.
`qwen35_full_attention_prefill(queries, keys, values, prefix_length=0)`:
queries (T, H, Dk); token t sees keys [:prefix_length + t + 1]; runs the
fp32 flash prefill kernel (fp32 operands and accumulation, any head_dim that
is a multiple of 4 up to 256, Qwen35's key_length 256 included).
Both need Dk == Dv (the kernels share one head_dim).
"""
from __future__ import annotations

import math

import numpy as np

from . import cuda as _cuda
from . import kernels as _kernels


def qwen35_full_attention_decode(queries, keys, values):
    queries = np.asarray(queries, np.float32)
    keys = np.asarray(keys, np.float32)
    values = np.asarray(values, np.float32)
    if queries.ndim != 2 or keys.ndim != 3 or values.ndim != 3:
        raise ValueError("queries (H, D), keys/values (T, KV, D)")
    if keys.shape[2] != values.shape[2]:
        raise ValueError("the B200 decode kernel needs key_dim == value_dim")
    H, D = queries.shape
    KV = keys.shape[1]
    if H % KV:
        raise ValueError("query heads must be a multiple of KV heads")
    return _kernels.attention_decode(queries.reshape(-1), keys, values, H // KV,
                                     1.0 / math.sqrt(D))


def qwen35_full_attention_prefill(queries, keys, values, prefix_length: int = 0):
    queries = np.asarray(queries, np.float32)
    keys = np.asarray(keys, np.float32)
    values = np.asarray(values, np.float32)
    if queries.ndim != 3 or keys.ndim != 3 or values.ndim != 3:
        raise ValueError("queries (T, H, D), keys/values (T_kv, KV, D)")
    if keys.shape[2] != values.shape[2]:
        raise ValueError("the B200 prefill kernels need key_dim == value_dim")
    T, H, D = queries.shape
    KV = keys.shape[1]
    if H % KV:
        raise ValueError("query heads must be a multiple of KV heads")
    n = prefix_length + T
    if n > keys.shape[0]:
        raise ValueError(f"prefix_length + T = {n} exceeds the {keys.shape[0]} cached keys")
    pos = np.arange(prefix_length, n, dtype=np.int32)
    out = _cuda.attention_batch(queries, keys[:n], values[:n], pos, H // KV, 1.0 / math.sqrt(D))
    if out is None:
        raise ValueError(f"prefill kernel does not serve head_dim {D} "
                         "(a multiple of 4 up to 256)")
    return out.reshape(T, H, D)
