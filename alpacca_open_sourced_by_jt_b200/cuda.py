"""Drop-in for the batched-attention entry point of alpaccaroo/cuda.py.

`attention_batch(q, K, V, positions, group, inv_sqrt, window=0, kv_start=0)`
keeps the reference's signature and contract (cuda.py:1186-1242): host
float32 q (t_q, n_head, hd), K/V (t_kv, n_kv, hd), int32 absolute
positions; returns (t_q, n_head*hd) float32, or None for a geometry the
kernels do not serve (the reference declines head_dim > 128 the same way and
its caller keeps the NumPy einsum).  Here every head_dim that is a multiple
of 4 up to 256 is served, so the gemma3 (256) and Qwen35 (256) geometries
the reference leaves on the CPU run on the GPU too.

The operands stay float32: the work runs on the fp32 flash prefill kernel
(b2a_prefill with F32 inputs: fp32 products and fp32 accumulation on the
CUDA cores), so results agree with the NumPy path to within fp32 rounding
(the tests hold them to 1e-4 normwise, and observe ~1e-6), for any input
magnitude.  16-bit callers with device-resident tensors use
`device.prefill`, which runs the tcgen05 tensor-core kernels.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from . import device as _dev
from ._hostio import to_device, to_host

MAX_HEAD_DIM = 256


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


def serves_head_dim(hd: int) -> bool:
    """Whether attention_batch serves this head_dim (fp32 kernel)."""
    return 0 < hd <= MAX_HEAD_DIM and hd % 4 == 0


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
    if (hd != hd_k or not serves_head_dim(hd) or t_q == 0 or t_kv == 0 or group < 1
            or n_kv * group != n_head or pos.shape != (t_q,)):
        return None
    qd = to_device(q)
    Kd = to_device(K)
    Vd = to_device(V)
    pd = to_device(pos)
    out = _dev.prefill(qd, Kd, Vd, pd, scale=float(inv_sqrt), window=int(window),
                       kv_start=int(kv_start), out_dtype=torch.float32)
    return to_host(out).reshape(t_q, n_head * hd)
