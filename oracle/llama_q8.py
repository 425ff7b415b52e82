"""Q8_0 weights and the llama decode step restated for the checker - TEST
INFRASTRUCTURE ONLY (see oracle/__init__.py).

* quantize_q8_0: alpaccaroo/quants.py:898-909 in NumPy.  Per 32 values:
  d = amax / 127 (double), codes = round-half-even(v / d) clamped to
  [-128, 127], stored as one little-endian f16 d then 32 int8 codes.
* q8_0_matvec: alpaccaroo/qmatrix.py:312-320: per 32-block dot of the codes
  with x in f32, times the block's d, summed over blocks.
* forward_token: Model._forward_np for a llama-architecture model
  (alpaccaroo/model.py:1374-1487): RMSNorm (tensor.py:349-356), q/k/v
  matvecs, RoPE (model.py:1162-1209), cache store, GQA attention
  (model.py:1231-1252), output projection + residual, RMSNorm, SwiGLU,
  down projection + residual; final RMSNorm and the output matvec.
"""
from __future__ import annotations

import math

import numpy as np

from .attention import attention_decode
from .rope import rope_vec


def quantize_q8_0(values: np.ndarray) -> bytes:
    """The reference's Q8_0 encoder (quants.py:898-909) for a flat array."""
    v = np.asarray(values, dtype=np.float64).reshape(-1, 32)
    amax = np.abs(v).max(axis=1)
    d = amax / 127.0
    inv = np.where(d != 0.0, 1.0 / np.where(d != 0.0, d, 1.0), 0.0)
    q = np.clip(np.rint(v * inv[:, None]), -128, 127).astype(np.int8)
    rec = np.empty(len(v), dtype=[("d", "<f2"), ("qs", "i1", 32)])
    rec["d"] = d.astype(np.float16)
    rec["qs"] = q
    return rec.tobytes()


def q8_0_unpack(data: bytes, rows: int, cols: int):
    """Q8_0 records -> (codes int8 (rows, cols), scales f32 (rows, cols/32))."""
    rec = np.frombuffer(data, dtype=[("d", "<f2"), ("qs", "i1", 32)])
    codes = rec["qs"].reshape(rows, cols)
    scales = rec["d"].astype(np.float32).reshape(rows, cols // 32)
    return codes, scales


def q8_0_matvec(data: bytes, rows: int, cols: int, x) -> np.ndarray:
    """qmatrix.py:312-320: blockdot (rows, n_blocks) in f32, times d, summed."""
    codes, d = q8_0_unpack(data, rows, cols)
    xs = np.asarray(x, dtype=np.float32).reshape(cols // 32, 32)
    blockdot = np.einsum("rsl,sl->rs", codes.reshape(rows, cols // 32, 32).astype(np.float32), xs)
    return np.einsum("rs,rs->r", blockdot, d).astype(np.float32)


def q8_0_row(data: bytes, rows: int, cols: int, r: int) -> np.ndarray:
    """One dequantized row (qmatrix.py:445-447): codes x d per block."""
    codes, d = q8_0_unpack(data, rows, cols)
    return (codes[r].reshape(-1, 32).astype(np.float32) * d[r][:, None]).reshape(-1)


def rmsnorm(x, w, eps: float) -> np.ndarray:
    """tensor.py:349-356 (1-D): x * (1 / sqrt(x.x / n + eps)) * w."""
    x = np.asarray(x, dtype=np.float32)
    inv = 1.0 / math.sqrt(float(x @ x) / x.shape[0] + eps)
    return x * np.float32(inv) * w


def forward_token(model: dict, token: int, pos: int, cache_k, cache_v, cos, sin) -> np.ndarray:
    """One llama decode token (model.py:1374-1487).  model: dict of hp values
    and weights ('layers': per-layer dicts of Q8_0 bytes and f32 norms);
    cache_k/cache_v: per-layer (n_ctx, KV, D) f32 arrays, updated in place."""
    E, H, KV, D, F = model["n_embd"], model["n_head"], model["n_kv"], model["head_dim"], \
        model["n_ff"]
    eps = model["rms_eps"]
    x = q8_0_row(model["tok_embd"], model["n_vocab"], E, token)
    for li, ly in enumerate(model["layers"]):
        h = rmsnorm(x, ly["attn_norm"], eps)
        q = q8_0_matvec(ly["wq"], H * D, E, h)
        k = q8_0_matvec(ly["wk"], KV * D, E, h)
        v = q8_0_matvec(ly["wv"], KV * D, E, h)
        q = rope_vec(q, H, pos, cos, sin, D, D, "norm").reshape(H, D)
        k = rope_vec(k, KV, pos, cos, sin, D, D, "norm").reshape(KV, D)
        cache_k[li][pos] = k
        cache_v[li][pos] = v.reshape(KV, D)
        att = attention_decode(q, cache_k[li][:pos + 1], cache_v[li][:pos + 1], H // KV,
                               1.0 / math.sqrt(D))
        x = x + q8_0_matvec(ly["wo"], E, H * D, att.reshape(-1))
        h = rmsnorm(x, ly["ffn_norm"], eps)
        gate = q8_0_matvec(ly["w_gate"], F, E, h)
        up = q8_0_matvec(ly["w_up"], F, E, h)
        act = gate / (np.float32(1.0) + np.exp(-gate)) * up
        x = x + q8_0_matvec(ly["w_down"], E, F, act)
    h = rmsnorm(x, model["out_norm"], eps)
    return q8_0_matvec(model["output"], model["n_vocab"], E, h)
