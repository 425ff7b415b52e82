"""Qwen35 full-attention layer (between its projections) restated for the
checker - TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows alpaccaroo/qwen35_runtime.py:597-664 (Qwen35Model._attention): split
the per-head interleaved [query | gate] rows, per-head RMSNorm of q and k
(qwen35_ops.py:46-75: double precision relative to max(|x|, sqrt(eps)),
rounded to f32), IMROPE of q and k at lanes [p, p, p, 0]
(qwen35_ops.py:102-108, 159-215, rounded to f32), append k and v, one-token
GQA over the cache (qwen35_runtime.py:103-148, math.fsum), and the sigmoid
gate (tensor.py:123-129, rounded to f32).  Pure Python over small cases.
"""
from __future__ import annotations

import math

import numpy as np

from .attention import causal_gqa_step
from .rope import imrope_rotate


def qwen35_rms_norm(values, weight, epsilon: float):
    """qwen35_ops.py:46-75: x / sqrt(mean(x^2) + eps) * w, evaluated in
    double relative to a common scale; returns doubles."""
    vec = [float(v) for v in values]
    w = [float(v) for v in weight]
    root = math.sqrt(epsilon)
    scale = max(root, max(abs(v) for v in vec))
    msq = math.fsum((v / scale) * (v / scale) for v in vec) / len(vec)
    den = math.sqrt(msq + (root / scale) ** 2)
    return [((v / scale) / den) * lw for v, lw in zip(vec, w)]


def stable_sigmoid(x: float) -> float:
    """tensor.py:123-129."""
    if x >= 0.0:
        return 1.0 / (1.0 + math.exp(-x))
    z = math.exp(x)
    return z / (1.0 + z)


def qwen35_attention_layer(query_gate, key, value, q_norm, k_norm, epsilon, sections,
                           freq_base, position, k_prev, v_prev):
    """One token.  query_gate (H * 2D,), key/value (KV * D,), q_norm/k_norm (D,),
    k_prev/v_prev (L, KV, D) earlier cache rows, position = L (the new row).
    Returns f32 arrays: q (H, D) normed+rotated, k (KV, D) normed+rotated,
    pregate (H, D) attention output, gated (H, D)."""
    KV, D = k_prev.shape[1], k_prev.shape[2]
    H = len(query_gate) // (2 * D)
    f32 = np.float32
    qg = np.asarray(query_gate, f32).reshape(H, 2 * D)
    lanes = (position, position, position, 0)
    qs = [np.array(imrope_rotate(np.array(qwen35_rms_norm(qg[h, :D], q_norm, epsilon), f32),
                                 lanes, sections, freq_base), f32) for h in range(H)]
    kh = np.asarray(key, f32).reshape(KV, D)
    ks = [np.array(imrope_rotate(np.array(qwen35_rms_norm(kh[g], k_norm, epsilon), f32),
                                 lanes, sections, freq_base), f32) for g in range(KV)]
    kc = np.concatenate([np.asarray(k_prev, f32), np.stack(ks)[None]], axis=0)
    vc = np.concatenate([np.asarray(v_prev, f32), np.asarray(value, f32).reshape(1, KV, D)],
                        axis=0)
    att = np.array(causal_gqa_step(qs, kc, vc), f32)
    gated = np.array([[float(att[h, c]) * stable_sigmoid(float(qg[h, D + c]))
                       for c in range(D)] for h in range(H)], f32)
    return np.stack(qs), np.stack(ks), att, gated
