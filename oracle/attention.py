"""Attention restatements (test infrastructure only; see oracle/__init__.py).

NumPy float32 throughout where the reference uses NumPy float32, Python
floats (double) where the reference's semantic contract does.
"""
from __future__ import annotations

import math

import numpy as np


def attention_decode(q, K, V, group: int, inv_sqrt: float):
    """Single-token GQA over the cache: alpaccaroo/model.py:1231-1252 (the
    NumPy branch of Model._attention_np).

    q (n_head*hd,) or (n_head, hd) f32; K, V (t, n_kv, hd) f32.  Query head h
    reads KV head h // group.  Scores = q.K^T * inv_sqrt, max-subtracted,
    exponentiated, normalised by their sum, then applied to V; returns
    (n_head, hd) f32.
    """
    K = np.asarray(K, np.float32)
    V = np.asarray(V, np.float32)
    t, n_kv, hd = K.shape
    qg = np.asarray(q, np.float32).reshape(n_kv, group, hd)
    s = np.matmul(qg, K.transpose(1, 2, 0)) * np.float32(inv_sqrt)  # (n_kv, g, t)
    s = s - s.max(axis=2, keepdims=True)
    w = np.exp(s)
    w = w / w.sum(axis=2, keepdims=True)
    o = np.matmul(w, V.transpose(1, 0, 2))  # (n_kv, g, hd)
    return o.reshape(n_kv * group, hd).astype(np.float32)


def attention_batch(q, K, V, positions, group: int, inv_sqrt: float, window: int = 0,
                    kv_start: int = 0):
    """Causal batched GQA (prefill): alpaccaroo/model.py:1254-1272 and the
    window/kv_start variant model.py:1567-1592.

    q (t_q, n_head, hd); K, V (t_kv, n_kv, hd); positions int32 (t_q,).  Key
    s (absolute position kv_start+s) is allowed for query t iff
    kv_start+s <= positions[t] and, with window > 0, kv_start+s >
    positions[t]-window.  Disallowed scores are set to -1e30 before the
    softmax, exactly like the reference.  Returns (t_q, n_head*hd) f32.
    """
    q = np.asarray(q, np.float32)
    K = np.asarray(K, np.float32)
    V = np.asarray(V, np.float32)
    t_q = q.shape[0]
    t_kv, n_kv, hd = K.shape
    positions = np.asarray(positions, np.int32)
    qg = q.reshape(t_q, n_kv, group, hd)
    s = np.einsum("tkgh,skh->tkgs", qg, K, optimize=True) * np.float32(inv_sqrt)
    kv_pos = np.arange(kv_start, kv_start + t_kv, dtype=np.int32)
    allowed = kv_pos[None, :] <= positions[:, None]
    if window > 0:
        allowed &= kv_pos[None, :] > (positions[:, None] - window)
    s = np.where(allowed[:, None, None, :], s, np.float32(-1.0e30))
    s = s - s.max(axis=-1, keepdims=True)
    w = np.exp(s)
    w = w / w.sum(axis=-1, keepdims=True)
    o = np.einsum("tkgs,skh->tkgh", w, V, optimize=True)
    return o.reshape(t_q, n_kv * group * hd).astype(np.float32)


def attention_decode_varlen(q, k_cache, v_cache, lens, group: int, inv_sqrt: float):
    """Batched variable-length decode: the reference serves one sequence per
    Model, so the batch is a loop of attention_decode calls, sequence b over
    its own cache rows [:lens[b]] (alpaccaroo/model.py:1438-1440).

    q (B, H, D); k_cache/v_cache (B, n_ctx, KV, D); returns (B, H, D) f32.
    """
    out = np.empty(q.shape, np.float32)
    for b in range(q.shape[0]):
        L = int(lens[b])
        out[b] = attention_decode(q[b], k_cache[b, :L], v_cache[b, :L], group, inv_sqrt)
    return out


def split_decode_partials(q, K, V, group: int, inv_sqrt: float, split: int):
    """Per-chunk online-softmax partials (m, l, unnormalised acc) over
    `split`-row chunks of the context: alpaccaroo/cuda.py:580-672
    (_attention_decode_part).  Returns pm (H, n), pl (H, n), pacc (H, n, hd)
    in float64 for use as a reference."""
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    t, n_kv, hd = K.shape
    H = n_kv * group
    qh = np.asarray(q, np.float64).reshape(H, hd)
    n = (t + split - 1) // split
    pm = np.empty((H, n))
    pl = np.empty((H, n))
    pacc = np.empty((H, n, hd))
    for h in range(H):
        kv = h // group
        for c in range(n):
            rows = slice(c * split, min(t, (c + 1) * split))
            s = K[rows, kv] @ qh[h] * inv_sqrt
            m = s.max()
            p = np.exp(s - m)
            pm[h, c] = m
            pl[h, c] = p.sum()
            pacc[h, c] = p @ V[rows, kv]
    return pm, pl, pacc


def split_combine(pm, pl, pacc):
    """LSE merge of chunk partials: alpaccaroo/cuda.py:674-694
    (_attention_decode_combine): M = max_c m_c, L = sum_c l_c e^(m_c-M),
    out = sum_c acc_c e^(m_c-M) / L.  Returns (H, hd)."""
    M = pm.max(axis=1, keepdims=True)
    w = np.exp(pm - M)
    L = (pl * w).sum(axis=1, keepdims=True)
    return (pacc * w[:, :, None]).sum(axis=1) / L


def lse_combine(o_parts, lse_parts):
    """Merge normalised shard outputs by their log-sum-exp (the same algebra
    as split_combine with o = acc/l, lse = m + log l).  o_parts (G, R, D),
    lse_parts (G, R); returns (out (R, D), lse (R,)) in float64."""
    o_parts = np.asarray(o_parts, np.float64)
    lse_parts = np.asarray(lse_parts, np.float64)
    M = lse_parts.max(axis=0)
    Mref = np.where(np.isfinite(M), M, 0.0)
    w = np.exp(lse_parts - Mref)
    L = w.sum(axis=0)
    out = (w[:, :, None] * o_parts).sum(axis=0) / np.where(L > 0, L, 1.0)[:, None]
    lse = np.where(L > 0, Mref + np.log(np.where(L > 0, L, 1.0)), -np.inf)
    return out, lse


def qwen35_full_attention_decode(queries, keys, values):
    """Online-softmax decode of the Qwen35 runtime: the NumPy fallback of
    alpaccaroo/qwen35_kernels.py:363-392.  queries (H, Dk), keys (T, KV, Dk),
    values (T, KV, Dv); scale 1/sqrt(Dk); contiguous grouping."""
    queries = np.asarray(queries, np.float32)
    keys = np.asarray(keys, np.float32)
    values = np.asarray(values, np.float32)
    out = np.zeros((queries.shape[0], values.shape[2]), np.float32)
    group = queries.shape[0] // keys.shape[1]
    scale = 1.0 / math.sqrt(queries.shape[1])
    for h in range(queries.shape[0]):
        kv = h // group
        mx = -math.inf
        den = 0.0
        for p in range(keys.shape[0]):
            sc = float(queries[h] @ keys[p, kv]) * scale
            nm = max(mx, sc)
            old = math.exp(mx - nm)
            new = math.exp(sc - nm)
            out[h] = out[h] * old + values[p, kv] * new
            den = den * old + new
            mx = nm
        out[h] /= den
    return out


def qwen35_full_attention_prefill(queries, keys, values, prefix_length: int = 0):
    """alpaccaroo/qwen35_kernels.py:395-411: token t attends to keys
    [:prefix_length + t + 1].  Vectorised restatement (same math as calling
    qwen35_full_attention_decode per token)."""
    queries = np.asarray(queries, np.float32)
    T, H, D = queries.shape
    KV = keys.shape[1]
    pos = np.arange(prefix_length, prefix_length + T, dtype=np.int32)
    out = attention_batch(queries, keys[:prefix_length + T], values[:prefix_length + T], pos,
                          H // KV, 1.0 / math.sqrt(D))
    return out.reshape(T, H, -1)


def causal_gqa_step(query_heads, key_cache, value_cache, scale=None):
    """Pure-Python semantic GQA with math.fsum: alpaccaroo/qwen35_ops.py:406-472
    (validation subset).  Returns a list of lists (doubles)."""
    queries = [[float(x) for x in h] for h in query_heads]
    keys = [[[float(x) for x in h] for h in tok] for tok in key_cache]
    values = [[[float(x) for x in h] for h in tok] for tok in value_cache]
    if not queries or not keys or len(keys) != len(values):
        raise ValueError("GQA requires queries and equal nonempty K/V caches")
    kv_heads = len(keys[0])
    if kv_heads <= 0 or len(queries) % kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    dk = len(queries[0])
    if scale is None:
        scale = 1.0 / math.sqrt(dk)
    group = len(queries) // kv_heads
    dv = len(values[0][0])
    result = []
    for qi, qv in enumerate(queries):
        kv = qi // group
        scores = [math.fsum(a * b for a, b in zip(qv, tok[kv])) * scale for tok in keys]
        mx = max(scores)
        ex = [math.exp(s - mx) for s in scores]
        den = math.fsum(ex)
        pr = [e / den for e in ex]
        result.append([math.fsum(pr[t] * values[t][kv][c] for t in range(len(values)))
                       for c in range(dv)])
    return result
