"""RoPE + KV-append restatements (test infrastructure only; see
oracle/__init__.py)."""
from __future__ import annotations

import math

import numpy as np


def rope_inv_freq(n_rot: int, rope_base: float, freq_scale: float = 1.0):
    """alpaccaroo/model.py:318-323: inv_freq = freq_scale *
    base^(-2i/n_rot), i = 0..n_rot/2-1, with the exponent evaluated on a
    float32 arange (so the array is float32)."""
    half = n_rot // 2
    return (freq_scale * rope_base ** (-2.0 * np.arange(half, dtype=np.float32) / n_rot))


def rope_tables(n_ctx: int, n_rot: int, rope_base: float, freq_scale: float = 1.0):
    """alpaccaroo/model.py:871-875: theta = float32 positions x inv_freq,
    cos/sin tables (n_ctx, n_rot/2) float32."""
    inv = rope_inv_freq(n_rot, rope_base, freq_scale)
    theta = np.arange(n_ctx, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(theta), np.sin(theta)


def _rotate(v, c, s, n_rot: int, style: str):
    half = n_rot // 2
    if style == "norm":
        x0 = v[..., 0:n_rot:2].copy()
        x1 = v[..., 1:n_rot:2].copy()
        v[..., 0:n_rot:2] = x0 * c - x1 * s
        v[..., 1:n_rot:2] = x0 * s + x1 * c
    else:
        x0 = v[..., :half].copy()
        x1 = v[..., half:n_rot].copy()
        v[..., :half] = x0 * c - x1 * s
        v[..., half:n_rot] = x0 * s + x1 * c
    return v


def rope_vec(vec, n_heads: int, pos: int, cos_tab, sin_tab, head_dim: int, n_rot: int,
             style: str):
    """Rotate one token's q or k vector: alpaccaroo/model.py:1191-1209
    (Model._rope_np, NumPy branch).  "norm" rotates adjacent pairs
    (2i, 2i+1), "neox" split halves (i, i+n_rot/2); dims >= n_rot pass
    through.  Elementwise f32 products and sums, no fused multiply-add."""
    v = np.asarray(vec, np.float32).reshape(n_heads, head_dim).copy()
    _rotate(v, cos_tab[pos], sin_tab[pos], n_rot, style)
    return v.reshape(-1)


def rope_batch(vecs, n_heads: int, positions, cos_tab, sin_tab, head_dim: int, n_rot: int,
               style: str):
    """alpaccaroo/model.py:1191-1209 (_rope_batch_np): rope_vec over a batch
    of tokens at their own positions.  Returns (n, n_heads*head_dim)."""
    vecs = np.asarray(vecs, np.float32)
    v = vecs.reshape(len(vecs), n_heads, head_dim).copy()
    positions = np.asarray(positions)
    _rotate(v, cos_tab[positions][:, None, :], sin_tab[positions][:, None, :], n_rot, style)
    return v.reshape(len(vecs), -1)


def rope_append(q, k, v, positions, k_cache, v_cache, cos_tab, sin_tab, n_rot: int,
                style: str, bq=None, bk=None, bv=None, seq_of_token=None):
    """The decode/prefill qkv stage: bias add, rope of q and k, and the k/v
    rows written at their absolute positions (alpaccaroo/model.py:1418-1432
    for one token, 1327-1337 for a batch; device kernels cuda.py:723-786,
    885-953).

    q (n, H, D), k (n, KV, D), v (n, KV, D) f32; k_cache/v_cache
    (S, n_ctx, KV, D) arrays updated in place (any dtype: rows are cast on
    store); seq_of_token[i] picks the sequence (default 0).  Returns the
    rotated q (n, H, D) f32."""
    q = np.asarray(q, np.float32).copy()
    k = np.asarray(k, np.float32).copy()
    v = np.asarray(v, np.float32).copy()
    n, H, D = q.shape
    KV = k.shape[1]
    if bq is not None:
        q = q + np.asarray(bq, np.float32).reshape(1, H, D)
    if bk is not None:
        k = k + np.asarray(bk, np.float32).reshape(1, KV, D)
    if bv is not None:
        v = v + np.asarray(bv, np.float32).reshape(1, KV, D)
    qr = rope_batch(q.reshape(n, -1), H, positions, cos_tab, sin_tab, D, n_rot, style)
    kr = rope_batch(k.reshape(n, -1), KV, positions, cos_tab, sin_tab, D, n_rot, style)
    for i in range(n):
        s = 0 if seq_of_token is None else int(seq_of_token[i])
        p = int(positions[i])
        k_cache[s, p] = kr[i].reshape(KV, D)
        v_cache[s, p] = v[i]
    return qr.reshape(n, H, D)


def imrope_lane_for_pair(pair_index: int, sections) -> int:
    """Interleaved T/H/W/E lane schedule: alpaccaroo/qwen35_ops.py:138-156."""
    sec = tuple(sections)
    sector = pair_index % sum(sec)
    if sector % 3 == 1 and sector < 3 * sec[1]:
        return 1
    if sector % 3 == 2 and sector < 3 * sec[2]:
        return 2
    if sector % 3 == 0 and sector < 3 * sec[0]:
        return 0
    return 3


def imrope_rotate(values, position_lanes, sections, frequency_base: float,
                  frequency_scale: float = 1.0):
    """One head with Qwen IMROPE: alpaccaroo/qwen35_ops.py:159-215.  Pairs
    (j, j+P), P = sum(sections); theta = lanes[lane(j)] * scale *
    base^(-2j/(2P)) in double precision; trailing dims copied."""
    vec = [float(x) for x in values]
    P = sum(sections)
    dims = 2 * P
    res = list(vec)
    for j in range(P):
        lane = imrope_lane_for_pair(j, sections)
        theta = position_lanes[lane] * frequency_scale * frequency_base ** (-2.0 * j / dims)
        c, s = math.cos(theta), math.sin(theta)
        a, b = vec[j], vec[j + P]
        res[j] = a * c - b * s
        res[j + P] = a * s + b * c
    return res


def imrope_append(q, k, v, lanes, positions, k_cache, v_cache, sections, frequency_base,
                  frequency_scale=1.0, seq_of_token=None):
    """IMROPE for q/k heads plus the k/v rows stored at `positions`
    (alpaccaroo/qwen35_cuda_graph.py:813-827 composition of imrope and
    kv_append).  q (n,H,D), k/v (n,KV,D); lanes (n,4).  Returns f32 q."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    n, H, D = q.shape
    KV = k.shape[1]
    qo = np.empty_like(q)
    for i in range(n):
        ln = [int(x) for x in lanes[i]]
        for h in range(H):
            qo[i, h] = np.asarray(imrope_rotate(q[i, h], ln, sections, frequency_base,
                                                frequency_scale), np.float32)
        s = 0 if seq_of_token is None else int(seq_of_token[i])
        p = int(positions[i])
        for h in range(KV):
            k_cache[s, p, h] = np.asarray(imrope_rotate(k[i, h], ln, sections, frequency_base,
                                                        frequency_scale), np.float32)
        v_cache[s, p] = v[i]
    return qo
