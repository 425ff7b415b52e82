"""Seeded input cases shared by the golden generator and the tests.

Every case returns its arrays plus `sha256`, a digest of the input bytes, so
a test can check that it regenerated exactly the inputs the golden file was
made from.  Shapes follow the benchmark configurations (config 1 exactly; the
others at sizes a CPU finishes in seconds).
"""
from __future__ import annotations

import hashlib

import numpy as np

CONFIG1_SAMPLE_ROWS = (0, 1, 2, 63, 64, 255, 300, 510, 511)


def _digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def decode_config1():
    """benchmark config 1: batch 1, 32 query / 8 KV heads, head_dim 64,
    context 512, fp32, Q/K/V ~ N(0,1) seed 0, RoPE theta 500000 ("norm",
    llama) on K positions 0..511 and q at 511, scale 1/sqrt(64)."""
    H, KV, D, L = 32, 8, 64, 512
    rng = np.random.default_rng(0)
    q = rng.standard_normal((H, D), dtype=np.float32)
    k = rng.standard_normal((L, KV, D), dtype=np.float32)
    v = rng.standard_normal((L, KV, D), dtype=np.float32)
    return dict(H=H, KV=KV, D=D, L=L, base=500000.0, q_raw=q, k_raw=k, v=v,
                sha256=_digest(q, k, v))


def rope_neox():
    """Partial-rotary neox case: 4 q / 2 KV heads, head_dim 64, n_rot 32,
    base 10000, six tokens at scattered positions."""
    H, KV, D, n_rot, n_ctx = 4, 2, 64, 32, 256
    rng = np.random.default_rng(11)
    positions = np.array([0, 1, 5, 77, 128, 255], np.int32)
    q = rng.standard_normal((len(positions), H, D), dtype=np.float32)
    k = rng.standard_normal((len(positions), KV, D), dtype=np.float32)
    return dict(H=H, KV=KV, D=D, n_rot=n_rot, n_ctx=n_ctx, base=10000.0, positions=positions,
                q=q, k=k, sha256=_digest(q, k, positions))


def prefill_small():
    """Causal prefill chunk after a 13-token prefix: 37 queries at positions
    13..49 over 50 keys, 8 q / 2 KV heads, head_dim 64, fp32 N(0,1)."""
    H, KV, D, pre, t = 8, 2, 64, 13, 37
    rng = np.random.default_rng(21)
    q = rng.standard_normal((t, H, D), dtype=np.float32)
    k = rng.standard_normal((pre + t, KV, D), dtype=np.float32)
    v = rng.standard_normal((pre + t, KV, D), dtype=np.float32)
    positions = np.arange(pre, pre + t, dtype=np.int32)
    return dict(H=H, KV=KV, D=D, t_kv=pre + t, q=q, k=k, v=v, positions=positions,
                sha256=_digest(q, k, v, positions))


def prefill_window():
    """Sliding-window variant (gemma3 semantics): window 16, kv_start 5."""
    H, KV, D, t = 4, 2, 64, 40
    rng = np.random.default_rng(22)
    q = rng.standard_normal((t, H, D), dtype=np.float32)
    k = rng.standard_normal((45, KV, D), dtype=np.float32)
    v = rng.standard_normal((45, KV, D), dtype=np.float32)
    positions = np.arange(10, 10 + t, dtype=np.int32)
    return dict(H=H, KV=KV, D=D, window=16, kv_start=5, q=q, k=k, v=v, positions=positions,
                sha256=_digest(q, k, v, positions))


def prefill_qwen35_d256():
    """Qwen35 full-attention prefill at its key_length 256: 12 tokens after a
    13-token prefix, 4 q / 2 KV heads, fp32 N(0,1)."""
    rng = np.random.default_rng(41)
    q = rng.standard_normal((12, 4, 256), dtype=np.float32)
    k = rng.standard_normal((25, 2, 256), dtype=np.float32)
    v = rng.standard_normal((25, 2, 256), dtype=np.float32)
    return dict(q=q, k=k, v=v, prefix=13, sha256=_digest(q, k, v))


def prefill_gemma3_window_d256():
    """gemma3-style sliding-window prefill at head_dim 256 (the geometry the
    reference's GPU tier declines): 4 q / 1 KV head, window 24, kv_start 7,
    24 queries at positions 40..63 over the 57 cached rows 7..63."""
    H, KV, D, t = 4, 1, 256, 24
    rng = np.random.default_rng(42)
    q = rng.standard_normal((t, H, D), dtype=np.float32)
    k = rng.standard_normal((57, KV, D), dtype=np.float32)
    v = rng.standard_normal((57, KV, D), dtype=np.float32)
    positions = np.arange(40, 40 + t, dtype=np.int32)
    return dict(H=H, KV=KV, D=D, window=24, kv_start=7, q=q, k=k, v=v, positions=positions,
                sha256=_digest(q, k, v, positions))


def prefill_empty_rows():
    """Rows with no visible key: kv_start 20 with queries at positions
    10..29, so rows 0..9 precede every cached key (the NumPy path gives them
    the mean of all value rows), plus a window of 4.  4 q / 2 KV heads, 64."""
    H, KV, D, t = 4, 2, 64, 20
    rng = np.random.default_rng(43)
    q = rng.standard_normal((t, H, D), dtype=np.float32)
    k = rng.standard_normal((10, KV, D), dtype=np.float32)
    v = rng.standard_normal((10, KV, D), dtype=np.float32)
    positions = np.arange(10, 10 + t, dtype=np.int32)
    return dict(H=H, KV=KV, D=D, window=4, kv_start=20, q=q, k=k, v=v, positions=positions,
                sha256=_digest(q, k, v, positions))


def prefill_large_magnitude():
    """fp32 values far outside fp16's range: q ~ N(0, 30^2) (peaked softmax
    rows), K ~ N(0,1), V ~ N(0, 1e5^2); causal over 40 keys with a 24-row
    prefix, 4 q / 2 KV heads, head_dim 128."""
    rng = np.random.default_rng(44)
    q = (30.0 * rng.standard_normal((16, 4, 128))).astype(np.float32)
    k = rng.standard_normal((40, 2, 128), dtype=np.float32)
    v = (1e5 * rng.standard_normal((40, 2, 128))).astype(np.float32)
    positions = np.arange(24, 40, dtype=np.int32)
    return dict(H=4, KV=2, D=128, q=q, k=k, v=v, positions=positions,
                sha256=_digest(q, k, v, positions))


def qwen35_decode():
    """Qwen35 full-attention decode: 8 q / 2 KV heads, head_dim 64, 40 keys."""
    rng = np.random.default_rng(31)
    q = rng.standard_normal((8, 64), dtype=np.float32)
    k = rng.standard_normal((40, 2, 64), dtype=np.float32)
    v = rng.standard_normal((40, 2, 64), dtype=np.float32)
    return dict(q=q, k=k, v=v, sha256=_digest(q, k, v))


def qwen35_prefill():
    """Qwen35 prefill: 9 tokens after a 6-token prefix, 4 q / 2 KV heads, 64."""
    rng = np.random.default_rng(32)
    q = rng.standard_normal((9, 4, 64), dtype=np.float32)
    k = rng.standard_normal((15, 2, 64), dtype=np.float32)
    v = rng.standard_normal((15, 2, 64), dtype=np.float32)
    return dict(q=q, k=k, v=v, prefix=6, sha256=_digest(q, k, v))


def imrope_case():
    """IMROPE on 3 tokens x 3 heads of head_dim 128 with sections
    (11, 11, 10, 0) (64 rotary dims, 64 pass-through), base 1e7; text
    positions [p, p, p, 0] and one multimodal lane set."""
    rng = np.random.default_rng(33)
    x = rng.standard_normal((3, 3, 128), dtype=np.float32)
    lanes = np.array([[0, 0, 0, 0], [17, 17, 17, 0], [5, 9, 3, 0]], np.int32)
    return dict(x=x, lanes=lanes, sections=(11, 11, 10, 0), base=10000000.0,
                sha256=_digest(x, lanes))


def gqa_step_case():
    """qwen35_ops.causal_gqa_step: 4 q / 2 KV heads, dim 16, 7 keys."""
    rng = np.random.default_rng(34)
    q = rng.standard_normal((4, 16))
    k = rng.standard_normal((7, 2, 16))
    v = rng.standard_normal((7, 2, 16))
    return dict(q=q, k=k, v=v, sha256=_digest(q, k, v))


def kv_state_case():
    """One attention layer's state: 37 appended K/V rows, 2 KV heads, key
    and value dim 16, f32 N(0,1); truncated to 20 rows afterwards."""
    rng = np.random.default_rng(21)
    L, KV, D = 37, 2, 16
    k = rng.standard_normal((L, KV, D), dtype=np.float32)
    v = rng.standard_normal((L, KV, D), dtype=np.float32)
    return dict(layer_index=3, L=L, KV=KV, D=D, truncate=20, k=k, v=v, sha256=_digest(k, v))


def qwen35_layer_case():
    """The device half of one Qwen35 full-attention layer for one token:
    4 query / 2 KV heads, key = value length 64, IMROPE sections (8, 8, 8, 0)
    (48 rotated dims of 64), base 1e7, RMS epsilon 1e-6; 40 earlier rows
    in the cache, the new token at position 40.  Inputs are the projected
    query|gate rows, key and value rows and the q/k norm weights."""
    rng = np.random.default_rng(33)
    H, KV, D, L = 4, 2, 64, 40
    qg = rng.standard_normal(H * 2 * D, dtype=np.float32)
    k = rng.standard_normal(KV * D, dtype=np.float32)
    v = rng.standard_normal(KV * D, dtype=np.float32)
    qn = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    k_prev = rng.standard_normal((L, KV, D), dtype=np.float32)
    v_prev = rng.standard_normal((L, KV, D), dtype=np.float32)
    return dict(H=H, KV=KV, D=D, L=L, sections=(8, 8, 8, 0), base=1e7, eps=1e-6,
                query_gate=qg, key=k, value=v, q_norm=qn, k_norm=kn, k_prev=k_prev,
                v_prev=v_prev, sha256=_digest(qg, k, v, qn, kn, k_prev, v_prev))


def llama_q8_case():
    """A small llama-architecture model with Q8_0 weights N(0, 0.02) (seed 5),
    quantized by the reference's Q8_0 rule (oracle.llama_q8.quantize_q8_0):
    2 layers, hidden 256, 4 q / 2 KV heads of 64, FFN 512, vocab 1024,
    RMSNorm eps 1e-5, RoPE base 5e5 (norm style); six decode tokens."""
    from oracle.llama_q8 import quantize_q8_0
    rng = np.random.default_rng(5)
    E, H, KV, D, F, V = 256, 4, 2, 64, 512, 1024

    def mat(rows, cols):
        return quantize_q8_0(rng.normal(0.0, 0.02, (rows, cols)).astype(np.float32))

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    layers = []
    for _ in range(2):
        layers.append(dict(attn_norm=norm(E), wq=mat(H * D, E), wk=mat(KV * D, E),
                           wv=mat(KV * D, E), wo=mat(E, H * D), ffn_norm=norm(E),
                           w_gate=mat(F, E), w_up=mat(F, E), w_down=mat(E, F)))
    tok_embd = mat(V, E)
    out_norm = norm(E)
    output = mat(V, E)
    blobs = [tok_embd, output, out_norm.tobytes()] + [
        (ly[k] if isinstance(ly[k], bytes) else ly[k].tobytes())
        for ly in layers for k in sorted(ly)]
    import hashlib
    h = hashlib.sha256()
    for b in blobs:
        h.update(b)
    return dict(n_layer=2, n_embd=E, n_head=H, n_kv=KV, head_dim=D, n_ff=F, n_vocab=V,
                rms_eps=1e-5, rope_base=500000.0, n_ctx=32, layers=layers,
                tok_embd=tok_embd, out_norm=out_norm, output=output,
                tokens=[1, 5, 17, 300, 1023, 42], sha256=h.hexdigest())

