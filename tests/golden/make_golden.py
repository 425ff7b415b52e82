"""Generate golden vectors by running the REFERENCE (alpaccaroo) itself.

Run where the reference is checked out, naming the directory that holds the
alpaccaroo package:

    ALPACCAROO_REF=<checkout> python tests/golden/make_golden.py

Inputs are regenerated from their seeds by tests/golden/cases.py (NumPy's
PCG64 default_rng is stable across versions); each .npz stores the
reference's outputs plus a SHA-256 of the input bytes, so a test can prove
it rebuilt exactly the inputs the reference saw.  The reference runs its
pure NumPy path here (its Numba kernels are disabled because the installed
numba differs from its pin), which is the path the oracle restates.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases  # noqa: E402

REF = os.environ.get("ALPACCAROO_REF")  # the alpaccaroo source checkout


def _import_reference():
    if not REF:
        sys.exit("set ALPACCAROO_REF to the alpaccaroo source checkout (the directory "
                 "holding the alpaccaroo package)")
    sys.path.insert(0, REF)
    from alpaccaroo import model, qwen35_kernels, qwen35_ops  # noqa: WPS433
    return model, qwen35_kernels, qwen35_ops


def _llama_model(model_mod, n_ctx, n_head, n_kv, head_dim, n_rot, base, style):
    hp = model_mod.Hyperparams(
        arch="llama", n_layer=1, n_embd=n_head * head_dim, n_head=n_head, n_kv=n_kv,
        n_ff=4 * n_head * head_dim, n_vocab=32, n_ctx_train=max(n_ctx, 4096),
        head_dim=head_dim, n_rot=n_rot, rms_eps=1e-5, rope_base=base, rope_style=style)
    m = model_mod.Model(hp, None)
    m.n_ctx = n_ctx
    m._init_cache()
    return m


def make_decode_config1(model_mod):
    c = cases.decode_config1()
    m = _llama_model(model_mod, c["L"], c["H"], c["KV"], c["D"], c["D"], c["base"], "norm")
    K = np.empty_like(c["k_raw"])
    for p in range(c["L"]):
        K[p] = m._rope_np(c["k_raw"][p].reshape(-1), c["KV"], p).reshape(c["KV"], c["D"])
    q = m._rope_np(c["q_raw"].reshape(-1), c["H"], c["L"] - 1)
    out = m._attention_np(q, K, c["v"], c["H"] // c["KV"], 1.0 / np.sqrt(c["D"]))
    rows = np.array(cases.CONFIG1_SAMPLE_ROWS)
    np.savez_compressed(
        os.path.join(HERE, "decode_config1.npz"), input_sha256=c["sha256"], q_rot=q,
        k_rot_rows=K[rows], sample_rows=rows, out=out, cos_tab=m._rope_cos[rows],
        sin_tab=m._rope_sin[rows])


def make_rope_neox(model_mod):
    c = cases.rope_neox()
    m = _llama_model(model_mod, c["n_ctx"], c["H"], c["KV"], c["D"], c["n_rot"], c["base"], "neox")
    single = np.stack([m._rope_np(c["q"][i].reshape(-1), c["H"], int(p))
                       for i, p in enumerate(c["positions"])])
    batch = m._rope_batch_np(c["k"].reshape(len(c["positions"]), -1), c["KV"], c["positions"])
    np.savez_compressed(os.path.join(HERE, "rope_neox.npz"), input_sha256=c["sha256"],
                        q_rot=single, k_rot=batch, cos_tab=m._rope_cos, sin_tab=m._rope_sin)


def make_prefill(model_mod):
    c = cases.prefill_small()
    m = _llama_model(model_mod, c["t_kv"], c["H"], c["KV"], c["D"], c["D"], 10000.0, "norm")
    out = m._attention_batch_np(c["q"], c["k"], c["v"], c["positions"], c["H"] // c["KV"],
                                1.0 / np.sqrt(c["D"]))
    w = cases.prefill_window()
    m = _llama_model(model_mod, 64, w["H"], w["KV"], w["D"], w["D"], 10000.0, "norm")
    outw = m._attention_batch_window_np(w["q"], w["k"], w["v"], w["positions"],
                                        w["H"] // w["KV"], 1.0 / np.sqrt(w["D"]),
                                        w["window"], w["kv_start"])
    np.savez_compressed(os.path.join(HERE, "prefill_small.npz"), input_sha256=c["sha256"],
                        out=out, window_input_sha256=w["sha256"], out_window=outw)


def make_prefill_more(model_mod, qk_mod):
    """Prefill geometries beyond the first fixture: Qwen35 at head_dim 256
    with a prefix (qwen35_kernels.py:395-411), gemma3's window variant at
    head_dim 256 (model.py:1567-1592), rows with no visible key, and fp32
    values outside fp16's range (model.py:1254-1272)."""
    c = cases.prefill_qwen35_d256()
    q35 = qk_mod.qwen35_full_attention_prefill(c["q"], c["k"], c["v"], c["prefix"])
    w = cases.prefill_gemma3_window_d256()
    m = _llama_model(model_mod, 128, w["H"], w["KV"], w["D"], w["D"], 10000.0, "norm")
    win = m._attention_batch_window_np(w["q"], w["k"], w["v"], w["positions"],
                                       w["H"] // w["KV"], 1.0 / np.sqrt(w["D"]),
                                       w["window"], w["kv_start"])
    e = cases.prefill_empty_rows()
    m = _llama_model(model_mod, 64, e["H"], e["KV"], e["D"], e["D"], 10000.0, "norm")
    empty = m._attention_batch_window_np(e["q"], e["k"], e["v"], e["positions"],
                                         e["H"] // e["KV"], 1.0 / np.sqrt(e["D"]),
                                         e["window"], e["kv_start"])
    g = cases.prefill_large_magnitude()
    m = _llama_model(model_mod, 64, g["H"], g["KV"], g["D"], g["D"], 10000.0, "norm")
    big = m._attention_batch_np(g["q"], g["k"], g["v"], g["positions"], g["H"] // g["KV"],
                                1.0 / np.sqrt(g["D"]))
    np.savez_compressed(
        os.path.join(HERE, "prefill_more.npz"), qwen35_d256_sha256=c["sha256"],
        qwen35_d256=q35, window_d256_sha256=w["sha256"], window_d256=win,
        empty_rows_sha256=e["sha256"], empty_rows=empty, large_sha256=g["sha256"], large=big)


def make_qwen35(qk_mod, ops_mod):
    c = cases.qwen35_decode()
    out = qk_mod.qwen35_full_attention_decode(c["q"], c["k"], c["v"])
    p = cases.qwen35_prefill()
    outp = qk_mod.qwen35_full_attention_prefill(p["q"], p["k"], p["v"], p["prefix"])
    r = cases.imrope_case()
    rot = np.array([[ops_mod.imrope_rotate(list(map(float, r["x"][i, h])),
                                           [int(x) for x in r["lanes"][i]], r["sections"],
                                           frequency_base=r["base"])
                     for h in range(r["x"].shape[1])] for i in range(r["x"].shape[0])])
    lanes = np.array([ops_mod.imrope_lane_for_pair(j, r["sections"])
                      for j in range(sum(r["sections"]))])
    g = cases.gqa_step_case()
    gqa = np.array(ops_mod.causal_gqa_step(g["q"].tolist(), g["k"].tolist(), g["v"].tolist()))
    np.savez_compressed(os.path.join(HERE, "qwen35.npz"), decode_sha256=c["sha256"],
                        decode_out=out, prefill_sha256=p["sha256"], prefill_out=outp,
                        imrope_sha256=r["sha256"], imrope_out=rot, imrope_lanes=lanes,
                        gqa_sha256=g["sha256"], gqa_out=gqa)


def make_kv_state():
    """The reference's own attention-layer state (alpaccaroo/memory.py:385-475):
    rows appended one at a time, snapshot, truncate, snapshot again."""
    from alpaccaroo import memory  # noqa: WPS433
    c = cases.kv_state_case()
    spec = memory.LayerMemorySpec(layer_index=c["layer_index"], kind="attention",
                                  kv_heads=c["KV"], key_dim=c["D"], value_dim=c["D"])
    st = memory.FullAttentionState(spec)
    for p in range(c["L"]):
        st.append(c["k"][p].ravel().tolist(), c["v"][p].ravel().tolist())
    full = st.snapshot()
    st.truncate(c["truncate"])
    cut = st.snapshot()
    np.savez_compressed(
        os.path.join(HERE, "kv_state.npz"), input_sha256=c["sha256"],
        key=np.frombuffer(full.key, np.uint8), value=np.frombuffer(full.value, np.uint8),
        length=full.logical_length, dtype=full.dtype, kind=full.kind,
        memory_bytes=full.memory_bytes(),
        key_cut=np.frombuffer(cut.key, np.uint8), value_cut=np.frombuffer(cut.value, np.uint8),
        length_cut=cut.logical_length, memory_bytes_cut=cut.memory_bytes())


def make_qwen35_layer():
    """The reference's Qwen35 full-attention layer (alpaccaroo/qwen35_runtime.py:
    597-664) run on preset projections: a stub supplies _matvec (the projected
    rows, and the identity for the output projection) and the layer's own
    trace boundaries are recorded."""
    import types
    from alpaccaroo import memory, qwen35_runtime  # noqa: WPS433
    c = cases.qwen35_layer_case()
    cfg = types.SimpleNamespace(query_heads=c["H"], kv_heads=c["KV"], key_length=c["D"],
                                value_length=c["D"], rms_epsilon=c["eps"],
                                rope_freq_base=c["base"],
                                rope_dimension_sections=c["sections"])
    out_proj = object()

    class Stub:
        config = cfg

        def _matvec(self, matrix, values):
            return values if matrix is out_proj else matrix

        def _attention_read(self, query_heads, state):
            return qwen35_runtime._causal_gqa_one(query_heads, state)

    w = types.SimpleNamespace(query_gate=c["query_gate"].tolist(), key=c["key"].tolist(),
                              value=c["value"].tolist(), query_norm=c["q_norm"].tolist(),
                              key_norm=c["k_norm"].tolist(), output=out_proj)
    spec = memory.LayerMemorySpec(layer_index=0, kind="attention", kv_heads=c["KV"],
                                  key_dim=c["D"], value_dim=c["D"])
    st = memory.FullAttentionState(spec)
    for p in range(c["L"]):
        st.append(c["k_prev"][p].ravel().tolist(), c["v_prev"][p].ravel().tolist())
    seen = {}

    def trace(name, values):
        seen[name.split(".", 2)[-1]] = np.asarray(values, dtype=np.float32).copy()

    qwen35_runtime.Qwen35Model._attention(Stub(), 0, w, [], st, c["L"], trace)
    np.savez_compressed(
        os.path.join(HERE, "qwen35_layer.npz"), input_sha256=c["sha256"],
        q_normed=seen["Qcur_normed"], k_normed=seen["Kcur_normed"],
        pregate=seen["attn_pregate"], gated=seen["attn_gated"],
        appended_key=np.frombuffer(bytes(st.key), np.float32)[-c["KV"] * c["D"]:],
        appended_value=np.frombuffer(bytes(st.value), np.float32)[-c["KV"] * c["D"]:])


def make_llama_q8(model_mod):
    """The reference's own decode step (Model._forward_np, model.py:1374-1487)
    on a small Q8_0 llama model built in memory; the oracle's Q8_0 encoder is
    checked byte for byte against the reference's quantize_q8_0 first."""
    from alpaccaroo import quants  # noqa: WPS433
    from alpaccaroo.qmatrix import QuantMatrix  # noqa: WPS433
    c = cases.llama_q8_case()
    rng = np.random.default_rng(99)
    probe = rng.normal(0.0, 0.02, 32 * 64).astype(np.float32)
    from oracle.llama_q8 import quantize_q8_0
    assert quants.quantize_q8_0(probe.tolist()) == quantize_q8_0(probe)
    E, H, KV, D, F, V = (c["n_embd"], c["n_head"], c["n_kv"], c["head_dim"], c["n_ff"],
                         c["n_vocab"])
    hp = model_mod.Hyperparams(arch="llama", n_layer=c["n_layer"], n_embd=E, n_head=H,
                               n_kv=KV, n_ff=F, n_vocab=V, n_ctx_train=4096, head_dim=D,
                               n_rot=D, rms_eps=c["rms_eps"], rope_base=c["rope_base"],
                               rope_style="norm")
    m = model_mod.Model(hp, None)
    m.n_ctx = c["n_ctx"]
    qm = lambda data, rows, cols: QuantMatrix(data, "Q8_0", rows, cols)  # noqa: E731
    for cl in c["layers"]:
        ly = model_mod.Layer()
        for slot in model_mod.Layer.__slots__:
            setattr(ly, slot, None)
        ly.attn_norm, ly.ffn_norm = cl["attn_norm"], cl["ffn_norm"]
        ly.wq, ly.wk, ly.wv = qm(cl["wq"], H * D, E), qm(cl["wk"], KV * D, E), qm(cl["wv"], KV * D, E)
        ly.wo = qm(cl["wo"], E, H * D)
        ly.w_gate, ly.w_up, ly.w_down = qm(cl["w_gate"], F, E), qm(cl["w_up"], F, E), \
            qm(cl["w_down"], E, F)
        m.layers.append(ly)
    m.tok_embd = qm(c["tok_embd"], V, E)
    m.out_norm = c["out_norm"]
    m.output = qm(c["output"], V, E)
    m._init_cache()
    import copy
    fresh = copy.deepcopy(m)  # the same weights, untouched cache, for the batch path
    logits = np.stack([np.asarray(m._forward_np(t), dtype=np.float32) for t in c["tokens"]])
    # the reference's batch path (Model.forward_batch, model.py:1274-1372) on
    # the first five tokens as one chunk, then one decode token on top of it
    n_chunk = 5
    chunk_logits = np.asarray(fresh.forward_batch(c["tokens"][:n_chunk]), dtype=np.float32)
    chunk_k0 = np.array(fresh.cache_k[0][:n_chunk], dtype=np.float32)
    after_logits = np.asarray(fresh._forward_np(c["tokens"][n_chunk]), dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "llama_q8.npz"), weights_sha256=c["sha256"],
                        tokens=np.array(c["tokens"], np.int32), logits=logits,
                        n_chunk=n_chunk, chunk_logits=chunk_logits, chunk_k0=chunk_k0,
                        after_chunk_logits=after_logits)


def main():
    model_mod, qk_mod, ops_mod = _import_reference()
    make_kv_state()
    make_llama_q8(model_mod)
    make_qwen35_layer()
    make_decode_config1(model_mod)
    make_rope_neox(model_mod)
    make_prefill(model_mod)
    make_prefill_more(model_mod, qk_mod)
    make_qwen35(qk_mod, ops_mod)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
