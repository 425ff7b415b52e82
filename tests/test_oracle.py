"""Pin the CPU oracle to the reference's own outputs (tests/golden/*.npz,
made by tests/golden/make_golden.py running alpaccaroo), and check the
oracle's internal identities (split combine == full softmax, etc.)."""
import math

import numpy as np
import pytest

import oracle
from tests.conftest import rel_err
from tests.golden import cases


def test_config1_inputs_regenerate(golden):
    g = golden("decode_config1.npz")
    assert cases.decode_config1()["sha256"] == str(g["input_sha256"])


def test_config1_rope_tables_bit_exact(golden):
    g = golden("decode_config1.npz")
    cos, sin = oracle.rope_tables(512, 64, 500000.0)
    rows = g["sample_rows"]
    assert np.array_equal(cos[rows], g["cos_tab"])
    assert np.array_equal(sin[rows], g["sin_tab"])


def test_config1_decode_matches_reference(golden):
    g = golden("decode_config1.npz")
    c = cases.decode_config1()
    cos, sin = oracle.rope_tables(c["L"], c["D"], c["base"])
    K = np.stack([oracle.rope_vec(c["k_raw"][p].reshape(-1), c["KV"], p, cos, sin, c["D"],
                                  c["D"], "norm").reshape(c["KV"], c["D"])
                  for p in range(c["L"])])
    q = oracle.rope_vec(c["q_raw"].reshape(-1), c["H"], c["L"] - 1, cos, sin, c["D"], c["D"],
                        "norm")
    # rotation is elementwise: bit-identical to the reference
    assert np.array_equal(q, g["q_rot"])
    assert np.array_equal(K[g["sample_rows"]], g["k_rot_rows"])
    out = oracle.attention_decode(q, K, c["v"], c["H"] // c["KV"], 1.0 / math.sqrt(c["D"]))
    assert rel_err(out, g["out"]) < 1e-5


def test_rope_neox_partial_bit_exact(golden):
    g = golden("rope_neox.npz")
    c = cases.rope_neox()
    assert c["sha256"] == str(g["input_sha256"])
    cos, sin = oracle.rope_tables(c["n_ctx"], c["n_rot"], c["base"])
    assert np.array_equal(cos, g["cos_tab"]) and np.array_equal(sin, g["sin_tab"])
    q = np.stack([oracle.rope_vec(c["q"][i].reshape(-1), c["H"], int(p), cos, sin, c["D"],
                                  c["n_rot"], "neox") for i, p in enumerate(c["positions"])])
    assert np.array_equal(q, g["q_rot"])
    k = oracle.rope_batch(c["k"].reshape(len(c["positions"]), -1), c["KV"], c["positions"], cos,
                          sin, c["D"], c["n_rot"], "neox")
    assert np.array_equal(k, g["k_rot"])


def test_prefill_matches_reference(golden):
    g = golden("prefill_small.npz")
    c = cases.prefill_small()
    assert c["sha256"] == str(g["input_sha256"])
    out = oracle.attention_batch(c["q"], c["k"], c["v"], c["positions"], c["H"] // c["KV"],
                                 1.0 / math.sqrt(c["D"]))
    assert rel_err(out, g["out"]) < 1e-5
    w = cases.prefill_window()
    assert w["sha256"] == str(g["window_input_sha256"])
    outw = oracle.attention_batch(w["q"], w["k"], w["v"], w["positions"], w["H"] // w["KV"],
                                  1.0 / math.sqrt(w["D"]), w["window"], w["kv_start"])
    assert rel_err(outw, g["out_window"]) < 1e-5


def test_prefill_more_matches_reference(golden):
    """Head_dim 256 (Qwen35 with a prefix, gemma3's window), rows with no
    visible key, fp32 values outside fp16's range."""
    g = golden("prefill_more.npz")
    c = cases.prefill_qwen35_d256()
    assert c["sha256"] == str(g["qwen35_d256_sha256"])
    assert rel_err(oracle.qwen35_full_attention_prefill(c["q"], c["k"], c["v"], c["prefix"]),
                   g["qwen35_d256"]) < 1e-5
    for name, case in (("window_d256", cases.prefill_gemma3_window_d256()),
                       ("empty_rows", cases.prefill_empty_rows())):
        assert case["sha256"] == str(g[name + "_sha256"])
        out = oracle.attention_batch(case["q"], case["k"], case["v"], case["positions"],
                                     case["H"] // case["KV"], 1.0 / math.sqrt(case["D"]),
                                     case["window"], case["kv_start"])
        assert rel_err(out, g[name]) < 1e-5
    # rows 0..9 of the empty-row case see no key: the reference gives them
    # the mean of all value rows (its -1e30 mask weighs every key equally)
    e = cases.prefill_empty_rows()
    mean_v = e["v"].mean(axis=0)  # (KV, D)
    got = g["empty_rows"].reshape(20, e["H"], e["D"])[:10]
    want = np.repeat(mean_v, e["H"] // e["KV"], axis=0)[None]
    assert np.abs(got - want).max() < 1e-6
    b = cases.prefill_large_magnitude()
    assert b["sha256"] == str(g["large_sha256"])
    out = oracle.attention_batch(b["q"], b["k"], b["v"], b["positions"], b["H"] // b["KV"],
                                 1.0 / math.sqrt(b["D"]))
    assert rel_err(out, g["large"]) < 1e-5
    assert np.abs(g["large"]).max() > 6.5e4  # beyond fp16's largest finite value


def test_qwen35_paths_match_reference(golden):
    g = golden("qwen35.npz")
    c = cases.qwen35_decode()
    assert c["sha256"] == str(g["decode_sha256"])
    assert rel_err(oracle.qwen35_full_attention_decode(c["q"], c["k"], c["v"]),
                   g["decode_out"]) < 1e-5
    p = cases.qwen35_prefill()
    assert p["sha256"] == str(g["prefill_sha256"])
    assert rel_err(oracle.qwen35_full_attention_prefill(p["q"], p["k"], p["v"], p["prefix"]),
                   g["prefill_out"]) < 1e-5
    r = cases.imrope_case()
    assert r["sha256"] == str(g["imrope_sha256"])
    lanes = [oracle.imrope_lane_for_pair(j, r["sections"]) for j in range(sum(r["sections"]))]
    assert lanes == list(g["imrope_lanes"])
    rot = np.array([[oracle.imrope_rotate(r["x"][i, h], r["lanes"][i], r["sections"], r["base"])
                     for h in range(3)] for i in range(3)])
    assert np.array_equal(rot, g["imrope_out"])
    q = cases.gqa_step_case()
    assert q["sha256"] == str(g["gqa_sha256"])
    assert np.allclose(np.array(oracle.causal_gqa_step(q["q"], q["k"], q["v"])), g["gqa_out"],
                       rtol=0, atol=1e-15)


@pytest.mark.parametrize("split", [1, 7, 64, 512])
def test_split_combine_equals_full(split):
    rng = np.random.default_rng(5)
    q = rng.standard_normal((8, 32), dtype=np.float32)
    K = rng.standard_normal((300, 2, 32), dtype=np.float32)
    V = rng.standard_normal((300, 2, 32), dtype=np.float32)
    pm, pl, pacc = oracle.split_decode_partials(q, K, V, 4, 0.2, split)
    full = oracle.attention_decode(q, K, V, 4, 0.2)
    assert rel_err(oracle.split_combine(pm, pl, pacc), full) < 1e-5


def test_lse_combine_of_shards_equals_full():
    rng = np.random.default_rng(6)
    H, D, L, G = 8, 16, 200, 3
    q = rng.standard_normal((H, D), dtype=np.float32)
    K = rng.standard_normal((L, 2, D), dtype=np.float32)
    V = rng.standard_normal((L, 2, D), dtype=np.float32)
    bounds = [0, 50, 51, 200]
    os_, ls_ = [], []
    for g in range(G):
        a, b = bounds[g], bounds[g + 1]
        pm, pl, pacc = oracle.split_decode_partials(q, K[a:b], V[a:b], 4, 0.25, 10 ** 9)
        os_.append(pacc[:, 0] / pl[:, :1])
        ls_.append(pm[:, 0] + np.log(pl[:, 0]))
    out, _ = oracle.lse_combine(np.stack(os_), np.stack(ls_))
    assert rel_err(out, oracle.attention_decode(q, K, V, 4, 0.25)) < 1e-5
    # an empty shard (lse = -inf) contributes nothing
    out2, _ = oracle.lse_combine(np.concatenate([np.stack(os_), np.zeros((1, H, D))]),
                                 np.concatenate([np.stack(ls_), np.full((1, H), -np.inf)]))
    assert rel_err(out2, out) < 1e-12


def test_qwen35_layer_matches_reference(golden):
    g = golden("qwen35_layer.npz")
    c = cases.qwen35_layer_case()
    assert c["sha256"] == str(g["input_sha256"])
    q, k, att, gated = oracle.qwen35_attention_layer(
        c["query_gate"], c["key"], c["value"], c["q_norm"], c["k_norm"], c["eps"],
        c["sections"], c["base"], c["L"], c["k_prev"], c["v_prev"])
    # same double-precision steps rounded to f32 at the same boundaries: bit-exact
    assert np.array_equal(q.ravel(), g["q_normed"])
    assert np.array_equal(k.ravel(), g["k_normed"])
    assert np.array_equal(k.ravel(), g["appended_key"])
    assert np.array_equal(c["value"], g["appended_value"])
    assert np.array_equal(att.ravel(), g["pregate"])
    assert np.array_equal(gated.ravel(), g["gated"])


def test_llama_q8_decode_matches_reference(golden):
    g = golden("llama_q8.npz")
    c = cases.llama_q8_case()
    assert c["sha256"] == str(g["weights_sha256"])
    n_ctx, KV, D = c["n_ctx"], c["n_kv"], c["head_dim"]
    cos, sin = oracle.rope_tables(n_ctx, D, c["rope_base"])
    ck = [np.zeros((n_ctx, KV, D), np.float32) for _ in range(c["n_layer"])]
    cv = [np.zeros((n_ctx, KV, D), np.float32) for _ in range(c["n_layer"])]
    for pos, tok in enumerate(c["tokens"]):
        logits = oracle.llama_q8.forward_token(c, tok, pos, ck, cv, cos, sin)
        # same f32 operations; BLAS/einsum reduction orders differ from NumPy's here
        assert rel_err(logits, g["logits"][pos]) < 1e-5
