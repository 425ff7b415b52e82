"""benchmark config 5 at its full size: the benchmarked model against the oracle.

The model is the one bench.py's decode_step leg times: LlamaQ8.random with
16 layers, hidden 2048, 32 q / 8 KV heads of 64, SwiGLU FFN 8192, vocab
128256, RMSNorm eps 1e-5, RoPE base 500000, Q8_0 weights N(0, 0.02) from
seed 5, an f16 KV cache of 4096 rows.  Its Q8_0 matrices are copied back
to the host as GGUF Q8_0 records and run through oracle/llama_q8.py's
restatement of Model._forward_np (alpaccaroo/model.py:1374-1487; pinned to
the reference's own logits by tests/test_oracle.py on the small golden
model).  Cache rows 0..4093 hold N(0, 1) values (the bench's fill), in f16
on the device and their exact f32 values in the oracle; tokens then run at
positions 4094 and 4095, so the second token attends to the first one's
appended row.  Bar: 1e-2 normwise on the logits, the f16-cache bar of
tests/test_decode_chain_gpu.py (the chain stores the new rows in f16, the
oracle keeps them in f32)."""
import numpy as np
import pytest
import torch

import oracle
from oracle import llama_q8 as L
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

C5 = dict(n_layer=16, n_embd=2048, n_head=32, n_kv=8, head_dim=64, n_ff=8192, n_vocab=128256,
          rms_eps=1e-5, rope_base=500000.0)
N_CTX = 4096


def _records(codes: np.ndarray, scales: np.ndarray) -> bytes:
    """(rows, cols) int8 codes and (rows, cols/32) f16 scales -> Q8_0 records."""
    rec = np.empty(codes.size // 32, dtype=[("d", "<f2"), ("qs", "i1", 32)])
    rec["d"] = scales.reshape(-1)
    rec["qs"] = codes.reshape(-1, 32)
    return rec.tobytes()


def _host(mat, r0=None, r1=None):
    codes = mat.codes[r0:r1].cpu().numpy()
    scales = mat.scales[r0:r1].cpu().numpy()
    return _records(codes, scales)


def _oracle_model(m) -> dict:
    """The device model's weights as the oracle's model dict."""
    E, H, KV, D, F, V = m.E, m.H, m.KV, m.D, m.F, m.V
    layers = []
    for ly in m.layers:
        qkv = ly["wqkv"]
        # gate/up rows are interleaved in 8-row groups (Q8Matrix.interleave)
        gu_c = ly["wgu"].codes.view(F // 8, 2, 8, E)
        gu_s = ly["wgu"].scales.view(F // 8, 2, 8, E // 32)
        layers.append(dict(
            attn_norm=ly["attn_norm"].cpu().numpy(), ffn_norm=ly["ffn_norm"].cpu().numpy(),
            wq=_host(qkv, 0, H * D), wk=_host(qkv, H * D, (H + KV) * D),
            wv=_host(qkv, (H + KV) * D, (H + 2 * KV) * D), wo=_host(ly["wo"]),
            w_gate=_records(gu_c[:, 0].reshape(F, E).cpu().numpy(),
                            gu_s[:, 0].reshape(F, E // 32).cpu().numpy()),
            w_up=_records(gu_c[:, 1].reshape(F, E).cpu().numpy(),
                          gu_s[:, 1].reshape(F, E // 32).cpu().numpy()),
            w_down=_host(ly["w_down"])))
    return dict(n_embd=E, n_head=H, n_kv=KV, head_dim=D, n_ff=F, n_vocab=V, rms_eps=m.eps,
                tok_embd=_host(m.tok_embd), out_norm=m.out_norm.cpu().numpy(),
                output=_host(m.output), layers=layers)


def test_config5_fullsize_logits_match_oracle(cuda_dev):
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    m = LlamaQ8.random(**C5, seed=5, dev=cuda_dev)
    chain = DecodeChain(m, N_CTX, torch.float16)
    g = torch.Generator(device=cuda_dev).manual_seed(6)
    for k, v in zip(chain.k_cache, chain.v_cache):
        k.normal_(generator=g)
        v.normal_(generator=g)
    torch.cuda.synchronize()
    cache_k = [k[0].float().cpu().numpy() for k in chain.k_cache]
    cache_v = [v[0].float().cpu().numpy() for v in chain.v_cache]
    model = _oracle_model(m)
    cos, sin = oracle.rope_tables(N_CTX, m.D, m.rope_base)
    for token, pos in ((1234, N_CTX - 2), (77, N_CTX - 1)):
        got = chain(token, pos).numpy().copy()
        want = L.forward_token(model, token, pos, cache_k, cache_v, cos, sin)
        err = rel_err(got, want)
        assert err < 1e-2, (pos, err)
    # the chain's own appended row equals the oracle's rotated k, rounded to f16
    k_dev = chain.k_cache[0][0, N_CTX - 1].float().cpu().numpy()
    assert np.abs(k_dev - cache_k[0][N_CTX - 1]).max() <= \
        2e-3 * max(1.0, float(np.abs(cache_k[0][N_CTX - 1]).max()))
