"""Device-resident prefill chunks (prefill_chain.py) vs the reference's batch
path.

tests/golden/llama_q8.npz holds, for the small Q8_0 llama model, the logits
of the reference's Model.forward_batch on the first five tokens as one chunk
(alpaccaroo/model.py:1274-1372), its layer-0 K rows, and the logits of the
decode token that follows.  The chunk runs its GEMMs on 16-bit dequantized
weights (decoded inside the kernel from the Q8_0 codes, or a 16-bit copy made
at set-up) and activations (f32 accumulation) and its attention on the 16-bit
cache, so the bar is 2e-2 normwise on the logits and 2e-2 absolute on the
stored K rows; the same chunk split in two (the second attending over the
first's cached rows) must agree with the single chunk, and the two weight
paths must agree with each other to fp32 rounding.
"""
import numpy as np
import pytest
import torch

from tests.conftest import max_abs_err, rel_err
from tests.golden import cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("weights", ["q8", "f16", "q8_dequant"])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("split", [None, 3])
def test_chunk_prefill_matches_reference(cuda_dev, golden, dt, split, weights):
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    from alpacca_open_sourced_by_jt_b200.prefill_chain import ChunkPrefill
    g = golden("llama_q8.npz")
    c = cases.llama_q8_case()
    assert c["sha256"] == str(g["weights_sha256"])
    n = int(g["n_chunk"])
    chain = DecodeChain(LlamaQ8.from_spec(c, cuda_dev), c["n_ctx"], dt)
    pre = ChunkPrefill(chain, max_chunk=8, weights=weights)
    if split is None:
        logits = pre(c["tokens"][:n], 0)
    else:
        assert pre(c["tokens"][:split], 0, want_logits=False) is None
        logits = pre(c["tokens"][split:n], split)
    torch.cuda.synchronize()
    assert rel_err(logits, g["chunk_logits"]) < 2e-2
    k0 = chain.k_cache[0][0, :n].float().cpu().numpy()
    assert max_abs_err(k0, g["chunk_k0"]) < 2e-2
    # decoding continues from the chunk's cache rows
    after = chain(c["tokens"][n], n).numpy()
    assert rel_err(after, g["after_chunk_logits"]) < 2e-2


def test_chunk_prefill_rejects_bad_requests(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    from alpacca_open_sourced_by_jt_b200.prefill_chain import ChunkPrefill
    c = cases.llama_q8_case()
    model = LlamaQ8.from_spec(c, cuda_dev)
    with pytest.raises(_lib.B2AShapeError):
        ChunkPrefill(DecodeChain(model, c["n_ctx"], torch.float32))
    pre = ChunkPrefill(DecodeChain(model, c["n_ctx"], torch.float16), max_chunk=4)
    with pytest.raises(_lib.B2AShapeError):
        pre([1, 2, 3, 4, 5], 0)
    with pytest.raises(_lib.B2AError):
        pre([1, 2], c["n_ctx"] - 1)
    with pytest.raises(_lib.B2AError):
        pre([c["n_vocab"]], 0)
    assert np.isfinite(pre([1, 2], 0)).all()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_chunk_q8_weights_equal_16bit_copy(cuda_dev, dt):
    """The in-kernel Q8_0 decode and the per-matrix dequantization give the
    products of the 16-bit copy: the same logits and K/V rows up to the
    residual sums' order."""
    from alpacca_open_sourced_by_jt_b200.decode_chain import DecodeChain, LlamaQ8
    from alpacca_open_sourced_by_jt_b200.prefill_chain import ChunkPrefill
    c = cases.llama_q8_case()
    model = LlamaQ8.from_spec(c, cuda_dev)
    res = []
    for weights in ("q8", "f16", "q8_dequant"):
        chain = DecodeChain(model, c["n_ctx"], dt)
        logits = ChunkPrefill(chain, max_chunk=8, weights=weights)(c["tokens"][:6], 0)
        res.append((logits, chain.k_cache[1][0, :6].float().cpu().numpy()))
    for other in res[1:]:
        assert rel_err(res[0][0], other[0]) < 1e-5
        assert max_abs_err(res[0][1], other[1]) < 1e-2  # one 16-bit rounding apart at most
