"""DecodeStep: the graph-replayed decode step (pinned host rows in, fused
RoPE + append, split-KV decode, pinned host output out).

Checked against the eager device calls on a copy of the same caches (same
kernels and split, so outputs and caches must be bit-identical), and one
step against the oracle (the reference's per-sequence rope, cache store and
_attention_np; alpaccaroo/model.py:1418-1440) within the 16-bit-cache
tolerance of the decode tests (2e-2 max abs error).
"""
import math

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import max_abs_err

pytestmark = pytest.mark.gpu


def test_decode_step_graph_matches_eager_and_oracle(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import device
    from alpacca_open_sourced_by_jt_b200.decode_step import DecodeStep
    rng = np.random.default_rng(60)
    B, H, KV, D, n_ctx = 4, 32, 8, 128, 1024
    kc = torch.from_numpy(rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)).to(
        cuda_dev).to(torch.bfloat16)
    vc = torch.from_numpy(rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)).to(
        cuda_dev).to(torch.bfloat16)
    k_ref, v_ref = kc.clone(), vc.clone()
    ct, st = device.rope_tables(n_ctx, D, 500000.0, device=cuda_dev)
    step = DecodeStep(kc, vc, ct, st, H)
    torch.cuda.synchronize()
    # construction leaves the caller's caches alone
    assert torch.equal(kc, k_ref) and torch.equal(vc, v_ref)
    cos, sin = oracle.rope_tables(n_ctx, D, 500000.0)
    pos = rng.integers(0, n_ctx - 8, size=B).astype(np.int32)
    for s in range(4):
        p = pos + s
        q = rng.standard_normal((B, H, D), dtype=np.float32)
        k = rng.standard_normal((B, KV, D), dtype=np.float32)
        v = rng.standard_normal((B, KV, D), dtype=np.float32)
        got = step(q, k, v, p).clone()
        # the same step through the eager device API on the copied caches
        qd = torch.from_numpy(q).to(cuda_dev)
        pd = torch.from_numpy(p).to(cuda_dev)
        device.rope_append(qd, torch.from_numpy(k).to(cuda_dev), torch.from_numpy(v).to(cuda_dev),
                           pd, ct, st, k_cache=k_ref, v_cache=v_ref, per_sequence=True)
        want = device.decode(qd, k_ref, v_ref, pd + 1)
        torch.cuda.synchronize()
        assert torch.equal(got, want.cpu())
        assert torch.equal(kc, k_ref) and torch.equal(vc, v_ref)
        if s == 3:
            kh, vh = kc.float().cpu().numpy(), vc.float().cpu().numpy()
            qr = oracle.rope_batch(q.reshape(B, -1), H, p, cos, sin, D, D, "norm").reshape(B, H, D)
            ref = oracle.attention_decode_varlen(qr, kh, vh, p + 1, H // KV, 1.0 / math.sqrt(D))
            assert max_abs_err(got.numpy(), ref) < 2e-2


def test_decode_step_rejects_positions_outside_the_cache(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    from alpacca_open_sourced_by_jt_b200.decode_step import DecodeStep
    B, H, KV, D, n_ctx = 2, 8, 2, 64, 64
    kc = torch.zeros((B, n_ctx, KV, D), dtype=torch.float16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    ct, st = device.rope_tables(n_ctx, D, 10000.0, device=cuda_dev)
    step = DecodeStep(kc, vc, ct, st, H)
    with pytest.raises(_lib.B2AError):
        step(positions=np.array([0, n_ctx], np.int32))
    with pytest.raises(_lib.B2AError):
        step(positions=np.array([-1, 0], np.int32))
    out = step(positions=np.array([0, n_ctx - 1], np.int32))
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("dt,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float32, 64)])
def test_programmatic_launches_match_plain(cuda_dev, dt, D):
    """RoPE + append and the decode launched as programmatic dependents
    (b2a_set_launch_flags(B2A_LAUNCH_PDL)): the decode streams the rows below
    each sequence's newest before waiting for the append, so eager calls and
    a captured graph must give the plain launches' outputs and caches bit for
    bit.  Lengths 1, 65 (the newest row opens a 64-row tile), 700 and 1024."""
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    rng = np.random.default_rng(61)
    H, KV, n_ctx = 16, 4, 1024
    lens = np.array([1, 65, 700, 1024], dtype=np.int32)
    B = len(lens)
    base_k = torch.from_numpy(rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)).to(
        cuda_dev).to(dt)
    base_v = torch.from_numpy(rng.standard_normal((B, n_ctx, KV, D), dtype=np.float32)).to(
        cuda_dev).to(dt)
    ct, st = device.rope_tables(n_ctx, D, 10000.0, device=cuda_dev)
    q = torch.from_numpy(rng.standard_normal((B, H, D), dtype=np.float32)).to(cuda_dev)
    k = torch.from_numpy(rng.standard_normal((B, KV, D), dtype=np.float32)).to(cuda_dev)
    v = torch.from_numpy(rng.standard_normal((B, KV, D), dtype=np.float32)).to(cuda_dev)
    pos = torch.from_numpy(lens - 1).to(cuda_dev)
    ln = torch.from_numpy(lens).to(cuda_dev)

    def step(kc, vc, out):
        qq = q.clone()
        device.rope_append(qq, k, v, pos, ct, st, k_cache=kc, v_cache=vc, per_sequence=True)
        device.decode(qq, kc, vc, ln, max_len=n_ctx, out=out)
        return qq

    kp, vp = base_k.clone(), base_v.clone()
    want = torch.zeros((B, H, D), device=cuda_dev)
    step(kp, vp, want)
    torch.cuda.synchronize()
    # eager, programmatic
    ke, ve = base_k.clone(), base_v.clone()
    got = torch.zeros_like(want)
    with device.launch_flags(_lib.LAUNCH_PDL):
        step(ke, ve, got)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(ke, kp) and torch.equal(ve, vp)
    # captured, programmatic (workspace preallocated; no allocation in the capture)
    kg, vg = base_k.clone(), base_v.clone()
    gout = torch.zeros_like(want)
    split = device.decode_split_rows(B, KV, n_ctx, dt)
    ws = device.decode_workspace(B, H, D, n_ctx, split, cuda_dev)
    qq = q.clone()
    s = torch.cuda.Stream(device=cuda_dev)
    g = torch.cuda.CUDAGraph()
    with device.launch_flags(_lib.LAUNCH_PDL), torch.cuda.graph(g, stream=s):
        qq.copy_(q)
        device.rope_append(qq, k, v, pos, ct, st, k_cache=kg, v_cache=vg, per_sequence=True)
        device.decode(qq, kg, vg, ln, max_len=n_ctx, out=gout, workspace=ws, split_rows=split)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, want)
    assert torch.equal(kg, kp) and torch.equal(vg, vp)
    # the flag is restored on exit
    assert _lib.load().b2a_set_launch_flags(0) == 0
