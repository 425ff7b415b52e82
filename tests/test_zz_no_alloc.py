"""b2a_decode_noalloc: decode for callers that can't allocate device memory.

Some callers of this library can't call cudaMalloc. A serving process may have
reserved nearly all of HBM for its KV cache. A host may route every device buffer
through its own allocator. A foreign-language host may have no device allocator at
all. The no-allocation entry point keeps the decode's split partials in a fixed
static device array instead of a caller workspace.

This test calls it through the C ABI (ctypes, raw device pointers) twice in a
row, each time on fresh inputs, and checks it against the regular b2a_decode
(given a caller workspace) within the 16-bit decode tolerance of the other
tests (2e-2 max abs).  The second call checks that leftovers of the first call
in the shared array do not leak into a later call.  It also checks the size
limit is enforced before any launch.  The file name makes pytest collect it
last; it needs nothing from the other tests and also passes alone in a fresh
process.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else t.data_ptr()


def _inputs(dev, seed, B, H, KV, D, n_ctx, lens):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B, H, D), device=dev, dtype=torch.float32, generator=g)
    k = torch.randn((B, n_ctx, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn((B, n_ctx, KV, D), device=dev, dtype=torch.bfloat16, generator=g)
    return q, k, v, torch.tensor(lens, dtype=torch.int32, device=dev)


def _decode_with_workspace(lib, q, k, v, lens, B, H, KV, D, n_ctx, split):
    from alpacca_open_sourced_by_jt_b200 import _lib
    out = torch.empty((B, H, D), dtype=torch.float32, device=q.device)
    lse = torch.empty((B, H), dtype=torch.float32, device=q.device)
    nbytes = lib.b2a_decode_workspace_bytes(B, H, D, n_ctx, split)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _lib.check(lib.b2a_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(lens), _ptr(out), _ptr(lse),
                              _ptr(ws), nbytes, B, H, KV, D, n_ctx, n_ctx * KV * D, _lib.BF16,
                              float(D) ** -0.5, n_ctx, split,
                              torch.cuda.current_stream().cuda_stream))
    return out, lse


def _decode_noalloc(lib, q, k, v, lens, B, H, KV, D, n_ctx, split):
    from alpacca_open_sourced_by_jt_b200 import _lib
    out = torch.empty((B, H, D), dtype=torch.float32, device=q.device)
    lse = torch.empty((B, H), dtype=torch.float32, device=q.device)
    _lib.check(lib.b2a_decode_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(lens), _ptr(out),
                                      _ptr(lse), B, H, KV, D, n_ctx, n_ctx * KV * D, _lib.BF16,
                                      float(D) ** -0.5, n_ctx, split,
                                      torch.cuda.current_stream().cuda_stream))
    return out, lse


def test_noalloc_matches_decode_on_two_calls(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib
    lib = _lib.load()
    calls = [
        # (seed, B, H, KV, D, n_ctx, lens, split_rows)
        (1, 4, 32, 8, 128, 8192, [8192, 77, 5000, 1], 0),
        (2, 3, 64, 8, 128, 4096, [4096, 3000, 129], 256),
    ]
    for seed, B, H, KV, D, n_ctx, lens, split in calls:
        q, k, v, lt = _inputs(cuda_dev, seed, B, H, KV, D, n_ctx, lens)
        ref_out, ref_lse = _decode_with_workspace(lib, q, k, v, lt, B, H, KV, D, n_ctx, split)
        out, lse = _decode_noalloc(lib, q, k, v, lt, B, H, KV, D, n_ctx, split)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert (out - ref_out).abs().max().item() < 2e-2
        assert (lse - ref_lse).abs().max().item() < 2e-2
    code, aux = _lib.device_error(clear=True)
    assert code == 0, (code, aux)


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib
    lib = _lib.load()
    p = 1 << 20  # never dereferenced: the size check returns before any launch
    rc = lib.b2a_decode_noalloc(p, p, p, p, p, None, 64, 64, 8, 256, 131072,
                                131072 * 8 * 256, _lib.BF16, 0.0625, 131072, 64, None)
    assert rc == _lib.ERR_WORKSPACE
    msg = _lib.last_error()
    assert "static array" in msg and str(16 << 20) in msg
