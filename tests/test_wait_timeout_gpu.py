"""The bounded device wait runs out without faulting or hanging the GPU.

Every mbarrier wait in the library's kernels gives up after a fixed limit
(2 s of %globaltimer), records B2A_ERR_TIMEOUT in the device error record
and lets the kernel return.  b2a_selftest_wait_timeout launches one thread
that waits on a barrier nothing arrives on: the test checks that the wait
ran out after about the limit, that the record names it, and that the
context still runs a decode correctly afterwards.
"""
import math
import time

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_mbarrier_wait_runs_out_and_context_survives(cuda_dev):
    from alpacca_open_sourced_by_jt_b200 import _lib, device
    _lib.device_error(clear=True)
    t0 = time.perf_counter()
    _lib.check(_lib.load().b2a_selftest_wait_timeout(None))
    code, aux = _lib.device_error(clear=True)
    elapsed = time.perf_counter() - t0
    assert code == _lib.ERR_TIMEOUT and aux == 0x7F000, (code, aux)
    assert 1.5 < elapsed < 30.0, elapsed
    # the context is intact: a decode still matches the oracle
    g = torch.Generator().manual_seed(3)
    H, KV, D, L = 8, 2, 64, 300
    q = torch.randn((1, H, D), generator=g)
    k = torch.randn((1, L, KV, D), generator=g).to(torch.bfloat16)
    v = torch.randn((1, L, KV, D), generator=g).to(torch.bfloat16)
    lens = torch.tensor([L], dtype=torch.int32)
    out = device.decode(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), lens.to(cuda_dev))
    ref = oracle.attention_decode(q[0].numpy(), k[0].float().numpy(), v[0].float().numpy(),
                                  H // KV, 1.0 / math.sqrt(D))
    assert np.abs(out[0].cpu().numpy() - ref).max() < 2e-2
    assert _lib.device_error(clear=True) == (0, 0)
