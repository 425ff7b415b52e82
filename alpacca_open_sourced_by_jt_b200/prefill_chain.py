"""Device-resident prefill chunks for a Q8_0 llama model.

The reference's batch path (Model.forward_batch, alpaccaroo/model.py:1274-1372;
its GPU twin DecodeChain.prefill_chunk, cuda.py:1943-2080, with the
codes-decoding SIMT GEMM of cuda.py:287-422) runs a chunk of T tokens per
layer as: RMSNorm, q/k/v GEMMs, RoPE with the K/V rows stored at their
positions, causal GQA attention, output GEMM + residual, RMSNorm, gate/up
GEMMs, SwiGLU, down GEMM + residual; then the last row's logits.

Here the chunk stays on the device end to end and writes its K/V rows
straight into a DecodeChain's caches, so decoding continues from it:

  embed rows              b2a_q8_embed (all T tokens)
  per layer:
    h    = RMSNorm(x)      b2a_rmsnorm_rows, written as the cache's 16-bit type
    q, k, v = h . Wqkv^T, RoPE, K/V rows appended, q rotated to 16 bits
                           b2a_gemm_qkv_rope (tcgen05, all in the epilogue)
    att  = causal prefill over cache rows 0..pos0+T-1  b2a_prefill (tcgen05)
    x   += att . Wo^T      b2a_gemm, the residual added in its epilogue, in place
    h    = RMSNorm(x)      b2a_rmsnorm_rows
    act  = SwiGLU(h . Wgu^T)  b2a_gemm with the SwiGLU epilogue, 16-bit out
    x   += act . Wdown^T   b2a_gemm, residual in the epilogue
  logits = Woutput . RMSNorm(x[T-1])   b2a_q8_gemv (the decode path's Q8_0 GEMV)

weights="f16" (the default): one 16-bit dequantized copy per matrix made at
set-up (2 bytes per weight) and the plain b2a_gemm.
weights="q8": the GEMMs read the decode chain's own Q8_0 matrices
(b2a_gemm_q8 / b2a_gemm_qkv_rope_q8: int8 codes into shared memory, d * code
written as 16-bit operand tiles inside the kernel), as the reference's
codes-decoding GEMM does, and the gate/up product takes the GEMV's 8-row
interleave (GEMM_SWIGLU8): no weight copy at all, for when the copy does not
fit; on one B200 its config-5 chunk takes 8.0 ms against 4.6 ms.
weights="q8_dequant": the decode chain's Q8_0 matrices again, each turned
into 16-bit rows (b2a_q8_dequant, HBM-bound) in one reusable buffer just
before its b2a_gemm: the buffer holds the largest matrix (the gate/up rows,
67 MB at config 5) instead of a copy of all of them.
All three give the same products bit for bit (the in-place residuals up to
their summation order); the 16-bit operands with fp32 accumulation are the one
precision step away from the reference's f32 SIMT GEMM.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib, device
from .decode_chain import DecodeChain, PDL, Q8Matrix


def _dequant(q: Q8Matrix, dt: torch.dtype) -> torch.Tensor:
    """(rows, cols) weights d * code in dt (exact codes, f16 scale, one rounding)."""
    w = q.codes.float().view(q.rows, q.cols // 32, 32) * q.scales.float()[:, :, None]
    return w.reshape(q.rows, q.cols).to(dt).contiguous()


class ChunkPrefill:
    """Prefill chunks of up to max_chunk tokens into `chain`'s caches (which
    must be f16 or bf16: the attention runs on the tcgen05 prefill kernel)."""

    def __init__(self, chain: DecodeChain, max_chunk: int = 256, weights: str = "f16"):
        _lib.load()
        m = chain.m
        self.chain, self.m = chain, m
        dt = chain.k_cache[0].dtype
        if dt not in (torch.float16, torch.bfloat16):
            raise _lib.B2AShapeError(_lib.ERR_DTYPE, "chunk prefill needs an f16 or bf16 cache")
        self.dt, self.code = dt, device._code(dt)
        dev = m.device
        self.max_chunk = int(max_chunk)
        self.scratch = None
        if weights in ("q8", "q8_dequant"):
            if m.F % 8:  # the gate/up matrix's rows: 16-row groups of 8 gate + 8 up
                raise _lib.B2AShapeError(_lib.ERR_SHAPE, "Q8_0 chunk GEMMs need n_ff % 8 == 0")
            self.w = [dict(qkv=ly["wqkv"], wo=ly["wo"], gu=ly["wgu"], down=ly["w_down"])
                      for ly in m.layers]
            if weights == "q8_dequant":
                biggest = max(q.rows * q.cols for q in self.w[0].values())
                self.scratch = torch.empty(biggest, dtype=dt, device=dev)
        elif weights == "f16":
            if m.F % 128:
                raise _lib.B2AShapeError(_lib.ERR_SHAPE, "16-bit chunk GEMMs need n_ff % 128 == 0")
            self.w = [dict(qkv=_dequant(ly["wqkv"], dt), wo=_dequant(ly["wo"], dt),
                           gu=self._gate_up(_dequant(ly["wgu"], dt), m.F),
                           down=_dequant(ly["w_down"], dt))
                      for ly in m.layers]
        else:
            raise _lib.B2AError(_lib.ERR_ARG, f"weights {weights!r} (f16, q8 or q8_dequant)")
        self.weights = weights
        T, E, H, KV, D, F = self.max_chunk, m.E, m.H, m.KV, m.D, m.F
        self.x = torch.zeros((T, E), dtype=torch.float32, device=dev)
        self.h = torch.zeros((T, E), dtype=dt, device=dev)
        self.qrot = torch.zeros((T, H, D), dtype=dt, device=dev)
        self.att = torch.zeros((T, H, D), dtype=dt, device=dev)
        self.act = torch.zeros((T, F), dtype=dt, device=dev)
        self.tokens = torch.zeros(T, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(T, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(m.V, dtype=torch.float32, device=dev)

    @staticmethod
    def _gate_up(w: torch.Tensor, F: int) -> torch.Tensor:
        """The decode path's gate/up matrix (8 gate rows, 8 up rows, ...) as
        the GEMM's SwiGLU layout: 128 gate rows, then the matching 128 up
        rows, for each 128 features."""
        g = w.view(F // 8, 2, 8, -1)
        gate, up = g[:, 0].reshape(F, -1), g[:, 1].reshape(F, -1)
        return torch.stack([gate.view(F // 128, 128, -1), up.view(F // 128, 128, -1)],
                           1).reshape(2 * F, -1).contiguous()

    def _norm(self, x, w, T):
        m = self.m
        _lib.check(_lib.load().b2a_rmsnorm_rows(
            x.data_ptr(), m.E, w.data_ptr(), m.eps, self.h.data_ptr(), m.E, self.code, T, m.E,
            device._stream(None)))
        return self.h[:T]

    def __call__(self, tokens, pos0: int, want_logits: bool = True):
        """Run tokens (a list of ids) at cache rows pos0.. and return the last
        row's logits (a host f32 array) or None."""
        m, ch = self.m, self.chain
        T = len(tokens)
        if not 0 < T <= self.max_chunk:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, f"chunk of {T} tokens (max {self.max_chunk})")
        if pos0 < 0 or pos0 + T > ch.n_ctx:
            raise _lib.B2AError(_lib.ERR_POSITION, f"rows [{pos0}, {pos0 + T}) outside the cache")
        toks = np.asarray(tokens, dtype=np.int32)
        if toks.min() < 0 or toks.max() >= m.V:
            raise _lib.B2AError(_lib.ERR_ARG, "token id outside the vocabulary")
        H, KV, D, E = m.H, m.KV, m.D, m.E
        qd = H * D
        lib = _lib.load()
        st = device._stream(None)
        self.tokens[:T].copy_(torch.from_numpy(toks))
        torch.arange(pos0, pos0 + T, dtype=torch.int32, out=self.positions[:T])
        pos = self.positions[:T]
        x = self.x[:T]
        _lib.check(lib.b2a_q8_embed(m.tok_embd.codes.data_ptr(), m.tok_embd.scales.data_ptr(),
                                    m.V, E, self.tokens.data_ptr(), T, x.data_ptr(), st))
        t_kv = pos0 + T
        def mat(q8):  # the 16-bit rows of a Q8_0 matrix, in the reusable buffer
            return device.q8_dequant(q8, out=self.scratch[:q8.rows * q8.cols].view(
                q8.rows, q8.cols))

        for li, (ly, w) in enumerate(zip(m.layers, self.w)):
            if self.scratch is not None:
                w = dict(qkv=None, wo=None, gu=None, down=None, q8=w)
            h = self._norm(x, ly["attn_norm"], T)
            if self.scratch is not None:
                w["qkv"] = mat(w["q8"]["qkv"])
            device.gemm_qkv_rope(h, w["qkv"], pos, ch.cos, ch.sin, H=H, KV=KV,
                                 k_cache=ch.k_cache[li], v_cache=ch.v_cache[li],
                                 q_out=self.qrot[:T])
            att = device.prefill(self.qrot[:T], ch.k_cache[li][0, :t_kv],
                                 ch.v_cache[li][0, :t_kv], pos, out=self.att[:T])
            if self.weights == "q8":
                device.gemm_q8(att.view(T, qd), w["wo"], out=x, c_in=x)
                h = self._norm(x, ly["ffn_norm"], T)
                device.gemm_q8(h, w["gu"], out=self.act[:T], epilogue=device.GEMM_SWIGLU8)
                device.gemm_q8(self.act[:T], w["down"], out=x, c_in=x)
            elif self.weights == "q8_dequant":
                device.gemm(att.view(T, qd), mat(w["q8"]["wo"]), out=x, c_in=x)
                h = self._norm(x, ly["ffn_norm"], T)
                device.gemm(h, mat(w["q8"]["gu"]), out=self.act[:T], epilogue=device.GEMM_SWIGLU8)
                device.gemm(self.act[:T], mat(w["q8"]["down"]), out=x, c_in=x)
            else:
                device.gemm(att.view(T, qd), w["wo"], out=x, c_in=x)
                h = self._norm(x, ly["ffn_norm"], T)
                device.gemm(h, w["gu"], out=self.act[:T], epilogue=device.GEMM_SWIGLU)
                device.gemm(self.act[:T], w["down"], out=x, c_in=x)
        if not want_logits:
            return None
        m.output.gemv(x[T - 1], self.logits, mode=1, aux=m.out_norm, eps=m.eps, flags=PDL)
        return self.logits.cpu().numpy()
