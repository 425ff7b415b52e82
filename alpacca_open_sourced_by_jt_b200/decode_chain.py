"""Whole-token llama decode on the device, replayed as one CUDA graph.

The reference's GPU decode chain (alpaccaroo/cuda.py:1682-2159,
DecodeChain.step at :2082-2159) runs a token as a sequence of Numba-CUDA
launches over Q8_0 weights in VRAM; Model._forward_np (model.py:1374-1487)
is the same computation on the host.  Here a token is one CUDA graph of
98 kernel launches: the embedding gather, 6 per layer, the LM head:

  embed       one dequantized Q8_0 embedding row          (b2a_q8_embed)
  per layer:
    qkv     = Wqkv . RMSNorm(x)          (fused RMSNorm; Wq|Wk|Wv rows), with
              RoPE of q and k and the k/v rows stored at the position in
              the epilogue                                 b2a_q8_gemv_qkv_rope
    att     = GQA decode over positions 0..pos             b2a_decode (split + combine)
    x      += Wo . att                   (residual in the epilogue)      b2a_q8_gemv
    act     = SwiGLU(Wgu . RMSNorm(x))   (gate/up rows interleaved, the
                                          SwiGLU of each row pair in the
                                          epilogue)                      b2a_q8_gemv
    x      += Wdown . act                                                b2a_q8_gemv
  logits    = Woutput . RMSNorm(x)                                       b2a_q8_gemv

with the token id and position copied from pinned host memory at the start
of the graph and the logits copied back at its end.  The matrix-vector
products are programmatic dependents of the kernel before them: each
starts loading its weights while that kernel finishes (the weights do not
depend on the activations).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib, device

_Q8_0 = np.dtype([("d", "<f2"), ("qs", "i1", 32)])
ACCUMULATE, SWIGLU_OUT, PDL = 1, 2, 4  # b2a_q8_gemv flags


def _fragment_order():
    """Byte order of a 16-row x 32-code tile as b2a_q8_gemv reads it: lane t
    (g = t/4, q = t%4) holds the A fragments of the block's two m16n8k16
    MMAs, registers a0..a3 = (row g | g+8) x (codes 2q, 2q+1 | 2q+8, 2q+9),
    codes + 16 for the second MMA."""
    rows, ks = [], []
    for t in range(32):
        g, q = t // 4, t % 4
        for j in range(16):
            m, reg, half = j // 8, (j % 8) // 2, j % 2
            rows.append(g + (8 if reg in (1, 3) else 0))
            ks.append(16 * m + 2 * q + half + (8 if reg in (2, 3) else 0))
    return rows, ks


_FRAG_ROWS, _FRAG_KS = _fragment_order()
_SCALE_ORDER = [r for g in range(8) for r in (g, g + 8)]


class Q8Matrix:
    """A Q8_0 matrix on the device: codes int8 (rows, cols) and scales f16
    (rows, cols/32) row-major (the embedding gather and dequantized copies
    read these), and, built on first use, the tiles b2a_q8_gemv streams:
    rows padded to 16, 512-byte tiles of 16 rows x one 32-code block in MMA
    fragment order, scales 16 per tile ordered (row 0, 8, 1, 9, ...)."""

    def __init__(self, codes: torch.Tensor, scales: torch.Tensor):
        if codes.dtype != torch.int8 or scales.dtype != torch.float16 or codes.dim() != 2:
            raise _lib.B2AShapeError(_lib.ERR_DTYPE, "codes int8 (rows, cols), scales f16")
        self.rows, self.cols = codes.shape
        if self.cols % 32 or tuple(scales.shape) != (self.rows, self.cols // 32):
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, "scales must be (rows, cols / 32)")
        self.codes, self.scales = codes.contiguous(), scales.contiguous()
        self._tiles = None

    def tiles(self):
        """(tiles int8 (groups, nb, 512), tile scales f16 (groups, nb, 16))."""
        if self._tiles is None:
            R, C = self.rows, self.cols
            nb, rg = C // 32, (R + 15) // 16
            codes, scales = self.codes, self.scales
            if rg * 16 != R:
                pad = rg * 16 - R
                codes = torch.cat([codes, codes.new_zeros((pad, C))])
                scales = torch.cat([scales, scales.new_zeros((pad, nb))])
            dev = codes.device
            t = codes.view(rg, 16, nb, 32).permute(0, 2, 1, 3)
            tiles = t[:, :, torch.tensor(_FRAG_ROWS, device=dev),
                      torch.tensor(_FRAG_KS, device=dev)].contiguous()
            ts = scales.view(rg, 16, nb).permute(0, 2, 1)[:, :, torch.tensor(_SCALE_ORDER,
                                                                             device=dev)]
            self._tiles = (tiles, ts.contiguous())
        return self._tiles

    @classmethod
    def from_q8_0(cls, data: bytes, rows: int, cols: int, dev) -> "Q8Matrix":
        """From GGUF Q8_0 records (an f16 scale then 32 int8 codes each)."""
        rec = np.frombuffer(data, dtype=_Q8_0)
        if rec.size * 32 != rows * cols:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, f"{len(data)} bytes for {rows}x{cols} Q8_0")
        codes = torch.from_numpy(np.array(rec["qs"]).reshape(rows, cols))
        scales = torch.from_numpy(np.array(rec["d"]).reshape(rows, cols // 32))
        return cls(codes.to(dev), scales.to(dev))

    @classmethod
    def quantize(cls, w: torch.Tensor) -> "Q8Matrix":
        """Q8_0-encode an f32 (rows, cols) device matrix with the reference's
        rule (quants.py:898-909: d = amax/127, codes = round-half-even(w/d)),
        evaluated in f32 on the device (used for synthetic weights)."""
        rows, cols = w.shape
        b = w.reshape(rows, cols // 32, 32)
        d = b.abs().amax(dim=2) / 127.0
        inv = torch.where(d != 0, 1.0 / torch.where(d != 0, d, torch.ones_like(d)),
                          torch.zeros_like(d))
        q = torch.round(b * inv[:, :, None]).clamp_(-128, 127).to(torch.int8)
        return cls(q.reshape(rows, cols), d.to(torch.float16))

    @staticmethod
    def stack(mats) -> "Q8Matrix":
        """Rows of several matrices with the same columns, concatenated."""
        return Q8Matrix(torch.cat([m.codes for m in mats]), torch.cat([m.scales for m in mats]))

    @staticmethod
    def interleave(a: "Q8Matrix", b: "Q8Matrix") -> "Q8Matrix":
        """Rows a0..a7, b0..b7, a8..a15, b8..b15, ... (the FFN's gate and up
        rows in one 16-row group, so the GEMV's SWIGLU_OUT epilogue finds
        gate i and up i in the same lane).  Row counts a multiple of 8."""
        if a.rows % 8 or a.rows != b.rows or a.cols != b.cols:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, "interleave: equal shapes, rows % 8 == 0")
        n, c, nb = a.rows // 8, a.cols, a.cols // 32
        return Q8Matrix(torch.stack((a.codes.view(n, 8, c), b.codes.view(n, 8, c)), 1)
                        .reshape(-1, c),
                        torch.stack((a.scales.view(n, 8, nb), b.scales.view(n, 8, nb)), 1)
                        .reshape(-1, nb))

    def nbytes(self) -> int:
        """Bytes a GEMV streams: the codes and scales of every row."""
        return self.codes.numel() + self.scales.numel() * 2

    def gemv(self, x: torch.Tensor, out: torch.Tensor, *, mode: int = 0, aux=None,
             eps: float = 0.0, flags: int = 0, stream=None) -> torch.Tensor:
        """out = self . xin (mode 0: x, 1: RMSNorm(x, aux, eps), 2: SwiGLU of
        x's two halves); flags ACCUMULATE / SWIGLU_OUT / PDL (b2a_q8_gemv)."""
        tiles, ts = self.tiles()
        _lib.check(_lib.load().b2a_q8_gemv(
            tiles.data_ptr(), ts.data_ptr(), self.rows, self.cols, x.data_ptr(),
            None if aux is None else aux.data_ptr(), mode, float(eps), out.data_ptr(),
            int(flags), device._stream(stream)))
        return out


    def gemv_qkv_rope(self, x: torch.Tensor, norm_w: torch.Tensor, eps: float, q_out, cos_tab,
                      sin_tab, pos: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      H: int, KV: int, D: int, *, flags: int = 0, stream=None):
        """This matrix as a layer's [q; k; v] projection of RMSNorm(x), with
        RoPE (norm style) and the K/V append at position *pos fused into its
        epilogue (b2a_q8_gemv_qkv_rope): rotated q into q_out, k and v into
        the caches' row pos."""
        if self.rows != (H + 2 * KV) * D:
            raise _lib.B2AShapeError(_lib.ERR_SHAPE, f"{self.rows} rows for H={H} KV={KV} D={D}")
        tiles, ts = self.tiles()
        _lib.check(_lib.load().b2a_q8_gemv_qkv_rope(
            tiles.data_ptr(), ts.data_ptr(), self.cols, x.data_ptr(), norm_w.data_ptr(),
            float(eps), q_out.data_ptr(), cos_tab.data_ptr(), sin_tab.data_ptr(),
            cos_tab.shape[0], pos.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
            device._code(k_cache.dtype), k_cache.shape[-3], H, KV, D, int(flags),
            device._stream(stream)))
        return q_out


class LlamaQ8:
    """Weights of a llama-architecture model with Q8_0 matrices, on the device."""

    def __init__(self, *, n_embd, n_head, n_kv, head_dim, n_ff, n_vocab, rms_eps, rope_base,
                 layers, tok_embd: Q8Matrix, out_norm, output: Q8Matrix, dev):
        self.E, self.H, self.KV, self.D, self.F, self.V = (int(n_embd), int(n_head), int(n_kv),
                                                          int(head_dim), int(n_ff), int(n_vocab))
        self.eps, self.rope_base = float(rms_eps), float(rope_base)
        self.layers, self.tok_embd, self.output = layers, tok_embd, output
        self.out_norm = torch.as_tensor(out_norm, dtype=torch.float32).to(dev).contiguous()
        self.device = dev

    @classmethod
    def from_spec(cls, spec: dict, dev) -> "LlamaQ8":
        """spec: hp values, per-layer dicts of Q8_0 bytes (wq, wk, wv, wo,
        w_gate, w_up, w_down) and f32 norms (attn_norm, ffn_norm), tok_embd,
        out_norm and output, as a GGUF loader would hand them over."""
        E, H, KV, D, F, V = (spec["n_embd"], spec["n_head"], spec["n_kv"], spec["head_dim"],
                             spec["n_ff"], spec["n_vocab"])
        q8 = lambda data, rows, cols: Q8Matrix.from_q8_0(data, rows, cols, dev)  # noqa: E731
        layers = []
        for ly in spec["layers"]:
            layers.append(dict(
                attn_norm=torch.as_tensor(ly["attn_norm"], dtype=torch.float32).to(dev),
                ffn_norm=torch.as_tensor(ly["ffn_norm"], dtype=torch.float32).to(dev),
                wqkv=Q8Matrix.stack([q8(ly["wq"], H * D, E), q8(ly["wk"], KV * D, E),
                                     q8(ly["wv"], KV * D, E)]),
                wo=q8(ly["wo"], E, H * D),
                wgu=Q8Matrix.interleave(q8(ly["w_gate"], F, E), q8(ly["w_up"], F, E)),
                w_down=q8(ly["w_down"], E, F)))
        return cls(n_embd=E, n_head=H, n_kv=KV, head_dim=D, n_ff=F, n_vocab=V,
                   rms_eps=spec["rms_eps"], rope_base=spec["rope_base"], layers=layers,
                   tok_embd=q8(spec["tok_embd"], V, E), out_norm=spec["out_norm"],
                   output=q8(spec["output"], V, E), dev=dev)

    @classmethod
    def random(cls, *, n_layer, n_embd, n_head, n_kv, head_dim, n_ff, n_vocab, rms_eps,
               rope_base, seed, dev, std=0.02) -> "LlamaQ8":
        """Random-init weights N(0, std), Q8_0-encoded on the device; norms 1."""
        g = torch.Generator(device=dev).manual_seed(seed)
        E, H, KV, D, F, V = n_embd, n_head, n_kv, head_dim, n_ff, n_vocab

        def mat(rows, cols):
            out = []
            step = max(1, (1 << 27) // cols)  # quantize in slices of <= 512 MB f32
            for r in range(0, rows, step):
                n = min(step, rows - r)
                out.append(Q8Matrix.quantize(
                    torch.randn((n, cols), generator=g, device=dev) * std))
            return Q8Matrix.stack(out) if len(out) > 1 else out[0]

        ones = torch.ones(E, dtype=torch.float32, device=dev)
        layers = [dict(attn_norm=ones.clone(), ffn_norm=ones.clone(),
                       wqkv=mat((H + 2 * KV) * D, E), wo=mat(E, H * D),
                       wgu=Q8Matrix.interleave(mat(F, E), mat(F, E)),
                       w_down=mat(E, F)) for _ in range(n_layer)]
        return cls(n_embd=E, n_head=H, n_kv=KV, head_dim=D, n_ff=F, n_vocab=V, rms_eps=rms_eps,
                   rope_base=rope_base, layers=layers, tok_embd=mat(V, E), out_norm=ones,
                   output=mat(V, E), dev=dev)

    def weight_bytes(self) -> int:
        n = self.tok_embd.nbytes() // self.V + self.output.nbytes()  # one embedding row
        for ly in self.layers:
            n += ly["wqkv"].nbytes() + ly["wo"].nbytes() + ly["wgu"].nbytes() + \
                ly["w_down"].nbytes() + 2 * self.E * 4
        return n + self.E * 4


class DecodeChain:
    """A KV cache (kv_dtype, n_ctx rows per layer) and the captured token step
    for one sequence.  chain(token, pos) runs the token at cache row pos and
    returns the pinned f32 logits (valid until the next call).  Building the
    chain runs one eager warm-up step at position 0 (writing cache row 0,
    which the first real token overwrites) before the capture."""

    def __init__(self, model: LlamaQ8, n_ctx: int, kv_dtype: torch.dtype = torch.float16):
        _lib.load()
        m = model
        dev = m.device
        self.m, self.n_ctx = m, int(n_ctx)
        self.k_cache = [torch.zeros((1, n_ctx, m.KV, m.D), dtype=kv_dtype, device=dev)
                        for _ in m.layers]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self.cos, self.sin = device.rope_tables(n_ctx, m.D, m.rope_base, device=dev)
        self.x = torch.zeros(m.E, dtype=torch.float32, device=dev)
        self.qkv = torch.zeros((m.H + 2 * m.KV) * m.D, dtype=torch.float32, device=dev)
        self.att = torch.zeros((1, m.H, m.D), dtype=torch.float32, device=dev)
        self.act = torch.zeros(m.F, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(m.V, dtype=torch.float32, device=dev)
        self._h_i = torch.zeros(3, dtype=torch.int32).pin_memory()  # token, pos, pos + 1
        self._h_i_np = self._h_i.numpy()
        self._d_i = torch.zeros(3, dtype=torch.int32, device=dev)
        self.h_logits = torch.zeros(m.V, dtype=torch.float32).pin_memory()
        self._split = device.decode_split_rows(1, m.KV, n_ctx, kv_dtype)
        self._ws = device.decode_workspace(1, m.H, m.D, n_ctx, self._split, dev)
        self._h_i_np[:] = (0, 0, 1)
        self._body()  # eager warm-up: kernel set-up stays out of the capture
        torch.cuda.synchronize(dev)
        _lib.raise_device_error()
        self._stream = torch.cuda.Stream(device=dev)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=self._stream):
            self._body()
        self.launches = 2 + 6 * len(m.layers)  # kernels per token

    def _body(self):
        m = self.m
        qd, kd = m.H * m.D, m.KV * m.D
        lib = _lib.load()
        st = device._stream(None)
        self._d_i.copy_(self._h_i, non_blocking=True)
        _lib.check(lib.b2a_q8_embed(m.tok_embd.codes.data_ptr(), m.tok_embd.scales.data_ptr(),
                                    m.V, m.E, self._d_i.data_ptr(), 1, self.x.data_ptr(), st))
        q = self.qkv[:qd].view(1, m.H, m.D)
        k = self.qkv[qd:qd + kd].view(1, m.KV, m.D)
        v = self.qkv[qd + kd:].view(1, m.KV, m.D)
        pos, lens = self._d_i[1:2], self._d_i[2:3]
        for li, ly in enumerate(m.layers):
            # QKV with the attention norm in front and RoPE + the K/V append
            # in its epilogue (the position comes from the host copy at the
            # head of the graph)
            ly["wqkv"].gemv_qkv_rope(self.x, ly["attn_norm"], m.eps, self.qkv, self.cos,
                                     self.sin, pos, self.k_cache[li], self.v_cache[li], m.H,
                                     m.KV, m.D, flags=PDL)
            # the decode (and its combine) as programmatic dependents: the
            # split CTAs stream the cache rows below the newest while the QKV
            # GEMV, latency-bound, still runs; they read q and the new row
            # after it completes (the length comes from the host copy above)
            with device.launch_flags(_lib.LAUNCH_PDL):
                device.decode(q, self.k_cache[li], self.v_cache[li], lens, max_len=self.n_ctx,
                              out=self.att, workspace=self._ws, split_rows=self._split)
            ly["wo"].gemv(self.att, self.x, flags=ACCUMULATE | PDL)
            ly["wgu"].gemv(self.x, self.act, mode=1, aux=ly["ffn_norm"], eps=m.eps,
                           flags=SWIGLU_OUT | PDL)
            ly["w_down"].gemv(self.act, self.x, flags=ACCUMULATE | PDL)
        m.output.gemv(self.x, self.logits, mode=1, aux=m.out_norm, eps=m.eps, flags=PDL)
        self.h_logits.copy_(self.logits, non_blocking=True)

    def __call__(self, token: int, pos: int) -> torch.Tensor:
        if not 0 <= pos < self.n_ctx:
            raise _lib.B2AError(_lib.ERR_POSITION, f"position {pos} outside [0, {self.n_ctx})")
        if not 0 <= token < self.m.V:
            raise _lib.B2AError(_lib.ERR_ARG, f"token {token} outside [0, {self.m.V})")
        self._h_i_np[:] = (token, pos, pos + 1)
        self._graph.replay()
        torch.cuda.current_stream().synchronize()
        return self.h_logits
