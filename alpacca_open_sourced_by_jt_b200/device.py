"""Device-tensor API over libb2attn.so.

PyTorch is only the carrier here: tensors supply device pointers, the
current CUDA stream and (outside this module) allocation.  Every function
validates shapes/dtypes on the host, then makes one C-ABI call; nothing here
synchronises, so the calls can be captured into a CUDA graph as long as the
caller supplies `out` and `workspace` buffers (the library never allocates).
"""
from __future__ import annotations

import contextlib
import math

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def _code(dtype: torch.dtype) -> int:
    try:
        return _DT[dtype]
    except KeyError:
        raise _lib.B2AShapeError(_lib.ERR_DTYPE, f"unsupported dtype {dtype}") from None


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream=None):
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


@contextlib.contextmanager
def launch_flags(flags: int):
    """Launch mode of this thread's library calls inside the block
    (b2a_set_launch_flags).  With LAUNCH_PDL, RoPE + append, decode and the
    LSE combine start as programmatic dependents of the kernel before them;
    lengths, positions and the cache rows below each sequence's newest must
    be complete before that kernel starts (as in a captured decode step)."""
    lib = _lib.load()
    old = lib.b2a_set_launch_flags(int(flags))
    try:
        yield
    finally:
        lib.b2a_set_launch_flags(old)


def _need(cond: bool, msg: str):
    if not cond:
        raise _lib.B2AShapeError(_lib.ERR_SHAPE, msg)


def _cuda_contig(name: str, t: torch.Tensor):
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.is_contiguous(), f"{name} must be contiguous")


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------

def decode_split_rows(batch: int, n_kv: int, max_len: int, kv_dtype: torch.dtype) -> int:
    return int(_lib.load().b2a_decode_split_rows(batch, n_kv, max_len, _code(kv_dtype)))


def decode_workspace_bytes(batch: int, n_head: int, head_dim: int, max_len: int,
                           split_rows: int) -> int:
    return int(_lib.load().b2a_decode_workspace_bytes(batch, n_head, head_dim, max_len,
                                                      split_rows))


def decode_workspace(batch: int, n_head: int, head_dim: int, max_len: int, split_rows: int,
                     device) -> torch.Tensor:
    """Allocate (via torch) a workspace big enough for b2a_decode."""
    n = decode_workspace_bytes(batch, n_head, head_dim, max_len, split_rows)
    return torch.empty(max(n, 16), dtype=torch.uint8, device=device)


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
           *, scale: float | None = None, max_len: int | None = None, out=None, lse=None,
           workspace=None, split_rows: int = 0, stream=None) -> torch.Tensor:
    """Split-KV GQA decode.

    q (B, H, D) f32; k_cache/v_cache (B, n_ctx, KV, D) or (n_ctx, KV, D) for
    B == 1, dtype f32/f16/bf16 (sequence stride may exceed n_ctx*KV*D: pass a
    view whose stride(0) is the stride); lens (B,) int32 on the device.
    max_len bounds every lens entry (default n_ctx).  Returns out (B, H, D)
    f32; lse (B, H) f32 receives the natural-log log-sum-exp if given.
    """
    if k_cache.dim() == 3:
        k_cache = k_cache.unsqueeze(0)
        v_cache = v_cache.unsqueeze(0)
    _need(q.dim() == 3 and q.dtype == torch.float32 and q.is_cuda and q.is_contiguous(),
          "q must be a contiguous CUDA f32 tensor (B, H, D)")
    B, H, D = q.shape
    _need(k_cache.dim() == 4 and k_cache.shape == v_cache.shape, "k_cache/v_cache shape mismatch")
    _need(k_cache.dtype == v_cache.dtype, "k_cache/v_cache dtype mismatch")
    Bc, n_ctx, KV, Dc = k_cache.shape
    _need(Bc == B and Dc == D, f"cache {tuple(k_cache.shape)} does not match q {tuple(q.shape)}")
    _need(k_cache[0].is_contiguous() and v_cache[0].is_contiguous(),
          "each sequence's cache block must be contiguous")
    _need(k_cache.stride(0) == v_cache.stride(0), "k/v caches need the same sequence stride")
    _need(lens.dtype == torch.int32 and lens.is_cuda and lens.numel() == B,
          "lens must be a CUDA int32 tensor (B,)")
    seq_stride = k_cache.stride(0) if B > 1 else n_ctx * KV * D
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if max_len is None:
        max_len = n_ctx
    if split_rows <= 0:
        split_rows = decode_split_rows(B, KV, max_len, k_cache.dtype)
    if out is None:
        out = torch.empty((B, H, D), dtype=torch.float32, device=q.device)
    if workspace is None:
        workspace = decode_workspace(B, H, D, max_len, split_rows, q.device)
    if lse is not None:
        _need(lse.dtype == torch.float32 and lse.numel() == B * H, "lse must be f32 (B, H)")
    _lib.check(_lib.load().b2a_decode(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(lens), _ptr(out), _ptr(lse), _ptr(workspace),
        workspace.numel() * workspace.element_size(), B, H, KV, D, n_ctx, seq_stride,
        _code(k_cache.dtype), float(scale), int(max_len), int(split_rows), _stream(stream)))
    return out


def decode_sharded(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                   lens: torch.Tensor, peer_table: torch.Tensor, rank: int, world: int, *,
                   scale: float | None = None, max_len: int | None = None, out=None, lse=None,
                   workspace=None, split_rows: int = 0, stream=None) -> torch.Tensor:
    """Long-context decode with the KV rows sharded over `world` GPUs
    (b2a_decode_sharded): this rank's split-KV decode over its rows, then
    one kernel that pushes the rank's (o, lse) rows into every rank's
    exchange buffer over NVLink and merges all ranks' parts.  Arguments as
    in decode() for this rank's rows; peer_table is the int64 device tensor
    of the ranks' exchange-buffer addresses (longctx.PeerExchange).  Every
    rank must make the same call; the merged (B, H, D) f32 output is the
    same on every rank."""
    if k_shard.dim() == 3:
        k_shard = k_shard.unsqueeze(0)
        v_shard = v_shard.unsqueeze(0)
    _need(q.dim() == 3 and q.dtype == torch.float32 and q.is_cuda and q.is_contiguous(),
          "q must be a contiguous CUDA f32 tensor (B, H, D)")
    B, H, D = q.shape
    _need(k_shard.dim() == 4 and k_shard.shape == v_shard.shape, "k/v shard shape mismatch")
    _need(k_shard.dtype == v_shard.dtype, "k/v shard dtype mismatch")
    Bc, n_ctx, KV, Dc = k_shard.shape
    _need(Bc == B and Dc == D, f"shard {tuple(k_shard.shape)} does not match q {tuple(q.shape)}")
    _need(k_shard[0].is_contiguous() and v_shard[0].is_contiguous(),
          "each sequence's shard block must be contiguous")
    _need(k_shard.stride(0) == v_shard.stride(0), "k/v shards need the same sequence stride")
    _need(lens.dtype == torch.int32 and lens.is_cuda and lens.numel() == B,
          "lens must be a CUDA int32 tensor (B,)")
    _need(peer_table.dtype == torch.int64 and peer_table.is_cuda and
          peer_table.numel() == world, "peer_table must be a CUDA int64 tensor (world,)")
    seq_stride = k_shard.stride(0) if B > 1 else n_ctx * KV * D
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if max_len is None:
        max_len = n_ctx
    if split_rows <= 0:
        split_rows = decode_split_rows(B, KV, max_len, k_shard.dtype)
    if out is None:
        out = torch.empty((B, H, D), dtype=torch.float32, device=q.device)
    if workspace is None:
        workspace = decode_workspace(B, H, D, max_len, split_rows, q.device)
    if lse is not None:
        _need(lse.dtype == torch.float32 and lse.numel() == B * H, "lse must be f32 (B, H)")
    _lib.check(_lib.load().b2a_decode_sharded(
        _ptr(q), _ptr(k_shard), _ptr(v_shard), _ptr(lens), _ptr(out), _ptr(lse),
        _ptr(workspace), workspace.numel() * workspace.element_size(), B, H, KV, D, n_ctx,
        seq_stride, _code(k_shard.dtype), float(scale), int(max_len), int(split_rows),
        _ptr(peer_table), int(rank), int(world), _stream(stream)))
    return out


def lse_combine(o_parts: torch.Tensor, lse_parts: torch.Tensor, *, out=None, lse=None,
                stream=None) -> torch.Tensor:
    """Merge G normalised partial outputs (G, R, D) by their lse (G, R).

    Each part must be contiguous ((R, D) and (R,)); the parts may sit at any
    stride from one another (e.g. views into one gathered buffer)."""
    G, R, D = o_parts.shape
    _need(lse_parts.shape == (G, R), "lse_parts must be (G, R)")
    _need(o_parts.is_cuda and lse_parts.is_cuda, "parts must be CUDA tensors")
    _need(o_parts.stride(2) == 1 and o_parts.stride(1) == D and lse_parts.stride(1) == 1,
          "each part must be contiguous")
    _need(o_parts.dtype == lse_parts.dtype == torch.float32, "parts must be f32")
    if out is None:
        out = torch.empty((R, D), dtype=torch.float32, device=o_parts.device)
    _lib.check(_lib.load().b2a_lse_combine(_ptr(o_parts), o_parts.stride(0), _ptr(lse_parts),
                                           lse_parts.stride(0), G, R, D, _ptr(out), _ptr(lse),
                                           _stream(stream)))
    return out


# ---------------------------------------------------------------------------
# prefill
# ---------------------------------------------------------------------------

def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor, *,
            scale: float | None = None, window: int = 0, kv_start: int = 0,
            out_dtype: torch.dtype | None = None, out=None, stream=None) -> torch.Tensor:
    """Causal flash prefill.

    q (T, H, D); k, v (t_kv, KV, D) (the cache rows kv_start..kv_start+t_kv-1),
    all of one dtype; positions (T,) int32 absolute positions.  f16/bf16
    inputs run the tcgen05 tensor-core kernels (D in {64, 128, 256}, fp32
    accumulation); f32 inputs run the fp32 CUDA-core kernel (D a multiple of
    4 up to 256), which keeps the reference's fp32 precision.  A query row
    with no visible key gets the mean of the t_kv value rows, as the
    reference's NumPy path does.  Returns (T, H, D) in out_dtype (default
    q.dtype)."""
    for n_, t_ in (("q", q), ("k", k), ("v", v), ("positions", positions)):
        _cuda_contig(n_, t_)
    _need(q.dim() == 3 and k.dim() == 3 and k.shape == v.shape, "q (T,H,D), k/v (t_kv,KV,D)")
    _need(q.dtype == k.dtype == v.dtype and q.dtype in (torch.float32, torch.float16,
                                                         torch.bfloat16),
          "q/k/v must share dtype f32, f16 or bf16")
    T, H, D = q.shape
    t_kv, KV, Dk = k.shape
    _need(Dk == D, "head_dim mismatch")
    _need(positions.dtype == torch.int32 and positions.numel() == T, "positions int32 (T,)")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((T, H, D), dtype=out_dtype or q.dtype, device=q.device)
    _lib.check(_lib.load().b2a_prefill(
        _ptr(q), _ptr(k), _ptr(v), _ptr(positions), _ptr(out), T, t_kv, H, KV, D,
        _code(q.dtype), _code(out.dtype), float(scale), int(window), int(kv_start),
        _stream(stream)))
    return out


# ---------------------------------------------------------------------------
# RoPE + append
# ---------------------------------------------------------------------------

_STYLE = {"norm": _lib.ROPE_NORM, "neox": _lib.ROPE_NEOX}


def rope_tables(n_ctx: int, n_rot: int, rope_base: float, freq_scale: float = 1.0,
                device=None):
    """The cos/sin tables (n_ctx, n_rot/2) float32 that rope_append reads.

    Built once per model on the host, in float32 as the reference's model
    set-up builds them (alpaccaroo/model.py:318-323 for inv_freq =
    freq_scale * base^(-2i/n_rot) over a float32 index, :871-875 for
    theta = position * inv_freq and its cos/sin), so the rotations agree
    with the reference bit for bit; then copied to `device` (default: the
    current CUDA device).  Set-up only, not part of the per-token path."""
    import numpy as np
    _need(n_rot > 0 and n_rot % 2 == 0, "n_rot must be even and positive")
    f32 = np.float32
    idx = np.arange(n_rot // 2, dtype=f32)
    inv = f32(freq_scale) * np.power(f32(rope_base), idx * f32(-2.0) / f32(n_rot))
    theta = np.arange(n_ctx, dtype=f32)[:, None] * inv[None, :]
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    return (torch.from_numpy(np.cos(theta)).to(dev), torch.from_numpy(np.sin(theta)).to(dev))


def rope_append(q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None,
                positions: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor, *,
                k_cache=None, v_cache=None, n_rot: int | None = None, style: str = "norm",
                per_sequence: bool = False, q_out=None, bq=None, bk=None, bv=None,
                stream=None):
    """Fused bias + RoPE + KV append for n tokens.

    q (n, H, D) f32 (rotated in place unless q_out is given); k, v (n, KV, D)
    f32 rows or None (rope-only); positions (n,) int32; caches (S, n_ctx, KV,
    D) or (n_ctx, KV, D).  per_sequence=True puts token i in sequence i
    (batched decode), else all tokens in sequence 0 (a prefill chunk).
    Returns the tensor holding the rotated q."""
    _need(q.dim() == 3 and q.dtype == torch.float32 and q.is_cuda, "q must be CUDA f32 (n,H,D)")
    n, H, D = q.shape
    _need(q.stride(2) == 1 and q.stride(1) == D, "q rows must be contiguous per token")
    _need(positions.dtype == torch.int32 and positions.is_cuda and positions.numel() == n,
          "positions int32 (n,)")
    _cuda_contig("cos_tab", cos_tab)
    _cuda_contig("sin_tab", sin_tab)
    if n_rot is None:
        n_rot = 2 * cos_tab.shape[1]
    _need(cos_tab.shape[1] * 2 == n_rot, "cos table width must be n_rot/2")
    KV, seq_stride, n_ctx, kv_dt = 0, 0, cos_tab.shape[0], _lib.F32
    ks = vs = 0
    if k is not None:
        _need(k_cache is not None and v_cache is not None, "k/v given without caches")
        if k_cache.dim() == 3:
            k_cache, v_cache = k_cache.unsqueeze(0), v_cache.unsqueeze(0)
        _need(k_cache.shape == v_cache.shape and k_cache.dtype == v_cache.dtype, "cache mismatch")
        _, n_ctx, KV, Dc = k_cache.shape
        _need(Dc == D and k.shape == (n, KV, D) and v.shape == (n, KV, D), "k/v shape")
        _need(k.stride(2) == 1 and v.stride(2) == 1 and k.stride(1) == D and v.stride(1) == D,
              "k/v rows must be contiguous per token")
        seq_stride = k_cache.stride(0)
        kv_dt = _code(k_cache.dtype)
        ks, vs = k.stride(0), v.stride(0)
    qo_dt = _lib.F32
    if q_out is not None:
        _cuda_contig("q_out", q_out)
        qo_dt = _code(q_out.dtype)
    _lib.check(_lib.load().b2a_rope_append(
        _ptr(q), q.stride(0), _ptr(k), ks, _ptr(v), vs, _ptr(bq), _ptr(bk), _ptr(bv),
        _ptr(cos_tab), _ptr(sin_tab), cos_tab.shape[0], _ptr(positions), int(per_sequence),
        _ptr(k_cache), _ptr(v_cache), seq_stride, n_ctx, kv_dt, _ptr(q_out), qo_dt, n, H, KV, D,
        int(n_rot), _STYLE[style], _stream(stream)))
    return q if q_out is None else q_out


def imrope_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lanes: torch.Tensor,
                  positions: torch.Tensor, sections, *, k_cache, v_cache, freq_base: float,
                  freq_scale: float = 1.0, per_sequence: bool = False, q_out=None,
                  stream=None) -> torch.Tensor:
    """Qwen35 IMROPE of q/k plus KV append.  lanes (n, 4) int32 position
    lanes; sections 4 ints; positions (n,) cache rows.  Returns q_out."""
    _need(q.dim() == 3 and q.dtype == torch.float32 and q.is_cuda, "q must be CUDA f32 (n,H,D)")
    n, H, D = q.shape
    if k_cache.dim() == 3:
        k_cache, v_cache = k_cache.unsqueeze(0), v_cache.unsqueeze(0)
    _, n_ctx, KV, _ = k_cache.shape
    for n_, t_ in (("q", q), ("k", k), ("v", v), ("lanes", lanes), ("positions", positions)):
        _cuda_contig(n_, t_)
    _need(lanes.dtype == torch.int32 and lanes.shape == (n, 4), "lanes int32 (n, 4)")
    if q_out is None:
        q_out = torch.empty_like(q)
    import ctypes
    sec = (ctypes.c_int * 4)(*[int(s) for s in sections])
    _lib.check(_lib.load().b2a_imrope_append(
        _ptr(q), H * D, _ptr(k), KV * D, _ptr(v), KV * D, _ptr(lanes), sec, float(freq_base),
        float(freq_scale), _ptr(positions), int(per_sequence), _ptr(k_cache), _ptr(v_cache),
        k_cache.stride(0), n_ctx, _code(k_cache.dtype), _ptr(q_out), _code(q_out.dtype), n, H,
        KV, D, _stream(stream)))
    return q_out


GEMM_STORE, GEMM_SWIGLU, GEMM_SWIGLU8 = 0, 1, 2


def gemm(a: torch.Tensor, w: torch.Tensor, *, out=None, out_dtype=torch.float32, c_in=None,
         epilogue: int = GEMM_STORE, stream=None) -> torch.Tensor:
    """out = a . w^T (+ c_in) on the tcgen05 tensor cores (b2a_gemm).

    a (M, K) and w (N, K) 16-bit with unit stride along K; c_in f32 (M, N)
    or None (may be out itself, for an in-place residual add).  With
    GEMM_SWIGLU, w's rows come in 256-row groups of 128 gate rows and the
    matching 128 up rows and out is silu(gate) * up, (M, N / 2); GEMM_SWIGLU8
    takes 16-row groups of 8 gate then 8 up rows (the decode GEMV's layout)."""
    _need(a.dim() == 2 and w.dim() == 2 and a.shape[1] == w.shape[1], "a (M,K), w (N,K)")
    _need(a.dtype == w.dtype and a.dtype in (torch.float16, torch.bfloat16), "16-bit a and w")
    _need(a.stride(1) == 1 and w.stride(1) == 1, "a and w need unit stride along K")
    M, K = a.shape
    N = w.shape[0]
    cols = N // 2 if epilogue in (GEMM_SWIGLU, GEMM_SWIGLU8) else N
    if out is None:
        out = torch.empty((M, cols), dtype=out_dtype, device=a.device)
    _need(out.dim() == 2 and out.shape == (M, cols) and out.stride(1) == 1, "out (M, cols)")
    if c_in is not None:
        _need(c_in.dtype == torch.float32 and c_in.shape == (M, N) and c_in.stride(1) == 1,
              "c_in f32 (M, N)")
    _lib.check(_lib.load().b2a_gemm(
        _ptr(a), a.stride(0), _ptr(w), w.stride(0), _code(a.dtype), _ptr(c_in),
        0 if c_in is None else c_in.stride(0), _ptr(out), out.stride(0), _code(out.dtype), M, N,
        K, int(epilogue), _stream(stream)))
    return out


def _q8_parts(q8):
    """(codes, scales) of a Q8_0 matrix: a Q8Matrix or a (codes, scales) pair,
    codes int8 (N, K) and scales f16 (N, K/32), each with unit stride along K."""
    codes, scales = (q8.codes, q8.scales) if hasattr(q8, "codes") else q8
    _need(codes.dtype == torch.int8 and codes.dim() == 2 and codes.stride(1) == 1 and codes.is_cuda,
          "codes int8 (N, K) on the device, unit stride along K")
    N, K = codes.shape
    _need(scales.dtype == torch.float16 and scales.shape == (N, K // 32) and scales.stride(1) == 1
          and scales.is_cuda, "scales f16 (N, K/32) on the device")
    return codes, scales


def q8_dequant(q8, dtype=torch.float16, *, out=None, stream=None) -> torch.Tensor:
    """Q8_0 matrix (a Q8Matrix or (codes, scales)) to 16-bit rows on the device
    (b2a_q8_dequant): d * code rounded once to dtype, the values gemm_q8
    feeds the tensor cores.  out, if given, is a (rows, cols) view with unit
    stride along the columns."""
    codes, scales = _q8_parts(q8)
    N, K = codes.shape
    if out is None:
        out = torch.empty((N, K), dtype=dtype, device=codes.device)
    _need(out.dtype in (torch.float16, torch.bfloat16) and out.shape == (N, K) and
          out.stride(1) == 1, "out (rows, cols) f16 or bf16")
    _lib.check(_lib.load().b2a_q8_dequant(
        _ptr(codes), codes.stride(0), _ptr(scales), scales.stride(0), _ptr(out), out.stride(0),
        _code(out.dtype), N, K, _stream(stream)))
    return out


def gemm_q8(a: torch.Tensor, q8, *, out=None, out_dtype=torch.float32, c_in=None,
            epilogue: int = GEMM_STORE, stream=None) -> torch.Tensor:
    """gemm() with Q8_0 weights decoded inside the kernel (b2a_gemm_q8): the
    result equals gemm(a, d * code rounded to a's dtype).  q8 is a Q8Matrix
    or (codes int8 (N, K), scales f16 (N, K/32)); a (M, K) f16 or bf16.
    GEMM_SWIGLU8 takes the decode GEMV's gate/up layout (16-row groups of 8
    gate rows then their 8 up rows) and writes silu(gate) * up, (M, N / 2)."""
    codes, scales = _q8_parts(q8)
    _need(a.dim() == 2 and a.shape[1] == codes.shape[1], "a (M, K), codes (N, K)")
    _need(a.dtype in (torch.float16, torch.bfloat16) and a.stride(1) == 1,
          "a f16 or bf16 with unit stride along K")
    M, K = a.shape
    N = codes.shape[0]
    cols = N // 2 if epilogue in (GEMM_SWIGLU, GEMM_SWIGLU8) else N
    if out is None:
        out = torch.empty((M, cols), dtype=out_dtype, device=a.device)
    _need(out.dim() == 2 and out.shape == (M, cols) and out.stride(1) == 1, "out (M, cols)")
    if c_in is not None:
        _need(c_in.dtype == torch.float32 and c_in.shape == (M, N) and c_in.stride(1) == 1,
              "c_in f32 (M, N)")
    _lib.check(_lib.load().b2a_gemm_q8(
        _ptr(a), a.stride(0), _ptr(codes), codes.stride(0), _ptr(scales), scales.stride(0),
        _code(a.dtype), _ptr(c_in), 0 if c_in is None else c_in.stride(0), _ptr(out),
        out.stride(0), _code(out.dtype), M, N, K, int(epilogue), _stream(stream)))
    return out


def gemm_qkv_rope(a: torch.Tensor, w: torch.Tensor, positions: torch.Tensor,
                  cos_tab: torch.Tensor, sin_tab: torch.Tensor, *, H: int, KV: int, k_cache,
                  v_cache, q_out, stream=None) -> torch.Tensor:
    """A chunk's QKV projection with RoPE and the K/V append in the GEMM
    epilogue (b2a_gemm_qkv_rope): q = (a . w^T)[:, :H*D] rotated into q_out
    (M, H, D); k rotated and v into the caches' rows `positions`.

    a (M, K) and w ((H + 2*KV)*D, K) 16-bit, unit stride along K; caches
    (n_ctx, KV, D) or (1, n_ctx, KV, D) of a's dtype; cos/sin f32 (rows,
    D/2): norm-style RoPE over the whole head.  The same result as gemm()
    to f32 followed by rope_append(q_out=...).  w may also be Q8_0 weights
    (a Q8Matrix or (codes, scales), as gemm_q8 takes them)."""
    q8 = not isinstance(w, torch.Tensor)
    if q8:  # Q8_0 weights (a Q8Matrix or (codes, scales)): b2a_gemm_qkv_rope_q8
        codes, scales = _q8_parts(w)
        w = codes
        _need(a.dim() == 2 and a.shape[1] == codes.shape[1], "a (M,K), codes (N,K)")
        _need(a.dtype in (torch.float16, torch.bfloat16) and a.stride(1) == 1,
              "a f16 or bf16 with unit stride along K")
    else:
        _need(a.dim() == 2 and w.dim() == 2 and a.shape[1] == w.shape[1], "a (M,K), w (N,K)")
        _need(a.dtype == w.dtype and a.dtype in (torch.float16, torch.bfloat16),
              "16-bit a and w")
        _need(a.stride(1) == 1 and w.stride(1) == 1, "a and w need unit stride along K")
    M, K = a.shape
    if k_cache.dim() == 4:
        _need(k_cache.shape[0] == 1 and v_cache.shape[0] == 1, "one sequence's cache")
        k_cache, v_cache = k_cache[0], v_cache[0]
    _need(k_cache.shape == v_cache.shape and k_cache.dim() == 3, "caches (n_ctx, KV, D)")
    n_ctx, kv_, D = k_cache.shape
    _need(kv_ == KV and w.shape[0] == (H + 2 * KV) * D, "w rows must be (H + 2*KV) * D")
    _need(k_cache.dtype == a.dtype and v_cache.dtype == a.dtype and q_out.dtype == a.dtype,
          "caches and q_out in a's dtype")
    for n_, t_ in (("k_cache", k_cache), ("v_cache", v_cache), ("q_out", q_out),
                   ("positions", positions), ("cos_tab", cos_tab), ("sin_tab", sin_tab)):
        _cuda_contig(n_, t_)
    _need(q_out.numel() == M * H * D, "q_out (M, H, D)")
    _need(positions.dtype == torch.int32 and positions.numel() == M, "positions int32 (M,)")
    _need(cos_tab.shape == sin_tab.shape and cos_tab.shape[1] * 2 == D,
          "cos/sin tables (rows, D/2)")
    if q8:
        _lib.check(_lib.load().b2a_gemm_qkv_rope_q8(
            _ptr(a), a.stride(0), _ptr(codes), codes.stride(0), _ptr(scales), scales.stride(0),
            _code(a.dtype), M, K, _ptr(positions), _ptr(cos_tab), _ptr(sin_tab),
            cos_tab.shape[0], H, KV, D, _ptr(q_out), _ptr(k_cache), _ptr(v_cache), n_ctx,
            _stream(stream)))
        return q_out
    _lib.check(_lib.load().b2a_gemm_qkv_rope(
        _ptr(a), a.stride(0), _ptr(w), w.stride(0), _code(a.dtype), M, K, _ptr(positions),
        _ptr(cos_tab), _ptr(sin_tab), cos_tab.shape[0], H, KV, D, _ptr(q_out), _ptr(k_cache),
        _ptr(v_cache), n_ctx, _stream(stream)))
    return q_out
