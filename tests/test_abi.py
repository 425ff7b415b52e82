"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/b2attn.h declares, and rejects bad arguments on the host with the
documented status codes (these returns happen before any CUDA call)."""
import ctypes
import os
import re

import pytest

from alpacca_open_sourced_by_jt_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "b2attn.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2a_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(n for n, _, _ in _lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_version(lib):
    assert lib.b2a_version() == 1


def test_workspace_and_split_helpers(lib):
    sr = lib.b2a_decode_split_rows(16, 8, 32768, _lib.BF16)
    assert sr % 64 == 0 and 256 <= sr <= 8192
    # every sequence of max_len keeps at least 4 splits, and no split is under 256 rows
    for args in ((16, 8, 32768), (64, 8, 8192), (4, 8, 131072), (1, 8, 4096), (2, 2, 512)):
        s = lib.b2a_decode_split_rows(*args, _lib.BF16)
        assert s % 64 == 0 and 256 <= s <= 8192
        assert s == 256 or 4 * s <= args[2]
    n_split = -(-32768 // sr)
    ws = lib.b2a_decode_workspace_bytes(16, 32, 128, 32768, sr)
    assert ws >= 16 * 32 * n_split * (128 + 2) * 4
    assert lib.b2a_decode_workspace_bytes(0, 32, 128, 1, 64) == 0


def _decode(lib, **kw):
    args = dict(q=1 << 20, k=1 << 20, v=1 << 20, lens=1 << 20, out=1 << 20, lse=None,
                ws=1 << 20, ws_bytes=1 << 30, B=1, H=32, KV=8, D=128, n_ctx=1024, seq_stride=0,
                dt=_lib.BF16, scale=0.088, max_len=1024, split=0, stream=None)
    args.update(kw)
    return lib.b2a_decode(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), _lib.ERR_ARG),
    (dict(B=0), _lib.ERR_ARG),
    (dict(H=30), _lib.ERR_SHAPE),
    (dict(H=8 * 17), _lib.ERR_UNSUPPORTED),
    (dict(max_len=2048), _lib.ERR_SHAPE),
    (dict(dt=7), _lib.ERR_DTYPE),
    (dict(scale=-1.0), _lib.ERR_ARG),
    (dict(split=100), _lib.ERR_ARG),
    (dict(ws_bytes=16), _lib.ERR_WORKSPACE),
    (dict(B=2, seq_stride=5), _lib.ERR_SHAPE),
    (dict(q=(1 << 20) + 4), _lib.ERR_ALIGN),
    (dict(D=96), _lib.ERR_UNSUPPORTED),
])
def test_decode_rejects_bad_arguments(lib, kw, code):
    assert _decode(lib, **kw) == code
    assert _lib.last_error()


def test_prefill_rejects_bad_arguments(lib):
    p = 1 << 20
    assert lib.b2a_prefill(None, p, p, p, p, 8, 8, 4, 2, 64, _lib.BF16, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_ARG
    assert lib.b2a_prefill(p, p, p, p, p, 8, 8, 5, 2, 64, _lib.BF16, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_SHAPE
    assert lib.b2a_prefill(p, p, p, p, p, 8, 8, 4, 2, 64, 7, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_DTYPE
    # 16-bit inputs: head_dim 64, 128 or 256 (tensor cores); f32 inputs: a
    # multiple of 4 up to 256 (fp32 kernel)
    assert lib.b2a_prefill(p, p, p, p, p, 8, 8, 4, 2, 96, _lib.BF16, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_UNSUPPORTED
    assert lib.b2a_prefill(p, p, p, p, p, 8, 8, 4, 2, 6, _lib.F32, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_UNSUPPORTED
    assert lib.b2a_prefill(p, p, p, p, p, 8, 8, 4, 2, 260, _lib.F32, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_UNSUPPORTED
    assert lib.b2a_prefill(p, p, p, p, p, 8, 8, 4, 2, 64, _lib.F32, 9, 0.1, 0, 0,
                           None) == _lib.ERR_DTYPE
    assert lib.b2a_prefill(p + 2, p, p, p, p, 8, 8, 4, 2, 64, _lib.BF16, _lib.F32, 0.1, 0, 0,
                           None) == _lib.ERR_ALIGN
    # zero query tokens is a successful no-op
    assert lib.b2a_prefill(p, p, p, p, p, 0, 8, 4, 2, 64, _lib.BF16, _lib.F32, 0.1, 0, 0,
                           None) == _lib.OK


def test_rope_rejects_bad_arguments(lib):
    p = 1 << 20
    # n_tok = 0: every argument check runs, then the call returns before any launch
    base = [p, 0, p, 0, p, 0, None, None, None, p, p, 16, p, 0, p, p, 0, 16, _lib.F32, None,
            _lib.F32, 0, 2, 1, 64, 64, _lib.ROPE_NORM, None]
    assert lib.b2a_rope_append(*base) == _lib.OK
    bad = list(base)
    bad[25] = 63  # odd n_rot
    assert lib.b2a_rope_append(*bad) == _lib.ERR_SHAPE
    bad = list(base)
    bad[26] = 9  # style
    assert lib.b2a_rope_append(*bad) == _lib.ERR_ARG
    bad = list(base)
    bad[13] = 2  # tok_seq_mode
    assert lib.b2a_rope_append(*bad) == _lib.ERR_ARG
    sec = (ctypes.c_int * 4)(0, 0, 0, 0)
    assert lib.b2a_imrope_append(p, 0, p, 0, p, 0, p, sec, 1e4, 1.0, p, 0, p, p, 0, 16, _lib.F32,
                                 p, _lib.F32, 1, 2, 1, 64, None) == _lib.ERR_ARG
    sec = (ctypes.c_int * 4)(40, 0, 0, 0)
    assert lib.b2a_imrope_append(p, 0, p, 0, p, 0, p, sec, 1e4, 1.0, p, 0, p, p, 0, 16, _lib.F32,
                                 p, _lib.F32, 1, 2, 1, 64, None) == _lib.ERR_SHAPE


def test_lse_combine_rejects_bad_arguments(lib):
    assert lib.b2a_lse_combine(None, 0, 16, 0, 2, 3, 4, 16, None, None) == _lib.ERR_ARG
    assert lib.b2a_lse_combine(16, 0, 16, 0, 0, 3, 4, 16, None, None) == _lib.ERR_ARG
    assert lib.b2a_lse_combine(16, 5, 16, 0, 2, 3, 4, 16, None, None) == _lib.ERR_SHAPE


def test_kv_convert_rejects_bad_arguments(lib):
    p, q = 1 << 20, 1 << 21  # never dereferenced: every case returns before a launch
    assert lib.b2a_kv_convert(p, _lib.BF16, q, _lib.F32, 0, None) == _lib.OK
    assert lib.b2a_kv_convert(None, _lib.BF16, q, _lib.F32, 8, None) == _lib.ERR_ARG
    assert lib.b2a_kv_convert(p, _lib.BF16, None, _lib.F32, 8, None) == _lib.ERR_ARG
    assert lib.b2a_kv_convert(p, _lib.BF16, q, _lib.F32, -1, None) == _lib.ERR_ARG
    assert lib.b2a_kv_convert(p, 7, q, _lib.F32, 8, None) == _lib.ERR_DTYPE
    assert lib.b2a_kv_convert(p, _lib.F16, q, 7, 8, None) == _lib.ERR_DTYPE
    assert lib.b2a_kv_convert(p, _lib.F32, p + 16, _lib.F16, 8, None) == _lib.ERR_ARG  # overlap


def test_qwen35_layer_entries_reject_bad_arguments(lib):
    p = 1 << 20
    sec = (ctypes.c_int * 4)(8, 8, 8, 0)
    args = [p, 512, p, 128, p, 128, p, p, 1e-6, p, sec, 1e7, 1.0, p, 1, p, p, 64 * 128, 64,
            _lib.F32, p, _lib.F32, 0, 4, 2, 64, None]
    assert lib.b2a_qwen35_attn_prep(*args) == _lib.OK  # n_tok = 0: checks only
    bad = list(args); bad[8] = 0.0  # epsilon
    assert lib.b2a_qwen35_attn_prep(*bad) == _lib.ERR_ARG
    bad = list(args); bad[23] = 3  # H not a multiple of KV
    assert lib.b2a_qwen35_attn_prep(*bad) == _lib.ERR_SHAPE
    bad = list(args); bad[25] = 40  # 2 * sum(sections) > D
    assert lib.b2a_qwen35_attn_prep(*bad) == _lib.ERR_SHAPE
    assert lib.b2a_sigmoid_gate(p, 64, p, 128, p, 64, 0, 64, None) == _lib.OK
    assert lib.b2a_sigmoid_gate(None, 64, p, 128, p, 64, 4, 64, None) == _lib.ERR_ARG
    assert lib.b2a_sigmoid_gate(p, 32, p, 128, p, 64, 4, 64, None) == _lib.ERR_SHAPE


def test_q8_gemm_entry_points_reject_bad_arguments(lib):
    """Host-side checks of the Q8_0 GEMM / dequantize entry points and of the
    SWIGLU8 epilogue (every rejection returns before any CUDA call)."""
    p = 1 << 20
    # b2a_gemm_q8(a, lda, codes, ldq, scales, lds, dtype, c_in, ldc, out, ldo, out_dtype,
    #             M, N, K, epilogue, stream)
    ok = [p, 96, p, 96, p, 3, _lib.F16, None, 0, p, 64, _lib.F32, 16, 64, 96, 0, None]
    for i, v, code in ((2, None, _lib.ERR_ARG),        # no codes
                       (14, 80, _lib.ERR_SHAPE),       # K not a multiple of 32
                       (3, 88, _lib.ERR_ALIGN),        # code rows not 16 bytes apart
                       (5, 2, _lib.ERR_ALIGN),         # scales row shorter than K/32
                       (4, p + 1, _lib.ERR_ALIGN),     # scales not 2-byte aligned
                       (15, 9, _lib.ERR_ARG),          # epilogue
                       (6, _lib.F32, _lib.ERR_DTYPE)):  # operand type
        bad = list(ok)
        bad[i] = v
        assert lib.b2a_gemm_q8(*bad) == code, (i, v)
    bad = list(ok)
    bad[13], bad[15] = 40, 2  # SWIGLU8 with rows not a multiple of 16
    assert lib.b2a_gemm_q8(*bad) == _lib.ERR_SHAPE
    # b2a_q8_dequant(codes, ldq, scales, lds, out, ldo, dtype, rows, cols, stream)
    assert lib.b2a_q8_dequant(p, 64, p, 2, None, 64, _lib.F16, 8, 64, None) == _lib.ERR_ARG
    assert lib.b2a_q8_dequant(p, 64, p, 2, p, 64, _lib.F16, 8, 48, None) == _lib.ERR_SHAPE
    assert lib.b2a_q8_dequant(p, 64, p, 2, p, 60, _lib.F16, 8, 64, None) == _lib.ERR_ALIGN
    assert lib.b2a_q8_dequant(p, 64, p, 2, p + 8, 64, _lib.F16, 8, 64, None) == _lib.ERR_ALIGN
    # b2a_gemm with SWIGLU8 and rows not a multiple of 16
    assert lib.b2a_gemm(p, 64, p, 64, _lib.BF16, None, 0, p, 64, _lib.F32, 16, 40, 64, 2,
                        None) == _lib.ERR_SHAPE
