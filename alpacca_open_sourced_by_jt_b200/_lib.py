"""ctypes binding of libb2attn.so (declarations in include/b2attn.h).

Every entry point returns an int status; `check` turns a non-zero status into
a typed exception carrying the library's message.  There is no fallback: if
the shared object is missing or does not load, importing the op modules
raises, so no caller can silently end up on a CPU path.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_float, c_int, c_longlong, c_size_t, c_void_p, c_char_p, POINTER

from .build import LIB_PATH

# element types / styles / status codes (b2attn.h)
F32, F16, BF16 = 0, 1, 2
ROPE_NORM, ROPE_NEOX = 0, 1
OK = 0
ERR_ARG, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_UNSUPPORTED = 1, 2, 3, 4, 5
ERR_WORKSPACE, ERR_CUDA, ERR_TIMEOUT, ERR_POSITION = 6, 7, 8, 9
LAUNCH_PDL = 1  # b2a_set_launch_flags

_NAMES = {
    ERR_ARG: "invalid argument", ERR_SHAPE: "shape", ERR_DTYPE: "dtype",
    ERR_ALIGN: "alignment", ERR_UNSUPPORTED: "unsupported", ERR_WORKSPACE: "workspace",
    ERR_CUDA: "cuda", ERR_TIMEOUT: "device wait timeout", ERR_POSITION: "position",
}


class B2AError(RuntimeError):
    """A libb2attn entry point returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"b2attn {_NAMES.get(code, code)} error: {message}")
        self.code = code


class B2AShapeError(B2AError, ValueError):
    """Bad sizes, shapes, dtypes or alignment (the caller's arguments)."""


class B2ADeviceError(B2AError):
    """A kernel recorded an error on the device (timeout, bad position)."""


# (name, restype, argtypes) for every symbol declared in include/b2attn.h
SIGNATURES = [
    ("b2a_version", c_int, []),
    ("b2a_last_error", c_char_p, []),
    ("b2a_device_error", c_int, [POINTER(c_int), POINTER(c_int), c_int]),
    ("b2a_set_launch_flags", c_int, [c_int]),
    ("b2a_selftest_wait_timeout", c_int, [c_void_p]),
    ("b2a_decode_workspace_bytes", c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    ("b2a_decode_split_rows", c_int, [c_int, c_int, c_int, c_int]),
    ("b2a_decode", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_size_t, c_int, c_int, c_int, c_int, c_int, c_longlong,
                           c_int, c_float, c_int, c_int, c_void_p]),
    ("b2a_decode_noalloc", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_int, c_int, c_int, c_int, c_int, c_longlong, c_int,
                                   c_float, c_int, c_int, c_void_p]),
    ("b2a_shard_exchange_bytes", c_size_t, [c_int, c_int, c_int, c_int]),
    ("b2a_decode_sharded", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_size_t, c_int, c_int, c_int, c_int, c_int,
                                   c_longlong, c_int, c_float, c_int, c_int, c_void_p, c_int,
                                   c_int, c_void_p]),
    ("b2a_ipc_handle", c_int, [c_void_p, c_void_p, POINTER(c_longlong)]),
    ("b2a_ipc_open", c_int, [c_void_p, c_longlong, POINTER(c_void_p), POINTER(c_void_p)]),
    ("b2a_ipc_close", c_int, [c_void_p]),
    ("b2a_lse_combine", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_int, c_int, c_int,
                                c_void_p, c_void_p, c_void_p]),
    ("b2a_prefill", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                            c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_void_p]),
    ("b2a_rope_append", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p,
                                c_longlong, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_int, c_void_p, c_int, c_void_p, c_void_p, c_longlong, c_int,
                                c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                c_int, c_void_p]),
    ("b2a_imrope_append", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p,
                                  c_longlong, c_void_p, POINTER(c_int), c_double, c_double,
                                  c_void_p, c_int, c_void_p, c_void_p, c_longlong, c_int, c_int,
                                  c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    ("b2a_kv_convert", c_int, [c_void_p, c_int, c_void_p, c_int, c_longlong, c_void_p]),
    ("b2a_qwen35_attn_prep", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p,
                                     c_longlong, c_void_p, c_void_p, c_double, c_void_p,
                                     POINTER(c_int), c_double, c_double, c_void_p, c_int,
                                     c_void_p, c_void_p, c_longlong, c_int, c_int, c_void_p,
                                     c_int, c_int, c_int, c_int, c_int, c_void_p]),
    ("b2a_sigmoid_gate", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p,
                                 c_longlong, c_int, c_int, c_void_p]),
    ("b2a_q8_gemv", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int,
                            c_float, c_void_p, c_int, c_void_p]),
    ("b2a_q8_embed", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p,
                             c_void_p]),
    ("b2a_rmsnorm_rows", c_int, [c_void_p, c_longlong, c_void_p, c_float, c_void_p, c_longlong,
                                 c_int, c_int, c_int, c_void_p]),
    ("b2a_swiglu_rows", c_int, [c_void_p, c_longlong, c_int, c_void_p, c_longlong, c_int, c_int,
                                c_int, c_void_p]),
    ("b2a_q8_gemv_qkv_rope", c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_float,
                                     c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                     c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                     c_void_p]),
    ("b2a_gemm", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_int, c_void_p, c_longlong,
                         c_void_p, c_longlong, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    ("b2a_gemm_qkv_rope", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_int, c_int,
                                  c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                  c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    ("b2a_gemm_q8", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p, c_longlong,
                            c_int, c_void_p, c_longlong, c_void_p, c_longlong, c_int, c_int,
                            c_int, c_int, c_int, c_void_p]),
    ("b2a_q8_dequant", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p, c_longlong,
                               c_int, c_int, c_int, c_void_p]),
    ("b2a_gemm_qkv_rope_q8", c_int, [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p,
                                     c_longlong, c_int, c_int, c_int, c_void_p, c_void_p,
                                     c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                     c_void_p, c_int, c_void_p]),
]

_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with argtypes set."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("B2ATTN_LIB", LIB_PATH)
    if not os.path.exists(path):
        raise ImportError(
            f"libb2attn.so not found at {path}; build it with "
            "`python -m alpacca_open_sourced_by_jt_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().b2a_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status == OK:
        return
    cls = B2AShapeError if status in (ERR_ARG, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN,
                                      ERR_UNSUPPORTED, ERR_WORKSPACE) else B2AError
    raise cls(status, last_error())


def device_error(clear: bool = True) -> tuple[int, int]:
    """Synchronise and return (code, aux) of the device error record."""
    code, aux = c_int(0), c_int(0)
    check(load().b2a_device_error(ctypes.byref(code), ctypes.byref(aux), int(clear)))
    return code.value, aux.value


def raise_device_error(clear: bool = True) -> None:
    code, aux = device_error(clear)
    if code:
        raise B2ADeviceError(code, f"kernel reported code {code} (aux {aux:#x})")
