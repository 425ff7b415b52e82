"""The arithmetic the Q8_0 decoders use (b2a_gemm_q8's converter warps and
b2a_q8_dequant), checked exhaustively on the host.

f16 operands: a code c (int8) becomes an exact f16 as (1024 + (c + 128)) -
1152: the byte c ^ 0x80 = c + 128 is placed under the f16 exponent of 1024
(bits 0x64xx), where the spacing is 1, and 1152 (0x6480) is subtracted.  The
result is then multiplied by the f16 scale d with one rounding.  The host's
dequantized copy is (float32(c) * float32(d)) rounded to f16; c * d has at
most 8 + 11 significant bits, so the f32 product is exact and both round the
same exact value once.  numpy's float16 arithmetic rounds each operation to
f16, as the device's f16x2 instructions do, so the steps are restated here
operation by operation for every code and every finite f16 scale.

bf16 operands: the code is formed exactly in f32 (2^23 + c + 128, minus
2^23 + 128), multiplied by float32(d) exactly and rounded once to bf16, the
same expression as the host copy; the test checks the exact-formation step.
"""
import numpy as np


def test_f16_bias_trick_is_exact_for_every_code_and_scale():
    codes = np.arange(-128, 128, dtype=np.int32)
    u = (codes.astype(np.int64) ^ 0x80) & 0xFF               # the byte c ^ 0x80
    biased = (0x6400 | u).astype(np.uint16).view(np.float16)  # 1024 + c + 128
    c16 = biased - np.float16(1152)                           # one f16 subtraction
    assert np.array_equal(c16.astype(np.float64), codes.astype(np.float64))

    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    d = bits.view(np.float16)
    d = d[np.isfinite(d)]                                     # every finite f16 scale
    with np.errstate(over="ignore"):  # large scales overflow to inf on both sides
        got = (c16[:, None] * d[None, :])                     # one f16 multiplication
        want = (codes.astype(np.float32)[:, None] * d.astype(np.float32)[None, :]).astype(
            np.float16)
    # bit-for-bit, infinities and signed zeros included
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def test_bf16_path_forms_codes_exactly_in_f32():
    codes = np.arange(-128, 128, dtype=np.int32)
    u = ((codes.astype(np.int64) ^ 0x80) & 0xFF).astype(np.uint32)
    f = (np.uint32(0x4B000000) | u).view(np.float32) - np.float32(8388736.0)  # 2^23 + 128
    assert np.array_equal(f, codes.astype(np.float32))
