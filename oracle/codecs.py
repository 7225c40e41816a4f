"""Number-format codecs used by the oracle (test infrastructure only).

Formats:
* fp8 e4m3fn (OCP "FN" variant, max 448, no infinities, NaN = S.1111.111): the
  activation / weight format of QuantType.per_1x128 on NVIDIA hardware
  (`aiter/utility/dtypes.py:10-14` picks float8_e4m3fn on gfx950).
* bf16 round-to-nearest-even, used where the reference casts to bf16
  (`aiter/fused_moe.py:1585`, `:1666`).
* e8m0 (biased power-of-two scale) with the reference's round-up rule
  (`aiter/utility/fp4_utils.py:49-69`).
* MXFP4 e2m1 values packed two per byte, low nibble first
  (`aiter/utility/fp4_utils.py:10-46,100-107`).
"""
import numpy as np

FP8_E4M3_MAX = 448.0

# --------------------------------------------------------------------------- bf16


def f32_to_bf16_bits(x):
    """Round float32 -> bf16 with round-to-nearest-even; returns uint16 bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x):
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --------------------------------------------------------------------------- fp8 e4m3fn

def _fp8_e4m3_table():
    vals = np.zeros(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = s * (m / 8.0) * 2.0 ** -6
        else:
            vals[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


FP8_E4M3_VALUES = _fp8_e4m3_table()


def fp8_e4m3_decode(codes):
    return FP8_E4M3_VALUES[np.asarray(codes, dtype=np.uint8)].astype(np.float32)


def fp8_e4m3_encode(x):
    """float32 -> e4m3fn code with round-to-nearest-even.

    Magnitudes that round to 480 or above become NaN (0x7F / 0xFF), the same
    overflow rule torch's float8_e4m3fn cast uses; the quantisers in this path
    never produce them (|x / scale| <= 448 by construction).
    """
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(x)
    a = np.abs(x)
    # quantum: 2^-9 in the subnormal range, 2^(e-3) in binade [2^e, 2^(e+1))
    _, ex = np.frexp(np.where(a > 0, a, 1.0))
    e = np.maximum(ex - 1, -6)
    q = np.ldexp(1.0, e - 3)
    r = np.rint(a / q) * q                      # exact in float64; rint is half-even
    mag_code = np.zeros(a.shape, dtype=np.int64)
    finite_vals = FP8_E4M3_VALUES[:127]         # codes 0..126, ascending
    idx = np.searchsorted(finite_vals, np.minimum(r, 448.0))
    mag_code = idx.astype(np.int64)
    mag_code = np.where(r >= 480.0, 0x7F, mag_code)
    mag_code = np.where(np.isnan(a), 0x7F, mag_code)
    code = mag_code | np.where(sign, 0x80, 0)
    return code.astype(np.uint8)


def round_fp8(x):
    return fp8_e4m3_decode(fp8_e4m3_encode(x))


# --------------------------------------------------------------------------- e8m0


def f32_to_e8m0(x):
    """Restates `f32_to_e8m0` (aiter/utility/fp4_utils.py:49-58): biased exponent,
    rounded up when mantissa bit 22 is set and (bit 21 or any lower bit or a
    non-zero exponent) -- i.e. round-half-up on the mantissa."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    exponent = ((u >> 23) & 0xFF).astype(np.uint16)
    nan_case = exponent == 0xFF
    round_case = ((u & 0x400000) > 0) & (((u & 0x200000) > 0) | ((u & 0x1FFFFF) > 0) | (exponent > 0))
    exponent = exponent + round_case.astype(np.uint16)
    exponent = (exponent & 0xFF).astype(np.uint8)
    exponent[nan_case] = 0xFF
    return exponent


def e8m0_to_f32(e):
    """Restates `e8m0_to_f32` (aiter/utility/fp4_utils.py:61-69)."""
    e = np.asarray(e, dtype=np.uint8)
    bits = e.astype(np.uint32) << 23
    bits = np.where(e == 0, np.uint32(0x00400000), bits)
    bits = np.where(e == 0xFF, np.uint32(0x7F800001), bits)
    return bits.astype(np.uint32).view(np.float32)


# --------------------------------------------------------------------------- e2m1 (MXFP4)

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e2m1_encode(x):
    """float32 -> 4-bit e2m1 code, round-to-nearest-even, saturating at 6.0.

    Same rounding as the torchao-derived `_f32_to_floatx_unpacked`
    (aiter/utility/fp4_utils.py:112-236): RNE on the e2m1 grid, saturation to
    the largest normal, sign kept for zero.
    """
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(x)
    a = np.minimum(np.abs(x), 6.0)
    # grid quantum: 0.5 below 2, 1.0 in [2,4), 2.0 in [4,6]
    q = np.where(a < 2.0, 0.5, np.where(a < 4.0, 1.0, 2.0))
    r = np.rint(a / q) * q
    r = np.minimum(r, 6.0)
    pos = E2M1_VALUES[:8].astype(np.float64)
    code = np.searchsorted(pos, r).astype(np.uint8)
    nan = np.isnan(x)
    code = np.where(nan, 7, code).astype(np.uint8)
    return (code | np.where(sign, 8, 0)).astype(np.uint8)


def e2m1_decode(codes):
    return E2M1_VALUES[np.asarray(codes, dtype=np.uint8) & 0xF]


def pack_fp4(codes):
    """Pack pairs of 4-bit codes, element 2i in the low nibble
    (`pack_uint4`, aiter/utility/fp4_utils.py:100-107)."""
    c = np.asarray(codes, dtype=np.uint8)
    assert c.shape[-1] % 2 == 0
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_fp4(packed):
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


def mxfp4_to_f32(packed):
    """Restates `mxfp4_to_f32` (aiter/utility/fp4_utils.py:19-46)."""
    return e2m1_decode(unpack_fp4(packed))
