"""Number-format codecs used by the oracle (numpy, written from the format definitions).

* E4M3 (OCP "e4m3fn"): 1 sign, 4 exponent bits (bias 7), 3 mantissa bits,
  no infinities, 0x7F/0xFF are NaN, max finite 448.  The reference always
  clamps to +-448 before the cast (``build/unified_acoustic_export.py:30-33``,
  ``runtime/zipvoice_fp8/quantization.py:13``), so the encoder here only has to
  be round-to-nearest-even on [-448, 448].
* E2M1 (NVFP4 element): magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}; ties go to the
  even code and magnitudes above 6 saturate, the rule ModelOpt's ``_cast_fp4``
  applies through its ``e2m1_bounds`` table (restated, see ``nvfp4.py``).
* BF16: round-to-nearest-even truncation of FP32, as ``Tensor.to(bfloat16)``.
* INT8: ``round`` half-to-even then clamp to [-128, 127]
  (``build/unified_acoustic_export.py:28-29``).
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def _e4m3_table() -> np.ndarray:
    table = np.zeros(256, np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 3) & 0xF
        man = code & 0x7
        if exp == 0xF and man == 0x7:
            table[code] = np.nan
        elif exp == 0:
            table[code] = sign * man * 2.0 ** -9
        else:
            table[code] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return table


E4M3_DECODE = _e4m3_table()


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3_DECODE[np.asarray(codes, np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """FP32 -> E4M3 codes, round-to-nearest-even; |x| must be <= 448 or NaN.

    Values are rounded on the quantum of their binade (2^(e-3), with the
    subnormal binade fixed at 2^-9), which is exactly RNE on the 3-bit
    mantissa.  Sign of zero is preserved, as torch's cast does.
    """
    x = np.asarray(x, np.float32)
    nan = np.isnan(x)
    a = np.abs(np.where(nan, 0.0, x)).astype(np.float64)
    if np.any(a > E4M3_MAX):
        raise ValueError("e4m3_encode expects values clamped to +-448")
    _, e = np.frexp(a)                       # a = m * 2^e, m in [0.5, 1)
    e = np.maximum(e - 1, -6)                # binade exponent, subnormals share -6
    q = np.ldexp(1.0, e - 3)                 # quantum of that binade
    v = np.round(a / q) * q                  # RNE, exact in float64
    _, ev = np.frexp(v)
    ev = ev - 1
    normal = v >= 2.0 ** -6
    exp_field = np.where(normal, ev + 7, 0)
    man_field = np.where(normal, np.round(np.ldexp(v, -ev) * 8.0) - 8.0, np.round(v * 2.0 ** 9))
    code = (exp_field.astype(np.int64) << 3) | man_field.astype(np.int64)
    code = np.where(v == 0.0, 0, code)
    code = code | (np.signbit(x).astype(np.int64) << 7)
    code = np.where(nan, 0x7F, code)
    return code.astype(np.uint8)


def e4m3_quantize(x: np.ndarray, scale) -> np.ndarray:
    """``(x / scale).clamp(-448, 448).to(float8_e4m3fn)`` as codes.

    Follows ``_QDQ.forward`` (``build/unified_acoustic_export.py:27-33``): true
    FP32 division (IEEE), clamp, RNE cast.
    """
    v = (np.asarray(x, np.float32) / np.asarray(scale, np.float32)).astype(np.float32)
    return e4m3_encode(np.clip(v, -E4M3_MAX, E4M3_MAX))


E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    return E2M1_VALUES[np.asarray(codes, np.uint8) & 0xF]


def e2m1_encode(x: np.ndarray) -> np.ndarray:
    """FP32 -> 4-bit E2M1 codes (sign in bit 3), ties to even, saturating at 6.

    Decision points are the midpoints of adjacent magnitudes; at a midpoint
    the even code wins (0.25->0, 0.75->1.0, 1.25->1.0, 1.75->2, 2.5->2,
    3.5->4, 5->4).  The sign bit is ``x < 0`` so -0.0 encodes as +0.
    """
    x = np.asarray(x, np.float32)
    a = np.abs(x)
    mag = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75)
           + (a > 2.5) + (a >= 3.5) + (a > 5.0)).astype(np.uint8)
    return (mag | ((x < 0).astype(np.uint8) << 3)).astype(np.uint8)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """Pack E2M1 codes along the last axis: low nibble = even index, high = odd.

    Mirrors ``packed_nibble_order='low=evenK;high=oddK'``
    (``scripts/export_nvfp4_weights.py:41``).
    """
    codes = np.asarray(codes, np.uint8)
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    packed = np.asarray(packed, np.uint8)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), np.uint8)
    out[..., 0::2] = packed & 0xF
    out[..., 1::2] = packed >> 4
    return out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """FP32 -> nearest-even BF16, returned as FP32 values."""
    x = np.ascontiguousarray(x, np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_to_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bits_to_bf16(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def int8_quantize(x: np.ndarray, scale) -> np.ndarray:
    """``(x / scale).round().clamp(-128, 127)`` (half-to-even), as int8.

    Follows the INT8 branch of ``_QDQ.forward``
    (``build/unified_acoustic_export.py:27-29``) and the INT8 weight export
    (``scripts/export_weights.py:62``).
    """
    v = (np.asarray(x, np.float32) / np.asarray(scale, np.float32)).astype(np.float32)
    return np.clip(np.round(v), -128, 127).astype(np.int8)
