"""Oracle for the scaled GEMM family (numpy).

The reference evaluates these products in FP32 (``F.linear`` over
dequantized operands, or Triton ``tl.dot`` with an FP32 accumulator).  The
oracle forms the integer/FP8 dot products exactly in float64 and then applies
the reference's FP32 epilogue in the reference's order, so it is the exact
value of the reference formula up to one FP32 rounding of the accumulator.
"""
from __future__ import annotations

import numpy as np

from .formats import E4M3_MAX, bf16_round, e4m3_decode, e4m3_encode


def _dot(a_vals: np.ndarray, w_vals: np.ndarray) -> np.ndarray:
    return (a_vals.astype(np.float64) @ w_vals.astype(np.float64).T)


def fp8_accumulate(a_codes: np.ndarray, w_codes: np.ndarray) -> np.ndarray:
    """sum_k e4m3(a[m,k]) * e4m3(w[n,k]) -> FP32 [M, N] (A is [M,K], W is [N,K])."""
    return _dot(e4m3_decode(a_codes), e4m3_decode(w_codes)).astype(np.float32)


def int8_accumulate(a_q: np.ndarray, w_q: np.ndarray) -> np.ndarray:
    """Exact int32 accumulator of ``tl.dot(..., out_dtype=int32)``
    (``ops/tensorrt/zipvoice/a1007/b1/i8_residual_runtime_kernel.py:15``)."""
    # float64 products and sums of int8 codes are exact while K * 128 * 128 < 2**53
    assert a_q.shape[-1] < (1 << 38)
    return (a_q.astype(np.float64) @ w_q.astype(np.float64).T).astype(np.int32)


def scaled_epilogue(acc, a_scale, w_scale, bias=None, residual=None):
    """``acc * sa[m] * sb[n] (+ bias) (+ residual)`` in FP32, the order of
    ``ops/triton/fp8.py:32-34`` and ``residual_kernel.py:9``."""
    acc = np.asarray(acc, np.float32)
    sa = np.asarray(a_scale, np.float32)
    sa = sa.reshape(-1, 1) if sa.ndim else sa
    v = (acc * sa).astype(np.float32)
    v = (v * np.asarray(w_scale, np.float32)[None, :]).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    if residual is not None:
        v = (v + np.asarray(residual, np.float32)).astype(np.float32)
    return v


def fp8_gemm(a_codes, w_codes, a_scale, w_scale, bias=None, residual=None, out="f32",
             out_scale=None):
    """W8A8 E4M3 GEMM with FP32 accumulation and the chosen output.

    out: 'f32' | 'bf16' (FP32 values of the BF16 result) | 'e4m3' (codes of
    ``clamp(v / out_scale)``, the static requant of ``_QDQ``).
    """
    v = scaled_epilogue(fp8_accumulate(a_codes, w_codes), a_scale, w_scale, bias, residual)
    return _emit(v, out, out_scale)


def int8_gemm(a_q, w_q, a_scale, w_scale, bias=None, residual=None, out="f32", out_scale=None):
    """INT8 W8A8 GEMM: ``acc.to(float32) * (AS * WS[n]) + bias + r``
    (``ops/tensorrt/zipvoice/a1007/b1/i8_residual_runtime_kernel.py:17-21``)."""
    acc = int8_accumulate(a_q, w_q).astype(np.float32)
    scale = (np.float32(a_scale) * np.asarray(w_scale, np.float32)).astype(np.float32)
    v = (acc * scale[None, :]).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    if residual is not None:
        v = (v + np.asarray(residual, np.float32)).astype(np.float32)
    return _emit(v, out, out_scale)


def _emit(v, out, out_scale):
    if out == "f32":
        return v
    if out == "bf16":
        return bf16_round(v)
    if out == "e4m3":
        return e4m3_encode(np.clip((v / np.float32(out_scale)).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    raise ValueError(out)


def residual_dual(a_codes, w_codes, alpha, bias, residual, inv):
    """``FusedProjectionResidual`` (``ops/tensorrt/zipvoice_fp8_b128/b128/residual_kernel.py:9-11``):
    ``z = acc*Alpha + bias + R``; outputs ``Y = z`` (FP32) and
    ``Q = e4m3_rtne(clamp(z * Inv, +-448))``."""
    acc = fp8_accumulate(a_codes, w_codes)
    z = (acc * np.float32(alpha)).astype(np.float32)
    z = (z + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    z = (z + np.asarray(residual, np.float32)).astype(np.float32)
    q = e4m3_encode(np.clip((z * np.float32(inv)).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    return z, q


def _sigmoid(g: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-g.astype(np.float32)))).astype(np.float32)


def swiglu_requant(gate_acc, up_acc, s1, s3, out_scale, dequant=True):
    """Paired gated-up epilogue of ``ops/triton/cfm_gated_up.py:21-26``:
    ``g = acc_g*S1[n]; u = acc_u*S3[n]; v = g*sigmoid(g)*u``;
    ``q = e4m3(clamp(v * (1/OUT_SCALE)))``; DEQUANT returns ``q*OUT_SCALE``.
    ``S1/S3`` already include the input scale (``cfm_gated_up.py:40``)."""
    g = (np.asarray(gate_acc, np.float32) * np.asarray(s1, np.float32)[None, :]).astype(np.float32)
    u = (np.asarray(up_acc, np.float32) * np.asarray(s3, np.float32)[None, :]).astype(np.float32)
    v = ((g * _sigmoid(g)).astype(np.float32) * u).astype(np.float32)
    inv = np.float32(1.0 / float(out_scale))
    q = e4m3_encode(np.clip((v * inv).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    if dequant:
        return (e4m3_decode(q) * np.float32(out_scale)).astype(np.float32), q
    return q, q


def gated_up(a_codes, w1_codes, w3_codes, s1, s3, out_scale, dequant=True):
    """Full ``_paired`` kernel: two FP8 GEMMs sharing A, then the SwiGLU requant."""
    return swiglu_requant(fp8_accumulate(a_codes, w1_codes), fp8_accumulate(a_codes, w3_codes),
                          s1, s3, out_scale, dequant)


def gated_up_interleaved(a_codes, w_codes, s, out_scale):
    """``_interleaved`` (``ops/triton/cfm_interleaved.py:19-30``): row 2n of W is
    gate n, row 2n+1 is up n; returns E4M3 codes."""
    acc = fp8_accumulate(a_codes, w_codes)
    s = np.asarray(s, np.float32)
    q, _ = swiglu_requant(acc[:, 0::2], acc[:, 1::2], s[0::2], s[1::2], out_scale, dequant=False)
    return q


def pack_weight(weight: np.ndarray):
    """``quantization/weights.py:5-17``: per-output-channel amax/448 (min
    1e-12) scale, E4M3 codes transposed to [K, pad32(N)]."""
    w = np.asarray(weight, np.float32)
    scale = np.maximum((np.abs(w).max(axis=1) / np.float32(448.0)).astype(np.float32), np.float32(1e-12))
    codes = e4m3_encode(np.clip((w / scale[:, None]).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    n, k = w.shape
    packed = np.zeros((k, ((n + 31) // 32) * 32), np.uint8)
    packed[:, :n] = codes.T
    return packed, scale.astype(np.float32)


def fp8_linear(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, bias=None, out_bf16=True):
    """``ops/triton/fp8.py:47-63`` ``linear``: dynamic per-row quant of x,
    FP8 GEMM against the packed [K, Npad] weight, ``acc*sa*sb (+bias)``,
    result in x's dtype."""
    from .normquant import quant_e4m3_row
    n = np.asarray(scales).size
    qa, sa = quant_e4m3_row(np.asarray(x, np.float32))
    w_codes = np.ascontiguousarray(np.asarray(packed, np.uint8)[:, :n].T)
    v = scaled_epilogue(fp8_accumulate(qa, w_codes), sa, scales, bias)
    return bf16_round(v) if out_bf16 else v


def int8_nonlinear_value(q, w, a_scale, w_scale, bias, groups=1):
    """``int8_nonlinear_value`` (``ops/tensorrt/zipvoice/a1007/b1/
    int8_nonlinear_value_runtime_kernel.py:6-34``): three INT8 projections of one
    activation, W = [W0; W1; W2] ([3N, K]), exact int32 accumulators,
    ``z_j = acc_j.to(f32) * (WS[jN + n] * AS) + bias[jN + n]`` (separate roundings,
    ``enable_fp_fusion=False``), ``value = tanh(z0) * z1``, ``gate = z2``.

    q: [M, K] int8 with rows m = t * groups + b (the plugin's [T, B, K]).
    Returns value [groups, M // groups, N] (``V[(b * T + t) * N + n]``, :31-33) and
    gate [M, N] (:34), FP32.  ``np.tanh`` stands in for CUDA's ``tanhf``."""
    q = np.asarray(q, np.int8).reshape(-1, np.asarray(w).shape[1])
    n = np.asarray(w).shape[0] // 3
    acc = int8_accumulate(q, np.asarray(w, np.int8)).astype(np.float32)
    s = (np.asarray(w_scale, np.float32) * np.float32(a_scale)).astype(np.float32)
    z = (acc * s[None, :]).astype(np.float32)
    z = (z + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    value = (np.tanh(z[:, :n]).astype(np.float32) * z[:, n:2 * n]).astype(np.float32)
    steps = q.shape[0] // groups
    return np.ascontiguousarray(value.reshape(steps, groups, n).transpose(1, 0, 2)), z[:, 2 * n:].copy()
