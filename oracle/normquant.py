"""Oracle for the fused norm -> quantize step (numpy).

Numeric contract shared with the CUDA kernel (``csrc/norm_quant.cu``):

* the row statistic (mean of squares, or of squared deviations for BiasNorm)
  squares each element in FP32, accumulates in float64 and rounds once to
  FP32, then divides by K in FP32 — the reference computes the same formula
  with an FP32 running sum (``torch.mean``), so on rare rows the reference's
  statistic differs by an ulp; the golden tests measure that rate;
* ``rsqrt`` is ``1 / sqrt`` with both steps IEEE-rounded, which is what
  torch's CPU ``rsqrt`` evaluates;
* every later step is a single IEEE FP32 operation in the reference's order.
"""
from __future__ import annotations

import numpy as np

from .formats import (E4M3_MAX, bf16_round, e2m1_encode, e4m3_decode, e4m3_encode,
                      int8_quantize, pack_nibbles)

NORM_NONE, NORM_RMS_GPTFAST, NORM_RMS_QWEN, NORM_BIAS = 0, 1, 2, 3
Q_E4M3_STATIC, Q_E4M3_ROW, Q_INT8_STATIC, Q_NVFP4 = 0, 1, 2, 3


def _mean_sq(v: np.ndarray) -> np.ndarray:
    sq = (v * v).astype(np.float32)
    s = sq.astype(np.float64).sum(axis=-1, keepdims=True).astype(np.float32)
    return (s / np.float32(v.shape[-1])).astype(np.float32)


def _rsqrt(v: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / np.sqrt(v.astype(np.float32))).astype(np.float32)


def rms_norm_gptfast(x: np.ndarray, gamma: np.ndarray, eps: float, input_is_bf16: bool) -> np.ndarray:
    """gpt_fast ``RMSNorm.forward``: ``_norm(x.float()).type_as(x) * weight``.

    ``models/indextts2/upstream/s2mel/modules/gpt_fast/model.py:246-258``:
    the normalized value is rounded to the input dtype before the FP32 gamma
    multiply (BF16 x FP32 promotes to FP32).
    """
    xf = np.asarray(x, np.float32)
    r = _rsqrt((_mean_sq(xf) + np.float32(eps)).astype(np.float32))
    y = (xf * r).astype(np.float32)
    if input_is_bf16:
        y = bf16_round(y)
    return (y * np.asarray(gamma, np.float32)).astype(np.float32)


def adaptive_layer_norm(x: np.ndarray, gamma: np.ndarray, eps: float, ada_w: np.ndarray, ada_b: np.ndarray,
                        rows_per_group: int, input_is_bf16: bool) -> np.ndarray:
    """gpt_fast ``AdaptiveLayerNorm.forward`` with its RMSNorm
    (``models/indextts2/upstream/s2mel/modules/gpt_fast/model.py:18-32``):
    ``weight * norm(x) + bias`` where (weight, bias) are the FP32 projection of
    the conditioning embedding, one [K] pair per utterance.  Rows are grouped
    ``rows_per_group`` per utterance (the [B, T, K] -> [B*T, K] flattening);
    the multiply and the add are separate FP32 roundings."""
    y = rms_norm_gptfast(x, gamma, eps, input_is_bf16)
    g = np.arange(y.shape[0]) // int(rows_per_group)
    w = np.asarray(ada_w, np.float32)[g]
    b = np.asarray(ada_b, np.float32)[g]
    return ((w * y).astype(np.float32) + b).astype(np.float32)


def rms_norm_qwen(x: np.ndarray, gamma: np.ndarray, eps: float, input_is_bf16: bool) -> np.ndarray:
    """Qwen-style ``RMSNorm.forward`` (``models/indextts2/dspark/draft.py:19-23``).

    ``(x.float() * rsqrt(mean(x^2) + eps) * weight.float()).to(dtype)``: gamma
    is applied in FP32 and the product is rounded to the input dtype once.
    """
    xf = np.asarray(x, np.float32)
    r = _rsqrt((_mean_sq(xf) + np.float32(eps)).astype(np.float32))
    y = ((xf * r).astype(np.float32) * np.asarray(gamma, np.float32)).astype(np.float32)
    return bf16_round(y) if input_is_bf16 else y


def bias_norm(x: np.ndarray, bias: np.ndarray, log_scale_exp: float, input_is_bf16: bool) -> np.ndarray:
    """Zipformer ``BiasNormFunction.forward``
    (``models/zipvoice/reference/models/modules/scaling.py:348-370``):
    ``scales = mean((x - b)^2) ** -0.5 * exp(log_scale); ans = x * scales``.

    ``log_scale_exp`` is ``exp(log_scale)`` already evaluated (the wrapper
    takes it from the module's own scalar).  The output is in the input dtype.
    """
    xf = np.asarray(x, np.float32)
    d = (xf - np.asarray(bias, np.float32)).astype(np.float32)
    s = (_rsqrt(_mean_sq(d)) * np.float32(log_scale_exp)).astype(np.float32)
    y = (xf * s).astype(np.float32)
    return bf16_round(y) if input_is_bf16 else y


def normalize(x, kind, gamma=None, bias=None, eps=1e-6, log_scale_exp=1.0, input_is_bf16=True):
    if kind == NORM_NONE:
        return np.asarray(x, np.float32)
    if kind == NORM_RMS_GPTFAST:
        return rms_norm_gptfast(x, gamma, eps, input_is_bf16)
    if kind == NORM_RMS_QWEN:
        return rms_norm_qwen(x, gamma, eps, input_is_bf16)
    if kind == NORM_BIAS:
        return bias_norm(x, bias, log_scale_exp, input_is_bf16)
    raise ValueError(kind)


def quant_e4m3_static(y: np.ndarray, scale: float) -> np.ndarray:
    """Static per-tensor E4M3 Q (``build/unified_acoustic_export.py:27-33``)."""
    return e4m3_encode(np.clip((np.asarray(y, np.float32) / np.float32(scale)).astype(np.float32),
                               -E4M3_MAX, E4M3_MAX))


def quant_e4m3_row(y: np.ndarray):
    """Dynamic per-row E4M3 (``ops/triton/fp8.py:11-17``):
    ``s = max(amax/448, 1e-12); q = e4m3(x / s)`` (saturating cast)."""
    y = np.asarray(y, np.float32)
    s = np.maximum((np.abs(y).max(axis=-1) / np.float32(448.0)).astype(np.float32),
                   np.float32(1e-12)).astype(np.float32)
    v = np.clip((y / s[:, None]).astype(np.float32), -E4M3_MAX, E4M3_MAX)
    return e4m3_encode(v), s


def quant_int8_static(y: np.ndarray, in_scale: float, smooth: np.ndarray | None) -> np.ndarray:
    """SmoothQuant activation path of ``ExportWeightOp.forward``
    (``build/unified_acoustic_export.py:160-162`` divide by ``smooth_scale``,
    then ``_QDQ`` INT8 at ``:27-29``)."""
    v = np.asarray(y, np.float32)
    if smooth is not None:
        v = (v / np.asarray(smooth, np.float32)).astype(np.float32)
    return int8_quantize(v, np.float32(in_scale))


def nvfp4_block_scales(y: np.ndarray, global_scale: float) -> np.ndarray:
    """Per-16-element E4M3 block scale of the two-level NVFP4 scheme.

    Restates ModelOpt 0.47 ``NVFP4QTensor.get_weights_scaling_factor``
    (called from ``scripts/export_nvfp4_weights.py:35``): block amax / (6 * g),
    zero scales replaced by 1.0, then cast to E4M3 (RNE).
    """
    y = np.asarray(y, np.float32)
    blocks = y.reshape(y.shape[:-1] + (y.shape[-1] // 16, 16))
    amax = np.abs(blocks).max(axis=-1).astype(np.float32)
    s = (amax / (np.float32(6.0) * np.float32(global_scale))).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s)
    return e4m3_encode(np.minimum(s, np.float32(E4M3_MAX)))


def quant_nvfp4(y: np.ndarray, global_scale: float):
    """Two-level NVFP4 quantization of the last axis (16-element K blocks).

    ``q = e2m1(x / (float(s_block) * g))`` with nibbles packed low = even K
    (``scripts/export_nvfp4_weights.py:35-41``; restated ModelOpt
    ``NVFP4QTensor.quantize``).  Returns (packed uint8 [..., K/2], E4M3 block
    scale codes [..., K/16]).
    """
    y = np.asarray(y, np.float32)
    scodes = nvfp4_block_scales(y, global_scale)
    denom = (e4m3_decode(scodes) * np.float32(global_scale)).astype(np.float32)
    blocks = y.reshape(y.shape[:-1] + (y.shape[-1] // 16, 16))
    with np.errstate(divide="ignore", invalid="ignore"):
        v = (blocks / denom[..., None]).astype(np.float32)
    codes = e2m1_encode(v.reshape(y.shape))
    return pack_nibbles(codes), scodes


def norm_quant(x, kind, fmt, *, gamma=None, bias=None, eps=1e-6, log_scale_exp=1.0,
               input_is_bf16=True, scale=None, smooth=None, global_scale=None):
    """Reference semantics of ``isp_norm_quant``: normalize, then quantize.

    Returns (codes, scales): scales is None (static formats), FP32 [M] (per
    row E4M3) or E4M3 codes [M, K/16] (NVFP4).
    """
    y = normalize(x, kind, gamma, bias, eps, log_scale_exp, input_is_bf16)
    if fmt == Q_E4M3_STATIC:
        return quant_e4m3_static(y, scale), None
    if fmt == Q_E4M3_ROW:
        return quant_e4m3_row(y)
    if fmt == Q_INT8_STATIC:
        return quant_int8_static(y, scale, smooth), None
    if fmt == Q_NVFP4:
        return quant_nvfp4(y, global_scale)
    raise ValueError(fmt)
