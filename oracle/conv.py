"""Oracle for the quantized learned convolutions of the vocoder (numpy).

Test infrastructure only (imported by tests/, never by the package).  Restates
  * ``ExportWeightOp.forward`` for conv roles (``build/unified_acoustic_export.py:
    156-216``): static per-tensor input Q/DQ (``_QDQ`` at ``:21-33``), per-output-
    channel weight Q/DQ, then ``F.conv1d`` in FP32 on the dequantized values; a
    ``ConvTranspose1d`` with ``conv_transpose_rewrite == "zero_insert_conv"`` is a
    stride-1 conv of the zero-inserted, padded input with the transposed, flipped
    weight (``:84``, ``:114-116``, ``:166-172``);
  * the FP8 MatrixConv kernel ``ops/triton/fp8_conv.py:6-62``: dynamic
    per-utterance input scale max(amax / 448, 1e-12), E4M3 codes, weights packed
    by ``quantization/weights.py:5-17`` ([CI * KW, pad32(CO)], row ci * KW + tap),
    the direct (gather) form of Conv1d with any stride and of ConvTranspose1d,
    ``acc * sx[b] * sw[co] (+ bias)`` in the input's dtype.
The sum of products is formed exactly (float64 over exactly representable code
products) and rounded once.
"""
from __future__ import annotations

import numpy as np

from .formats import E4M3_MAX, e4m3_decode, e4m3_encode, int8_quantize


def quantize_input(x: np.ndarray, in_scale, fmt: str = "e4m3", smooth=None) -> np.ndarray:
    """[B, C, T] FP32 -> codes (E4M3 uint8 or int8) with the static scale
    (INT8: divided by the SmoothQuant factors per channel first)."""
    v = np.asarray(x, np.float32)
    if smooth is not None:
        v = (v / np.asarray(smooth, np.float32)[None, :, None]).astype(np.float32)
    if fmt == "e4m3":
        return e4m3_encode(np.clip((v / np.float32(in_scale)).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    return int8_quantize(v, np.float32(in_scale))


def quantize_weight(w: np.ndarray, w_scale, fmt: str = "e4m3") -> np.ndarray:
    """[CO, CI, KW] -> per-output-channel codes."""
    w = np.asarray(w, np.float32)
    s = np.asarray(w_scale, np.float32)[:, None, None]
    if fmt == "e4m3":
        return e4m3_encode(np.clip((w / s).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    return np.clip(np.rint((w / s).astype(np.float32)), -128, 127).astype(np.int8)


def _values(codes, fmt):
    return e4m3_decode(codes).astype(np.float64) if fmt == "e4m3" else np.asarray(codes).astype(np.float64)


def zero_insert(x: np.ndarray, stride: int) -> np.ndarray:
    """``F.pad(x.unsqueeze(-1), (0, s-1)).reshape(...)[..., :-(s-1)]``."""
    if stride == 1:
        return np.asarray(x)
    b, c, t = x.shape
    out = np.zeros((b, c, (t - 1) * stride + 1), dtype=np.asarray(x).dtype)
    out[..., ::stride] = x
    return out


def conv1d_codes(xq: np.ndarray, wq: np.ndarray, fmt: str, dilation: int, pad_left: int, t_out: int) -> np.ndarray:
    """Exact sum over (ci, tap) of code products: out[b, co, t] =
    sum x[b, ci, t - pad_left + tap*dilation] * w[co, ci, tap] (zero outside)."""
    xv = _values(xq, fmt)
    wv = _values(wq, fmt)
    b, ci, t_in = xv.shape
    co, _, kw = wv.shape
    acc = np.zeros((b, co, t_out), np.float64)
    t = np.arange(t_out)
    for tap in range(kw):
        src = t - pad_left + tap * dilation
        ok = (src >= 0) & (src < t_in)
        xs = np.zeros((b, ci, t_out), np.float64)
        xs[..., ok] = xv[..., src[ok]]
        acc += np.einsum("bct,oc->bot", xs, wv[:, :, tap])
    return acc


def fp8_conv1d(x, w, bias, in_scale, w_scale, *, dilation=1, padding=0, fmt="e4m3", smooth=None):
    """Quantized Conv1d (stride 1): FP32 [B, CO, T_out] =
    (acc * in_scale) * w_scale[co] + bias[co] in FP32, acc the exact code sum."""
    xq = quantize_input(x, in_scale, fmt, smooth)
    wq = quantize_weight(w if smooth is None else np.asarray(w, np.float32) * np.asarray(smooth, np.float32)[None, :, None],
                         w_scale, fmt)
    kw = wq.shape[-1]
    t_out = xq.shape[-1] + 2 * padding - dilation * (kw - 1)
    acc = conv1d_codes(xq, wq, fmt, dilation, padding, t_out).astype(np.float32)
    v = (acc * np.float32(in_scale)).astype(np.float32)
    v = (v * np.asarray(w_scale, np.float32)[None, :, None]).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, np.float32)[None, :, None]).astype(np.float32)
    return v


def fp8_conv_transpose1d(x, w_t, bias, in_scale, w_scale, *, stride, padding=0, output_padding=0, dilation=1,
                         fmt="e4m3", smooth=None):
    """ConvTranspose1d (weight [CI, CO, KW], w_scale per output channel) through
    the zero-insertion rewrite: transposed, flipped weight; input zero-inserted by
    the stride and padded (pad, pad + output_padding), pad = dil (KW-1) - padding.
    INT8 SmoothQuant: the weight is multiplied by smooth along CI (its axis 0,
    ``build/unified_acoustic_export.py:108-111``) and the input divided by it."""
    w_t = np.asarray(w_t, np.float32)
    if smooth is not None:
        w_t = (w_t * np.asarray(smooth, np.float32)[:, None, None]).astype(np.float32)
    w = np.ascontiguousarray(np.flip(np.transpose(w_t, (1, 0, 2)), -1))
    kw = w.shape[-1]
    pad = dilation * (kw - 1) - padding
    xi = zero_insert(np.asarray(x, np.float32), stride)
    xq = quantize_input(xi, in_scale, fmt, smooth)
    wq = quantize_weight(w, w_scale, fmt)
    t_out = xq.shape[-1] + 2 * pad + output_padding - dilation * (kw - 1)
    acc = conv1d_codes(xq, wq, fmt, dilation, pad, t_out).astype(np.float32)
    v = (acc * np.float32(in_scale)).astype(np.float32)
    v = (v * np.asarray(w_scale, np.float32)[None, :, None]).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, np.float32)[None, :, None]).astype(np.float32)
    return v


def gather_conv_codes(xq: np.ndarray, wq: np.ndarray, fmt: str, *, stride: int, padding: int, dilation: int,
                      transpose: bool, t_out: int) -> np.ndarray:
    """Exact code sum of the direct form (``ops/triton/fp8_conv.py:29-37``):
    Conv1d reads x[t * S - padding + tap * dil]; ConvTranspose1d reads
    x[(t + padding - tap * dil) / S] where that division is exact.  wq is
    [CO, CI, KW] (ConvTranspose1d: the [CI, CO, KW] weight permuted (1, 0, 2))."""
    xv = _values(xq, fmt)
    wv = _values(wq, fmt)
    b, ci, t_in = xv.shape
    co, _, kw = wv.shape
    acc = np.zeros((b, co, t_out), np.float64)
    t = np.arange(t_out)
    for tap in range(kw):
        if transpose:
            num = t + padding - tap * dilation
            src = num // stride
            ok = (num % stride == 0) & (src >= 0) & (src < t_in)
        else:
            src = t * stride - padding + tap * dilation
            ok = (src >= 0) & (src < t_in)
        xs = np.zeros((b, ci, t_out), np.float64)
        xs[..., ok] = xv[..., src[ok]]
        acc += np.einsum("bct,oc->bot", xs, wv[:, :, tap])
    return acc


def conv_out_length(t: int, kw: int, stride: int, padding: int, dilation: int, transpose: bool,
                    output_padding: int = 0) -> int:
    """``ops/triton/fp8_conv.py:45``."""
    if transpose:
        return (t - 1) * stride - 2 * padding + dilation * (kw - 1) + output_padding + 1
    return (t + 2 * padding - dilation * (kw - 1) - 1) // stride + 1


def dynamic_input_scale(x: np.ndarray) -> np.ndarray:
    """Per-utterance max(amax / 448, 1e-12) (``ops/triton/fp8_conv.py:6-16``).
    ``tl.max`` and ``tl.maximum`` default to maxnum (NaN operands dropped), so a
    NaN input leaves its utterance's scale finite (``np.fmax`` semantics)."""
    a = np.abs(np.asarray(x, np.float32)).reshape(x.shape[0], -1)
    amax = np.fmax.reduce(np.concatenate([np.zeros((a.shape[0], 1), np.float32), a], axis=1), axis=1)
    return np.fmax((amax.astype(np.float32) / np.float32(448.0)).astype(np.float32), np.float32(1e-12))


def matrix_conv1d(x, packed, scales, bias, ci, co, kw, stride, padding, dilation, transpose, output_padding=0,
                  out_bf16=False):
    """``ops/triton/fp8_conv.conv1d`` (``:43-62``): x [B, CI, T] FP32 values
    (BF16 inputs pass their FP32 values and out_bf16=True)."""
    x = np.asarray(x, np.float32)
    if x.shape[1] != ci:
        raise ValueError("Input channels changed")
    t_out = conv_out_length(x.shape[-1], kw, stride, padding, dilation, transpose, output_padding)
    if t_out <= 0:
        raise ValueError("Non-positive output extent")
    sx = dynamic_input_scale(x)
    xq = e4m3_encode(np.clip((x / sx[:, None, None]).astype(np.float32), -E4M3_MAX, E4M3_MAX))
    wq = np.ascontiguousarray(np.asarray(packed, np.uint8)[: ci * kw, :co].T).reshape(co, ci, kw)
    acc = gather_conv_codes(xq, wq, "e4m3", stride=stride, padding=padding, dilation=dilation, transpose=transpose,
                            t_out=t_out).astype(np.float32)
    v = (acc * sx[:, None, None]).astype(np.float32)
    v = (v * np.asarray(scales, np.float32)[None, :co, None]).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, np.float32)[None, :, None]).astype(np.float32)
    if out_bf16:
        from .formats import bf16_round
        v = bf16_round(v)
    return v
