"""Oracle for BigVGAN's anti-aliased Snake activation (numpy, FP32).

``Activation1d(Snake)`` (``models/indextts2/upstream/s2mel/modules/bigvgan/
alias_free_activation/torch/act.py:16-21``) is: replicate-pad 5, 2x
``conv_transpose1d`` with a 12-tap Kaiser-sinc filter, x2, crop 15/15
(``.../torch/resample.py:22-27``), Snake ``v + 1/(a+1e-9) * sin(a v)^2``
(``.../bigvgan/activations.py:48-54``), replicate-pad (5, 6) and a stride-2
12-tap low-pass (``.../torch/filter.py:64-70``).  Written out per sample:

  U[u]  = 2 * sum_{tap<6} up[k] * x[clamp((u + 5 - k) / 2, 0, T-1)],
          k = 2*tap + (u+1)%2                    (``ops/triton/vocoder_tiled_fir.py:22-29``)
  H[u]  = U[u] + inv_beta * sin(alpha * U[u])^2
  y[t]  = sum_{k<12} down[k] * H[clamp(2t + k - 5, 0, 2T-1)]   (``ops/triton/alias_free.py:20-26``)
"""
from __future__ import annotations

import math

import numpy as np


def kaiser_sinc_filter1d(cutoff: float, half_width: float, kernel_size: int) -> np.ndarray:
    """Restates ``.../alias_free_activation/torch/filter.py:19-42`` (float64, then FP32)."""
    even = kernel_size % 2 == 0
    half_size = kernel_size // 2
    delta_f = 4 * half_width
    a = 2.285 * (half_size - 1) * math.pi * delta_f + 7.95
    if a > 50.0:
        beta = 0.1102 * (a - 8.7)
    elif a >= 21.0:
        beta = 0.5842 * (a - 21) ** 0.4 + 0.07886 * (a - 21.0)
    else:
        beta = 0.0
    window = np.kaiser(kernel_size, beta)
    time = (np.arange(-half_size, half_size) + 0.5) if even else (np.arange(kernel_size) - half_size)
    if cutoff == 0:
        return np.zeros(kernel_size, np.float32)
    filt = 2 * cutoff * window * np.sinc(2 * cutoff * time)
    filt = filt / filt.sum()
    return filt.astype(np.float32)


def bigvgan_filters():
    """(up, down) filters of ``UpSample1d(2, 12)`` / ``DownSample1d(2, 12)``:
    both are ``kaiser_sinc_filter1d(0.25, 0.3, 12)`` (``.../torch/resample.py:18,33``)."""
    f = kaiser_sinc_filter1d(0.25, 0.3, 12)
    return f.copy(), f.copy()


def snake_inverse_beta(alpha: np.ndarray) -> np.ndarray:
    """``1.0 / (alpha + 1e-9)`` in FP32 (``.../bigvgan/activations.py:53``)."""
    a = np.asarray(alpha, np.float32)
    return (np.float32(1.0) / (a + np.float32(1e-9)).astype(np.float32)).astype(np.float32)


def upsample2(x: np.ndarray, up: np.ndarray) -> np.ndarray:
    """High-rate signal U [..., 2T] (taps summed in tap order, FP32)."""
    x = np.asarray(x, np.float32)
    t = x.shape[-1]
    idx = np.arange(t)
    out = np.empty(x.shape[:-1] + (2 * t,), np.float32)
    even = np.zeros(x.shape, np.float32)
    odd = np.zeros(x.shape, np.float32)
    for tap in range(6):
        # even u = 2i: k = 2*tap+1, source i + 2 - tap; odd u = 2i+1: k = 2*tap, source i + 3 - tap
        even = (even + x[..., np.clip(idx + 2 - tap, 0, t - 1)] * np.float32(up[2 * tap + 1])).astype(np.float32)
        odd = (odd + x[..., np.clip(idx + 3 - tap, 0, t - 1)] * np.float32(up[2 * tap])).astype(np.float32)
    out[..., 0::2] = np.float32(2.0) * even
    out[..., 1::2] = np.float32(2.0) * odd
    return out


def snake(u: np.ndarray, alpha: np.ndarray, inv_beta: np.ndarray) -> np.ndarray:
    """``x + inv_beta * sin(x * alpha)^2`` per channel (axis -2), FP32."""
    a = np.asarray(alpha, np.float32)[:, None]
    ib = np.asarray(inv_beta, np.float32)[:, None]
    s = np.sin((u * a).astype(np.float32)).astype(np.float32)
    return (u + (ib * (s * s).astype(np.float32)).astype(np.float32)).astype(np.float32)


def downsample2(h: np.ndarray, down: np.ndarray) -> np.ndarray:
    h = np.asarray(h, np.float32)
    n = h.shape[-1]
    t = n // 2
    base = 2 * np.arange(t)
    acc = np.zeros(h.shape[:-1] + (t,), np.float32)
    for k in range(12):
        acc = (acc + h[..., np.clip(base + k - 5, 0, n - 1)] * np.float32(down[k])).astype(np.float32)
    return acc


def alias_free_snake(x, up, down, alpha, inv_beta):
    """Full fused activation on [B, C, T] FP32 (or [C, T])."""
    return downsample2(snake(upsample2(x, up), alpha, inv_beta), down)


def alias_free_snake_int8(x, up, down, alpha, inv_beta, smooth, scale):
    """FIR followed by the INT8 SmoothQuant rule of
    ``deployment/multibatch/fir_quant_kernel.py:36-39``:
    ``rint(div_rn(div_rn(y, smooth[c]), scale))`` clamped to [-128, 127]."""
    y = alias_free_snake(x, up, down, alpha, inv_beta)
    sm = np.asarray(smooth, np.float32)[:, None]
    v = ((y / sm).astype(np.float32) / np.float32(scale)).astype(np.float32)
    return np.clip(np.rint(v), -128, 127).astype(np.int8)
