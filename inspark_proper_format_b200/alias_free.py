"""BigVGAN anti-aliased Snake activation on the fused sm_100a FIR kernel.

Mirrors the reference's torch-level and plugin surface:
  * ``FusedAliasFree`` / ``install``  — ``ops/triton/alias_free.py:28-52``
  * ``TiledFIR`` / ``SmallFIR``       — ``ops/triton/vocoder_tiled_fir.py:43-62``,
                                        ``ops/triton/vocoder_small_fir.py:31-40``
  * ``fir_quant``                     — ``deployment/multibatch/fir_quant_kernel.py:10-40``
The reference's two-kernel version writes a [B, C, 2T] FP32 intermediate;
this one keeps the high-rate row in shared memory.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_Taps = ctypes.c_float * 12


def host_taps(filt) -> "ctypes.Array":
    """12 FIR taps as a host array for the C ABI (the taps travel by value to
    the kernel).  Accepts a tensor on any device, a numpy array or a sequence;
    a CUDA tensor costs one device-to-host copy, so modules convert once."""
    if isinstance(filt, _Taps):
        return filt
    if isinstance(filt, torch.Tensor):
        values = filt.detach().float().reshape(-1).cpu().tolist()
    else:
        values = [float(v) for v in (filt.reshape(-1) if hasattr(filt, "reshape") else filt)]
    if len(values) != 12:
        raise ValueError("Tiled FIR requires complete 12-tap filters")
    return _Taps(*values)


def kaiser_sinc_filter(cutoff: float = 0.25, half_width: float = 0.3, kernel_size: int = 12) -> torch.Tensor:
    """Kaiser-windowed sinc low-pass taps (FP32), the published design BigVGAN's
    ``kaiser_sinc_filter1d`` uses (``.../alias_free_activation/torch/filter.py:19-42``):
    Kaiser beta from the attenuation estimate 2.285 (N/2 - 1) pi (4 hw) + 7.95,
    half-sample-centred taps for even lengths, unit DC gain."""
    even = kernel_size % 2 == 0
    half = kernel_size // 2
    atten = 2.285 * (half - 1) * math.pi * (4 * half_width) + 7.95
    if atten > 50.0:
        beta = 0.1102 * (atten - 8.7)
    elif atten >= 21.0:
        beta = 0.5842 * (atten - 21) ** 0.4 + 0.07886 * (atten - 21.0)
    else:
        beta = 0.0
    window = torch.kaiser_window(kernel_size, beta=beta, periodic=False)
    t = (torch.arange(-half, half) + 0.5) if even else (torch.arange(kernel_size) - half)
    taps = 2 * cutoff * window * torch.sinc(2 * cutoff * t)
    return (taps / taps.sum()).float()


def snake_inverse_beta(beta: torch.Tensor) -> torch.Tensor:
    """``1 / (beta + 1e-9)`` in FP32, the Snake magnitude factor."""
    return 1.0 / (beta.float() + 1e-9)


def fir_snake(x: torch.Tensor, up, down, alpha: torch.Tensor,
              inverse_beta: torch.Tensor, out: torch.Tensor | None = None,
              smooth: torch.Tensor | None = None, scale: float | None = None) -> torch.Tensor:
    """y = down-FIR(Snake(up-FIR(x))) on contiguous CUDA FP32 [B, C, T].

    ``up``/``down``: 12 taps (tensor on any device, sequence, or a
    ``host_taps`` array).  With ``smooth``/``scale`` the output is the INT8
    SmoothQuant code of y.
    """
    if x.ndim != 3 or x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("Tiled FIR expects contiguous CUDA FP32 B,C,F")
    b, c, t = x.shape
    up, down = host_taps(up), host_taps(down)
    for name, v, n in (("alpha", alpha, c), ("inverse_beta", inverse_beta, c)):
        if v.numel() != n or v.dtype != torch.float32 or not v.is_cuda or not v.is_contiguous():
            raise ValueError(f"Tiled FIR channel/length mismatch ({name})")
    quant = smooth is not None
    if quant:
        if smooth.numel() != c or scale is None:
            raise ValueError("Unchanged FIR/source scale geometry required")
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=torch.int8 if quant else torch.float32)
    status = _lib.load().isp_fir_snake(
        x.data_ptr(), b * c, c, t, ctypes.addressof(up), ctypes.addressof(down), alpha.data_ptr(), inverse_beta.data_ptr(),
        out.data_ptr(), _lib.I8 if quant else _lib.F32, _lib.ptr(smooth), float(scale or 0.0),
        _lib.stream_handle(x.device))
    _lib.check(status, "isp_fir_snake")
    return out


def _filter(t: torch.Tensor) -> torch.Tensor:
    return t.detach().float().reshape(-1).contiguous()


class FusedAliasFree(torch.nn.Module):
    """Drop-in for ``Activation1d`` (``ops/triton/alias_free.py:28-43``):
    linear alpha and ``inverse_beta = 1/(beta + 1e-9)`` buffers."""

    def __init__(self, original):
        super().__init__()
        assert original.up_ratio == original.down_ratio == 2
        assert original.upsample.kernel_size == original.downsample.lowpass.kernel_size == 12
        a = original.act
        alpha = a.alpha.detach().float()
        beta = getattr(a, "beta", a.alpha).detach().float()
        if a.alpha_logscale:
            alpha, beta = alpha.exp(), beta.exp()
        self.register_buffer("alpha", alpha.contiguous())
        self.register_buffer("inverse_beta", (1.0 / (beta + 1e-9)).contiguous())
        self.register_buffer("up", _filter(original.upsample.filter))
        self.register_buffer("down", _filter(original.downsample.lowpass.filter))
        self._taps = (host_taps(self.up), host_taps(self.down))

    def forward(self, x):
        if x.dtype != torch.float32:
            raise ValueError("Only tested FP32 activation interface")
        return fir_snake(x.contiguous(), *self._taps, self.alpha, self.inverse_beta)


def install(vocoder):
    """Swap every ``Activation1d`` below ``vocoder`` (``ops/triton/alias_free.py:45-52``)."""
    changed = []

    def walk(module, prefix):
        for name, child in list(module.named_children()):
            path = prefix + "." + name
            if type(child).__name__ == "Activation1d":
                module.add_module(name, FusedAliasFree(child).to(next(child.buffers()).device))
                changed.append(path)
            else:
                walk(child, path)

    walk(vocoder, "vocoder")
    return changed


def _linear_params(alpha, beta):
    """Log-scale (alpha, beta) of the plugin ABI -> (alpha, 1/(beta+1e-9))."""
    a = alpha.detach().float().exp().contiguous()
    ib = (1.0 / (beta.detach().float().exp() + 1e-9)).contiguous()
    return a, ib


class TiledFIR:
    """``ops/triton/vocoder_tiled_fir.py:43-62`` surface: log-scale alpha/beta,
    ``block``/``warps`` accepted and validated like the reference; the sm_100a
    kernel uses its own fixed tile.  Reuses one output buffer per instance."""

    def __init__(self, up, down, alpha, beta, block=256, warps=4):
        if block not in (64, 128, 256, 512) or warps not in (4, 8):
            raise ValueError("Unsupported tiled FIR schedule")
        if up.numel() != 12 or down.numel() != 12:
            raise ValueError("Tiled FIR requires complete 12-tap filters")
        self.parameters = (host_taps(up), host_taps(down), *_linear_params(alpha, beta))
        self.block, self.warps = block, warps
        self.output = None

    def __call__(self, x):
        if x.ndim != 3 or x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("Tiled FIR expects contiguous CUDA FP32 B,C,F")
        b, c, f = x.shape
        if f <= 0 or self.parameters[2].numel() != c or self.parameters[3].numel() != c:
            raise ValueError("Tiled FIR channel/length mismatch")
        if self.output is None:
            self.output = torch.empty_like(x)
        if self.output.shape != x.shape:
            raise ValueError("Tiled FIR instance has fixed shape")
        return fir_snake(x, *self.parameters, out=self.output)


class SmallFIR:
    """``ops/triton/vocoder_small_fir.py:31-40`` surface (rows up to 4096 samples)."""

    def __init__(self, up, down, alpha, beta):
        self.parameters = (host_taps(up), host_taps(down), *_linear_params(alpha, beta))
        self.output = None

    def __call__(self, x):
        if x.dtype != torch.float32 or not x.is_contiguous() or x.shape[-1] > 4096:
            raise ValueError("Expected contiguous FP32 short vocoder activation")
        if self.output is None:
            self.output = torch.empty_like(x)
        return fir_snake(x, *self.parameters, out=self.output)


def fir_quant(x, up, down, alpha, beta, smooth, scale):
    """``inspark_custom::small_fir_activation_quantized``
    (``deployment/multibatch/fir_quant_plugin.py:11-26``): log-scale alpha/beta,
    FP32 FIR math, then ``clamp(rint((y / smooth[c]) / scale))`` as int8."""
    a, ib = _linear_params(alpha, beta)
    s = float(scale) if not isinstance(scale, torch.Tensor) else float(scale.reshape(-1)[0])
    return fir_snake(x, host_taps(up), host_taps(down), a, ib, smooth=smooth.float().contiguous(), scale=s)
