"""Quantized learned convolutions on tcgen05: a phase-folded implicit GEMM over
channels-last codes (``isp_conv1d_pack_weight`` / ``isp_conv1d_quant`` /
``isp_conv1d``).

Reference surfaces mirrored here:
  * ``ops.triton.fp8_conv.conv1d`` (``ops/triton/fp8_conv.py:43-62``) -- same
    signature; dynamic per-utterance E4M3 input scale, weights packed by
    ``quantization/weights.pack_weight`` ([CI * KW, pad32(CO)]), Conv1d with any
    stride and ConvTranspose1d, output in ``x.dtype``;
  * ``MatrixConv`` with precision 'fp8' (``ops/eager/matrix.py:33-41``,
    ``quantization/precision.py:15-56``, dispatch ``ops/matrix.py:21-31``) ->
    ``FP8MatrixConv``;
  * ``ExportWeightOp`` for ``nn.Conv1d`` / ``nn.ConvTranspose1d`` roles with an
    FP8 or INT8 spec (``build/unified_acoustic_export.py:75-216``): static input
    scale, INT8 SmoothQuant folded into the weight, ConvTranspose1d through the
    zero-insertion rewrite -> ``QuantConv1d``.  The phase-folded form multiplies
    the same code pairs as that rewrite and skips its zero rows.
Groups = 1 and zero padding, as the reference requires.
"""
from __future__ import annotations

import ctypes
import weakref

import torch
from torch import nn

from . import _lib
from .gemm import pack_weight

_CODES = {"fp8": (_lib.E4M3, torch.float8_e4m3fn, 448.0), "int8": (_lib.I8, torch.int8, 127.0)}
_OUT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _pad128(c: int) -> int:
    return (c + 127) // 128 * 128


def out_length(t: int, kw: int, stride: int, padding: int, dilation: int, transpose: bool,
               output_padding: int = 0) -> int:
    """Output extent (``ops/triton/fp8_conv.py:45``)."""
    if transpose:
        return (t - 1) * stride - 2 * padding + dilation * (kw - 1) + output_padding + 1
    return (t + 2 * padding - dilation * (kw - 1) - 1) // stride + 1


def geometry(kw: int, stride: int, dilation: int, padding: int, transpose: bool) -> tuple[int, int]:
    """(phases P, window slots W) of the phase-folded form."""
    phases, taps = ctypes.c_int(), ctypes.c_int()
    _lib.check(_lib.load().isp_conv1d_geometry(kw, stride, dilation, padding, int(transpose), ctypes.byref(phases),
                                               ctypes.byref(taps)), "isp_conv1d_geometry")
    return phases.value, taps.value


def pack_folded(codes_kn: torch.Tensor, co: int, ci: int, kw: int, stride: int, dilation: int, padding: int,
                transpose: bool) -> torch.Tensor:
    """Weight codes [CI * KW, ldw] (row ci * KW + tap; E4M3 or INT8) -> the
    phase-folded B operand [CO * P, W, C_pad] on the codes' device."""
    codes = codes_kn.contiguous()
    if codes.dim() != 2 or codes.shape[0] != ci * kw or codes.shape[1] < co:
        raise ValueError("weight codes must be [CI * KW, >= CO]")
    phases, taps = geometry(kw, stride, dilation, padding, transpose)
    c_pad = _pad128(ci)
    out = torch.empty(co * phases, taps, c_pad, device=codes.device, dtype=codes.dtype)
    _lib.check(_lib.load().isp_conv1d_pack_weight(codes.data_ptr(), codes.shape[1], co, ci, kw, stride, dilation,
                                                  padding, int(transpose), out.data_ptr(), c_pad,
                                                  _lib.stream_handle(codes.device)), "isp_conv1d_pack_weight")
    return out


def run(x: torch.Tensor, w_folded: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None, *, ci: int, co: int,
        kw: int, stride: int, padding: int, dilation: int, transpose: bool, output_padding: int = 0,
        code: str = "fp8", in_scale: float | None = None, smooth: torch.Tensor | None = None,
        out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Quantize x [B, CI, T] and run the phase-folded conv.  in_scale None: the
    dynamic per-utterance E4M3 scale; else the static scale (INT8: x / smooth
    first)."""
    if x.dim() != 3 or x.shape[1] != ci:
        raise ValueError("Input channels changed")
    out_dtype = out_dtype or (x.dtype if x.dtype in _OUT else torch.float32)
    if out_dtype not in _OUT:
        raise ValueError(f"unsupported output dtype {out_dtype}")
    xin = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    xin = xin.contiguous()
    b, _, t = xin.shape
    t_out = out_length(t, kw, stride, padding, dilation, transpose, output_padding)
    if t_out <= 0:
        raise ValueError("Non-positive output extent")
    code_dtype = _CODES[code][0]
    c_pad = w_folded.shape[-1]
    row_multiple = 1 if transpose else stride
    t_rows = (t + row_multiple - 1) // row_multiple * row_multiple
    lib = _lib.load()
    stream = _lib.stream_handle(x.device)
    xq = torch.empty(b, t_rows, c_pad, device=x.device, dtype=torch.uint8)
    amax = torch.empty(b, device=x.device, dtype=torch.float32) if in_scale is None else None
    x_dtype = _lib.BF16 if xin.dtype == torch.bfloat16 else _lib.F32
    _lib.check(lib.isp_conv1d_quant(xin.data_ptr(), x_dtype, b, ci, t, row_multiple, _lib.ptr(smooth),
                                    0.0 if in_scale is None else float(in_scale), _lib.ptr(amax), code_dtype,
                                    xq.data_ptr(), c_pad, stream), "isp_conv1d_quant")
    y = torch.empty(b, co, t_out, device=x.device, dtype=out_dtype)
    _lib.check(lib.isp_conv1d(xq.data_ptr(), code_dtype, b, c_pad, t, w_folded.data_ptr(), co, kw, stride, dilation,
                              padding, output_padding, int(transpose), t_out,
                              0.0 if in_scale is None else float(in_scale), _lib.ptr(amax), w_scale.data_ptr(),
                              _lib.ptr(bias), y.data_ptr(), _OUT[out_dtype], stream), "isp_conv1d")
    return y


_FOLDED: dict = {}


def _folded_cached(packed: torch.Tensor, co, ci, kw, stride, dilation, padding, transpose) -> torch.Tensor:
    """pack_folded of a reference-packed weight, done once per tensor object
    and geometry (invalidated when the tensor is freed or modified in place)."""
    key = (id(packed), co, ci, kw, stride, dilation, padding, bool(transpose))
    hit = _FOLDED.get(key)
    if hit is not None:
        ref, version, folded = hit
        if ref() is packed and version == packed._version:
            return folded
    folded = pack_folded(packed.view(torch.uint8), co, ci, kw, stride, dilation, padding, transpose)
    _FOLDED[key] = (weakref.ref(packed, lambda _r, k=key: _FOLDED.pop(k, None)), packed._version, folded)
    return folded


def conv1d(x, weight, scales, bias, ci, co, kw, stride, padding, dilation, transpose, output_padding, tile=None):
    """Drop-in for ``ops.triton.fp8_conv.conv1d``: ``weight`` is the
    ``pack_weight`` output [CI * KW, pad32(CO)] (E4M3), ``scales`` [CO];
    dynamic per-utterance input scale; result in ``x.dtype``.  ``tile`` is
    accepted for signature compatibility (one sm_100a schedule)."""
    if x.shape[1] != ci:
        raise ValueError("Input channels changed")
    folded = _folded_cached(weight, co, ci, kw, stride, dilation, padding, transpose)
    return run(x, folded, scales.float().contiguous(), None if bias is None else bias.float().contiguous(), ci=ci,
               co=co, kw=kw, stride=stride, padding=padding, dilation=dilation, transpose=transpose,
               output_padding=output_padding)


class FP8MatrixConv(nn.Module):
    """``MatrixConv(module, 'fp8', ...)``: weights packed once by ``pack_weight``
    (ConvTranspose1d: of ``weight.permute(1, 0, 2)``), forward = ``conv1d``."""

    def __init__(self, module: nn.Module):
        super().__init__()
        if not isinstance(module, (nn.Conv1d, nn.ConvTranspose1d)):
            raise TypeError(f"Unsupported convolution {type(module).__name__}")
        self.transpose = isinstance(module, nn.ConvTranspose1d)
        for name in ("in_channels", "out_channels", "kernel_size", "stride", "padding", "dilation", "groups"):
            setattr(self, name, getattr(module, name))
        self.output_padding = getattr(module, "output_padding", (0,))
        if self.groups != 1 or module.padding_mode != "zeros":
            raise ValueError("Only groups1/zero-padding learned convolutions")
        weight = module.weight.detach()
        ci, co, kw = self.in_channels, self.out_channels, self.kernel_size[0]
        dense = weight.permute(1, 0, 2) if self.transpose else weight
        packed, scales = pack_weight(dense.reshape(co, ci * kw))
        self.register_buffer("weight", packed)
        self.register_buffer("scales", scales)
        self.register_buffer("bias", module.bias.detach().clone() if module.bias is not None else None)
        self.precision = "fp8"

    def forward(self, x):
        return conv1d(x, self.weight, self.scales, self.bias, self.in_channels, self.out_channels,
                      self.kernel_size[0], self.stride[0], self.padding[0], self.dilation[0], self.transpose,
                      self.output_padding[0])


class QuantConv1d(nn.Module):
    """``ExportWeightOp(original, spec)`` for a conv role, run on the kernels.

    spec: ``precision`` ('fp8' | 'int8'), ``input_scale``, optional
    ``weight_scale`` (per output channel, or one value; computed as amax/448 or
    /127 when absent), ``weight_axis``, ``smooth_scale`` (INT8),
    ``conv_transpose_rewrite``.
    """

    def __init__(self, original: nn.Module, spec: dict):
        super().__init__()
        if not isinstance(original, (nn.Conv1d, nn.ConvTranspose1d)):
            raise TypeError(f"Unsupported weighted operator {type(original).__name__}")
        transpose = isinstance(original, nn.ConvTranspose1d)
        if original.groups != 1 or original.padding_mode != "zeros":
            raise ValueError("Learned acoustic Conv export requires groups=1 and zero padding")
        if spec.get("precision") not in _CODES:
            raise ValueError(f"QuantConv1d needs an fp8 or int8 spec, got {spec.get('precision')!r}")
        if "input_scale" not in spec:
            raise ValueError("Quantized export requires a calibrated input_scale")
        self.precision = spec["precision"]
        _, torch_dtype, qmax = _CODES[self.precision]
        self.transpose = transpose
        self.stride = original.stride[0]
        self.padding = original.padding[0]
        self.dilation = original.dilation[0]
        self.output_padding = getattr(original, "output_padding", (0,))[0]
        self.kernel_size = original.kernel_size[0]
        self.in_channels, self.out_channels = original.in_channels, original.out_channels
        weight = original.weight.detach().float().clone()
        smooth = spec.get("smooth_scale")
        if smooth is not None:
            if self.precision != "int8":
                raise ValueError("SmoothQuant scale belongs only to an INT8 recipe")
            smooth = torch.as_tensor(smooth, dtype=torch.float32, device=weight.device).reshape(-1)
            if smooth.numel() != self.in_channels or not bool((smooth > 0).all()):
                raise ValueError("smooth_scale has invalid shape or values")
            weight = weight * smooth.reshape((-1, 1, 1) if transpose else (1, -1, 1))
        # dense [CO, CI, KW] in the gather form: ConvTranspose1d weight [CI, CO, KW] permuted
        axis = int(spec.get("weight_axis", 0))
        dense = weight.permute(1, 0, 2) if transpose else weight
        out_axis = 1 if transpose else 0
        co, ci, kw = dense.shape
        if "weight_scale" in spec:
            w_scale = torch.as_tensor(spec["weight_scale"], dtype=torch.float32, device=weight.device).reshape(-1)
            if w_scale.numel() == 1:
                w_scale = w_scale.expand(co).contiguous()
            elif axis != out_axis or w_scale.numel() != co:
                raise ValueError("QuantConv1d needs per-output-channel weight scales")
        else:
            if axis != out_axis:
                raise ValueError("QuantConv1d needs per-output-channel weight scales")
            w_scale = dense.abs().amax(dim=(1, 2)).clamp_min(1e-12) / qmax
        if not bool(torch.isfinite(w_scale).all()) or not bool((w_scale > 0).all()):
            raise ValueError("weight_scale must contain finite positive values")
        normalized = dense / w_scale[:, None, None]
        codes = (normalized.round().clamp(-128, 127).to(torch.int8) if self.precision == "int8"
                 else normalized.clamp(-448, 448).to(torch.float8_e4m3fn))
        self.register_buffer("weight_codes", codes.reshape(co, ci * kw).t().contiguous())   # [CI * KW, CO]
        self.register_buffer("weight_scale", w_scale.contiguous())
        self.register_buffer("bias", None if original.bias is None else original.bias.detach().float().clone())
        self.register_buffer("smooth_scale", smooth)
        self.input_scale = float(spec["input_scale"])
        if not self.input_scale > 0:
            raise ValueError("input_scale must be positive")
        self._folded = None

    def folded_weight(self) -> torch.Tensor:
        if self._folded is None or self._folded.device != self.weight_codes.device:
            self._folded = pack_folded(self.weight_codes.view(torch.uint8), self.out_channels, self.in_channels,
                                        self.kernel_size, self.stride, self.dilation, self.padding, self.transpose)
        return self._folded

    def out_length(self, t: int) -> int:
        return out_length(t, self.kernel_size, self.stride, self.padding, self.dilation, self.transpose,
                          self.output_padding)

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return run(x, self.folded_weight(), self.weight_scale, self.bias, ci=self.in_channels,
                   co=self.out_channels, kw=self.kernel_size, stride=self.stride, padding=self.padding,
                   dilation=self.dilation, transpose=self.transpose, output_padding=self.output_padding,
                   code=self.precision, in_scale=self.input_scale, smooth=self.smooth_scale, out_dtype=out_dtype)
