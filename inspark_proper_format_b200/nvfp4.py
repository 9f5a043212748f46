"""NVFP4 linear path: E2M1 codes, one E4M3 scale per 16 K elements, an FP32
global scale per tensor (torch-level wrappers over ``isp_nvfp4_gemm``,
``isp_nvfp4_gated_up`` and ``isp_nvfp4_scales_to_mma``).

Reference surfaces mirrored here:
  * ``MatrixWeightOp(linear).apply_nvfp4(activation_amax)`` followed by its
    forward (``build/nvfp4_graph.py:12-87``; installed per role by
    ``quantization/nvfp4.py:11-56``) -> ``NVFP4Linear``: dynamic per-16-K
    activation quantization with the calibrated FP32 global scale
    ``fp16(amax) / (6 * 448)``, native FP4 GEMM, FP32 bias;
  * the exporter's storage format (``scripts/export_nvfp4_weights.py:25-42``):
    ``weight`` uint8 [N, K/2] (low nibble = even K), ``block_scale`` E4M3
    [N, K/16], ``global_scale`` FP32 -> ``NVFP4Weight.from_export``;
  * the CFM feed-forward ``w2(silu(w1 x) * w3 x)`` (``gpt_fast/model.py:235-244``)
    under the NVFP4 recipe -> ``NVFP4GatedUp`` (gate/up GEMMs + SiLU-gate + NVFP4
    requant of h in one kernel, then the down GEMM).

Block scales are kept in the tensor-core layout (128-row x 4-block chunks of
512 bytes, K chunks first) that the kernels read with one bulk copy per
stage; ``scales_to_mma`` converts the exporter's row-major scales once.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from . import _lib
from .norm_quant import mma_scale_bytes, norm_quant

E2M1_MAX = 6.0
E4M3_MAX = 448.0
_OUT = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16, torch.float32: _lib.F32}


def activation_global_scale(activation_amax) -> float:
    """``amax.half().float() / (6 * 448)`` (``scripts/export_nvfp4_weights.py:39``)."""
    a = torch.as_tensor(activation_amax, dtype=torch.float32).max().half().float()
    return float(a / torch.tensor(E2M1_MAX * E4M3_MAX, dtype=torch.float32))


def weight_global_scale(w: torch.Tensor) -> float:
    """Max-PTQ global scale ``amax(W) / (6 * 448)`` in FP32."""
    return float(w.detach().float().abs().max() / torch.tensor(E2M1_MAX * E4M3_MAX, dtype=torch.float32,
                                                                 device=w.device))


def scales_to_mma(block_scale: torch.Tensor, k: int) -> torch.Tensor:
    """Row-major E4M3 block scales [R, K/16] -> flat uint8 tensor-core layout
    (rows padded to 128 with zero scales)."""
    if not block_scale.is_cuda:
        raise ValueError("scales_to_mma expects a CUDA tensor")
    src = block_scale.contiguous().view(torch.uint8).reshape(-1, k // 16)
    rows = src.shape[0]
    dst = torch.empty(mma_scale_bytes(rows, k), device=src.device, dtype=torch.uint8)
    status = _lib.load().isp_nvfp4_scales_to_mma(src.data_ptr(), rows, k, dst.data_ptr(),
                                                 _lib.stream_handle(src.device))
    _lib.check(status, "isp_nvfp4_scales_to_mma")
    return dst


def stack_gate_up(w1: torch.Tensor, w3: torch.Tensor) -> torch.Tensor:
    """Stack gate and up rows in blocks of 64 (rows [128j, 128j+64) = w1 rows
    [64j, 64j+64), the next 64 = the same rows of w3): one 128-row tile of the
    stacked matrix holds the gate and up halves of 64 outputs.  Works on any
    [N, ...] tensors (codes or row-major block scales); N % 64 == 0."""
    if w1.shape != w3.shape or w1.shape[0] % 64:
        raise ValueError("gate and up weights must have equal shapes with N % 64 == 0")
    n = w1.shape[0]
    rest = w1.shape[1:]
    return torch.stack([w1.reshape(n // 64, 64, *rest), w3.reshape(n // 64, 64, *rest)], 1).reshape(2 * n, *rest)


@dataclass
class NVFP4Weight:
    """One NVFP4 weight: codes [N, K/2], block scales (tensor-core layout) and g."""
    codes: torch.Tensor
    scales: torch.Tensor
    global_scale: float
    n: int
    k: int

    @classmethod
    def from_export(cls, packed: torch.Tensor, block_scale: torch.Tensor, global_scale) -> "NVFP4Weight":
        """From the exporter's tensors (``weight``, ``weight.block_scale``, ``weight.global_scale``)."""
        n, half_k = packed.shape
        k = 2 * half_k
        if k % 64:
            raise ValueError("K must be a multiple of 64 for the tensor-core scale layout")
        return cls(packed.contiguous().view(torch.uint8), scales_to_mma(block_scale, k),
                   float(torch.as_tensor(global_scale).float().reshape(-1)[0]), n, k)

    @classmethod
    def from_float(cls, w: torch.Tensor, global_scale: float | None = None) -> "NVFP4Weight":
        """Max-PTQ of a float [N, K] weight on the device: the FP16 matrix the
        exporter quantizes (``export_nvfp4_weights.py:33-36``), g = amax / 2688,
        block scales and codes by the fused quantizer."""
        if w.ndim != 2 or not w.is_cuda:
            raise ValueError("expected a CUDA [N, K] weight")
        wf = w.detach().half().float().contiguous()
        g = weight_global_scale(wf) if global_scale is None else float(global_scale)
        codes, scales = norm_quant(wf, kind="none", fmt="nvfp4_mma", global_scale=g)
        return cls(codes, scales, g, w.shape[0], w.shape[1])


def quantize_activation(x: torch.Tensor, global_scale: float, **norm):
    """Dynamic NVFP4 quantization of activations [..., K] (optionally fused
    with a row norm, see ``norm_quant``): (codes [..., K/2], MMA-layout scales)."""
    return norm_quant(x, kind=norm.pop("kind", "none"), fmt="nvfp4_mma", global_scale=global_scale, **norm)


def nvfp4_gemm(a_codes: torch.Tensor, a_scales: torch.Tensor, a_global: float, weight: NVFP4Weight, *,
               bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
               out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """``(a_global * g_w) * sum_blocks(...) + bias + residual`` for NVFP4 ``a`` [..., K/2]."""
    if out_dtype not in _OUT:
        raise ValueError(f"unsupported output dtype {out_dtype}")
    k = weight.k
    if a_codes.shape[-1] * 2 != k:
        raise ValueError("Input channels differ")
    m = a_codes.numel() // (k // 2)
    lead = a_codes.shape[:-1]
    if a_scales.numel() < mma_scale_bytes(m, k):
        raise ValueError("activation scales are smaller than the tensor-core layout of [M, K]")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != weight.n or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous FP32 tensor of N elements")
    res_dtype = _lib.F32
    if residual is not None:
        if residual.dtype not in (torch.float32, torch.bfloat16) or residual.numel() != m * weight.n:
            raise ValueError("residual must be FP32 or BF16 [..., N]")
        residual = residual.contiguous()
        res_dtype = _lib.F32 if residual.dtype == torch.float32 else _lib.BF16
    y = out if out is not None else torch.empty(*lead, weight.n, device=a_codes.device, dtype=out_dtype)
    alpha = float(torch.tensor(a_global, dtype=torch.float32) * torch.tensor(weight.global_scale, dtype=torch.float32))
    status = _lib.load().isp_nvfp4_gemm(
        a_codes.contiguous().data_ptr(), a_scales.data_ptr(), weight.codes.data_ptr(), weight.scales.data_ptr(),
        m, weight.n, k, alpha, _lib.ptr(bias), _lib.ptr(residual), res_dtype, y.data_ptr(), _OUT[y.dtype],
        _lib.stream_handle(a_codes.device))
    _lib.check(status, "isp_nvfp4_gemm")
    return y


def nvfp4_gated_up(a_codes: torch.Tensor, a_scales: torch.Tensor, a_global: float, w13: NVFP4Weight,
                   g_gate: float, g_up: float, h_global: float, *, h_codes: torch.Tensor | None = None,
                   h_scales: torch.Tensor | None = None):
    """``h = silu(alpha_g A.W1^T) * (alpha_u A.W3^T)`` -> NVFP4 (codes [..., N/2],
    MMA-layout scales) with global scale ``h_global``.  ``w13`` is the stacked
    weight of ``stack_gate_up``; ``g_gate``/``g_up`` are the global scales of
    W1 and W3."""
    n = w13.n // 2
    k = w13.k
    if a_codes.shape[-1] * 2 != k:
        raise ValueError("Input channels differ")
    m = a_codes.numel() // (k // 2)
    lead = a_codes.shape[:-1]
    f32 = lambda v: torch.tensor(v, dtype=torch.float32)
    alpha_g = float(f32(a_global) * f32(g_gate))
    alpha_u = float(f32(a_global) * f32(g_up))
    hc = h_codes if h_codes is not None else torch.empty(*lead, n // 2, device=a_codes.device, dtype=torch.uint8)
    hs = h_scales if h_scales is not None else torch.zeros(mma_scale_bytes(m, n), device=a_codes.device,
                                                           dtype=torch.uint8)
    status = _lib.load().isp_nvfp4_gated_up(
        a_codes.contiguous().data_ptr(), a_scales.data_ptr(), w13.codes.data_ptr(), w13.scales.data_ptr(),
        m, n, k, alpha_g, alpha_u, float(h_global), hc.data_ptr(), hs.data_ptr(), _lib.stream_handle(a_codes.device))
    _lib.check(status, "isp_nvfp4_gated_up")
    return hc, hs


class NVFP4Linear(nn.Module):
    """``MatrixWeightOp(nn.Linear).apply_nvfp4(activation_amax)`` (linear
    geometry): y = nvfp4_gemm(quantize(x)) + bias in FP32.  K is padded to a
    multiple of 64 (the reference pads to 16, ``nvfp4_graph.py:34``; the extra
    zero columns change nothing)."""

    def __init__(self, module: nn.Linear, activation_amax, *, weight: NVFP4Weight | None = None):
        super().__init__()
        w = module.weight.detach().float()
        self.logical_k = w.shape[1]
        self.padded_k = (self.logical_k + 63) // 64 * 64
        self.out_features = w.shape[0]
        self.a_global = activation_global_scale(activation_amax)
        if weight is None:
            weight = NVFP4Weight.from_float(torch.nn.functional.pad(w, (0, self.padded_k - self.logical_k)))
        self.weight_q = weight
        self.register_buffer("bias", None if module.bias is None else module.bias.detach().float().clone())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.logical_k:
            raise ValueError("Input channels differ")
        if self.padded_k != self.logical_k:
            x = torch.nn.functional.pad(x, (0, self.padded_k - self.logical_k))
        if x.dtype not in (torch.bfloat16, torch.float32):
            x = x.float()
        codes, scales = quantize_activation(x, self.a_global)
        return nvfp4_gemm(codes, scales, self.a_global, self.weight_q, bias=self.bias, out_dtype=torch.float32)


class NVFP4GatedUp(nn.Module):
    """CFM feed-forward under NVFP4: x -> [norm] NVFP4 quant -> gated-up (SwiGLU +
    NVFP4 requant of h, one kernel) -> down GEMM (BF16 or FP32 out)."""

    def __init__(self, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, x_amax, h_amax):
        super().__init__()
        q1, q3 = NVFP4Weight.from_float(w1), NVFP4Weight.from_float(w3)
        self.g_gate, self.g_up = q1.global_scale, q3.global_scale
        n, k = w1.shape
        codes = stack_gate_up(q1.codes, q3.codes)
        # re-derive row-major scales per weight and stack them in the same 64-row blocks
        s1 = _rows_from_mma(q1.scales, n, k)
        s3 = _rows_from_mma(q3.scales, n, k)
        self.w13 = NVFP4Weight(codes, scales_to_mma(stack_gate_up(s1, s3), k), 1.0, 2 * n, k)
        self.w2 = NVFP4Weight.from_float(w2)
        self.x_global = activation_global_scale(x_amax)
        self.h_global = activation_global_scale(h_amax)

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16, **norm) -> torch.Tensor:
        codes, scales = quantize_activation(x, self.x_global, **norm)
        hc, hs = nvfp4_gated_up(codes, scales, self.x_global, self.w13, self.g_gate, self.g_up, self.h_global)
        return nvfp4_gemm(hc, hs, self.h_global, self.w2, out_dtype=out_dtype)


def _rows_from_mma(scales: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Inverse of ``scales_to_mma`` (host-side index arithmetic on the device tensor)."""
    kb = k // 16
    r = torch.arange(rows, device=scales.device)[:, None]
    c = torch.arange(kb, device=scales.device)[None, :]
    off = ((r // 128) * (kb // 4) + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4
    return scales[off]
