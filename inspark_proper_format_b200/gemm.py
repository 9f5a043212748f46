"""W8A8 scaled GEMMs on tcgen05 (torch-level wrappers over ``isp_scaled_gemm`` /
``isp_gated_up``) and the reference's module-level surfaces built on them.

Reference surfaces mirrored here:
  * ``linear(x, packed, scales, bias, tile)`` — ``ops/triton/fp8.py:47-63``
    (dynamic per-row E4M3 quant + FP8 GEMM, output in x's dtype);
  * ``GatedUp(weights, config)``              — ``ops/triton/cfm_gated_up.py:30-51``;
  * ``FP8Linear(original, input_scale, weight_scale)`` — ``runtime/zipvoice_fp8/quantization.py:64-82``;
  * ``Int8SmoothQuantLinear(original, spec)`` — the INT8 branch of
    ``ExportWeightOp`` (``build/unified_acoustic_export.py:104-112, 160-204``);
  * ``fused_projection_residual``             — ``ops/tensorrt/zipvoice_fp8_b128/b128/residual_kernel.py:4-11``;
  * ``i8_residual``                           — ``ops/tensorrt/zipvoice/a1007/b1/i8_residual_runtime_kernel.py:5-21``;
  * ``int8_nonlinear_value``                  — ``ops/tensorrt/zipvoice/a1007/b1/int8_nonlinear_value_runtime_kernel.py:6-34``
    (plugin contract ``int8_nonlinear_value_plugin.py:7-35``).
"""
from __future__ import annotations

import weakref

import torch

from . import _lib
from .norm_quant import norm_quant

_OUT = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16, torch.float32: _lib.F32,
        torch.float8_e4m3fn: _lib.E4M3}


def _vec(t, n, name):
    if t is None:
        return None
    if t.dtype != torch.float32 or not t.is_cuda or t.numel() != n or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA FP32 tensor of {n} elements")
    return t


def scaled_gemm(a: torch.Tensor, w: torch.Tensor, *, a_scale: float = 1.0,
                a_scale_rows: torch.Tensor | None = None, w_scale: torch.Tensor | None = None,
                bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.bfloat16, out_inv_scale: float = 1.0,
                dual_inv_scale: float | None = None, out: torch.Tensor | None = None):
    """``epilogue(a @ w.T)`` for 8-bit codes ``a`` [..., K] and ``w`` [N, K].

    ``a``/``w`` are both float8_e4m3fn (FP32 accumulate) or both int8 (int32
    accumulate).  v = ((acc * a_s) * w_scale[n]) + bias[n] + residual (INT8:
    acc * (a_s * w_scale[n])).  With ``out_dtype=float8_e4m3fn`` the result is
    ``e4m3(clamp(v * out_inv_scale))``.  With ``dual_inv_scale`` a second E4M3
    output ``e4m3(clamp(v * dual_inv_scale))`` is returned as well.
    """
    if a.dtype != w.dtype or a.dtype not in (torch.float8_e4m3fn, torch.int8):
        raise ValueError("operands must both be float8_e4m3fn or both int8")
    if not (a.is_cuda and w.is_cuda) or w.ndim != 2:
        raise ValueError("expected CUDA operands and a 2-D [N, K] weight")
    a = a.contiguous()
    w = w.contiguous()
    n, k = w.shape
    if a.shape[-1] != k:
        raise ValueError("Input channels differ")
    m = a.numel() // k
    if out_dtype not in _OUT:
        raise ValueError(f"unsupported output dtype {out_dtype}")
    lead = a.shape[:-1]
    if out is None:
        out = torch.empty(*lead, n, device=a.device, dtype=out_dtype)
    if a_scale_rows is not None:
        a_scale_rows = _vec(a_scale_rows.reshape(-1), m, "a_scale_rows")
    w_scale = _vec(w_scale, n, "w_scale")
    bias = _vec(bias, n, "bias")
    res_dtype = _lib.F32
    if residual is not None:
        if residual.shape[-1] != n or residual.numel() != m * n or residual.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("residual must be [..., N] FP32 or BF16")
        residual = residual.contiguous()
        res_dtype = _lib.F32 if residual.dtype == torch.float32 else _lib.BF16
    out2 = None
    if dual_inv_scale is not None:
        out2 = torch.empty(*lead, n, device=a.device, dtype=torch.float8_e4m3fn)
    status = _lib.load().isp_scaled_gemm(
        a.data_ptr(), w.data_ptr(), _lib.E4M3 if a.dtype == torch.float8_e4m3fn else _lib.I8, m, n, k,
        float(a_scale), _lib.ptr(a_scale_rows), _lib.ptr(w_scale), _lib.ptr(bias), _lib.ptr(residual), res_dtype,
        out.data_ptr(), _OUT[out_dtype], float(out_inv_scale), _lib.ptr(out2),
        float(dual_inv_scale or 0.0), _lib.stream_handle(a.device))
    _lib.check(status, "isp_scaled_gemm")
    return (out, out2) if out2 is not None else out


def gated_up(a: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor | None, s1: torch.Tensor,
             s3: torch.Tensor | None, output_scale: float, *, dequant: bool = True,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU gated-up on E4M3 codes: ``silu(a.w1^T s1) * (a.w3^T s3)`` requantized
    with ``e4m3(clamp(h * (1/output_scale)))``; FP32 ``q * output_scale`` when
    ``dequant`` (``_paired``'s DEQUANT), else the E4M3 codes.  ``w3=None``
    selects the interleaved layout (``w1`` is [2N, K], row 2n = gate n)."""
    if a.dtype != torch.float8_e4m3fn or w1.dtype != torch.float8_e4m3fn:
        raise ValueError("gated-up operands are E4M3 codes")
    a = a.contiguous()
    k = a.shape[-1]
    interleaved = w3 is None
    n = w1.shape[0] // 2 if interleaved else w1.shape[0]
    if w1.shape[1] != k or (not interleaved and tuple(w3.shape) != tuple(w1.shape)):
        raise ValueError("Input channels differ")
    m = a.numel() // k
    s1 = _vec(s1, 2 * n if interleaved else n, "s1")
    s3 = None if interleaved else _vec(s3, n, "s3")
    dtype = torch.float32 if dequant else torch.float8_e4m3fn
    if out is None:
        out = torch.empty(*a.shape[:-1], n, device=a.device, dtype=dtype)
    status = _lib.load().isp_gated_up(
        a.data_ptr(), w1.contiguous().data_ptr(), None if interleaved else w3.contiguous().data_ptr(),
        int(interleaved), m, n, k, s1.data_ptr(), _lib.ptr(s3), float(output_scale), out.data_ptr(),
        _lib.F32 if dequant else _lib.E4M3, _lib.stream_handle(a.device))
    _lib.check(status, "isp_gated_up")
    return out


# ---------------------------------------------------------------------------
# Weight layouts
# ---------------------------------------------------------------------------
def pack_weight(weight: torch.Tensor):
    """Per-output-channel E4M3 weight quantization (``quantization/weights.py:5-17``).

    Returns the reference's packed layout ``[K, pad32(N)]`` and the FP32
    scales [N], exactly as the reference computes them.
    """
    w = weight.detach().float()
    scale = (w.abs().amax(1) / 448).clamp_min(1e-12)
    n, k = w.shape
    packed = torch.zeros(k, ((n + 31) // 32) * 32, device=w.device, dtype=torch.float8_e4m3fn)
    packed[:, :n].copy_((w / scale[:, None]).to(torch.float8_e4m3fn).t())
    return packed, scale


_CANONICAL: dict = {}


def canonical_weight(packed: torch.Tensor, n: int) -> torch.Tensor:
    """[K, Npad] reference packing -> the K-major [N, K] operand tcgen05 reads.

    The transpose is done once per packed tensor object and cached; the entry
    is keyed by object identity and invalidated when the tensor is freed or
    modified in place (its version counter changes)."""
    key = (id(packed), n)
    hit = _CANONICAL.get(key)
    if hit is not None:
        ref, version, canon = hit
        if ref() is packed and version == packed._version:
            return canon
    canon = packed[:, :n].t().contiguous()
    _CANONICAL[key] = (weakref.ref(packed, lambda _r, k=key: _CANONICAL.pop(k, None)), packed._version, canon)
    return canon


def linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None = None,
           tile=None, return_kernel: bool = False):
    """Drop-in for ``ops.triton.fp8.linear``: dynamic per-row E4M3 quantization
    (``max(amax/448, 1e-12)``), FP8 GEMM with FP32 accumulation, epilogue
    ``acc*sa[m]*sb[n] (+bias)``, output in ``x.dtype``.  ``tile`` is accepted
    for signature compatibility; the sm_100a kernel has one schedule."""
    k, n = packed.shape[0], scales.numel()
    x = x.contiguous()
    flat = x.view(-1, k)
    q, sx = norm_quant(flat, kind="none", fmt="e4m3_row")
    w = canonical_weight(packed, n)
    out_dtype = x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
    out = scaled_gemm(q, w, a_scale_rows=sx, w_scale=scales.float().contiguous(),
                      bias=None if bias is None else bias.float().contiguous(), out_dtype=out_dtype)
    output = out.view(*x.shape[:-1], n)
    return (output, None) if return_kernel else output


class GatedUp:
    """Drop-in for ``ops/triton/cfm_gated_up.py:30-51``."""

    def __init__(self, weights, config=None):
        self.config = config
        self.input_scale = float(weights["input_scale"])
        self.output_scale = float(weights["output_scale"])
        self.weights = []
        self.scales = []
        for name in ("w1", "w3"):
            w = torch.as_tensor(weights[name].copy() if hasattr(weights[name], "copy") else weights[name],
                                device="cuda", dtype=torch.float32)
            s = torch.as_tensor(weights[name + "_scale"].copy() if hasattr(weights[name + "_scale"], "copy")
                                else weights[name + "_scale"], device="cuda", dtype=torch.float32)
            self.weights.append((w / s[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).contiguous())
            self.scales.append((s * self.input_scale).contiguous())
        self.output = None

    def __call__(self, x):
        if not x.is_contiguous() or x.dtype != torch.float32:
            raise ValueError("Expected contiguous FP32 CFM normalized input")
        n, k = self.weights[0].shape
        if x.shape[-1] != k:
            raise ValueError("Input channels differ")
        a, _ = norm_quant(x, kind="none", fmt="e4m3", scale=self.input_scale)
        if self.output is None or self.output.shape != (*x.shape[:-1], n):
            self.output = torch.empty((*x.shape[:-1], n), device=x.device, dtype=torch.float32)
        return gated_up(a, self.weights[0], self.weights[1], self.scales[0], self.scales[1], self.output_scale,
                        dequant=True, out=self.output)


def fp8_gated_up_plugin(x_codes, w1, w3, s1, s3, input_scale: float, output_scale: float):
    """``inspark_custom::fp8_gated_up`` contract (``ops/tensorrt/cfm_gated_up_plugin.py:33-49``):
    E4M3 inputs/weights, ``s = w_scale * input_scale``, E4M3 output codes."""
    return gated_up(x_codes, w1, w3, s1, s3, output_scale, dequant=False)


def fp8_gated_up_interleaved_plugin(x_codes, w, s, input_scale: float, output_scale: float):
    """``inspark_custom::fp8_gated_up_interleaved`` (``ops/tensorrt/cfm_interleaved_plugin.py:15-41``)."""
    if w.shape[0] % 2 or s.numel() != w.shape[0]:
        raise ValueError("Interleaved gate/up geometry mismatch")
    return gated_up(x_codes, w, None, s, None, output_scale, dequant=False)


class FP8Linear(torch.nn.Module):
    """ZipVoice static W8A8 E4M3 projection (``runtime/zipvoice_fp8/quantization.py:64-82``):
    per-tensor input scale, per-tensor weight scale, FP32 bias, FP32 output."""

    def __init__(self, original, input_scale, weight_scale):
        super().__init__()
        device = original.weight.device
        self.register_buffer("input_scale", torch.tensor(input_scale, dtype=torch.float32, device=device))
        self.register_buffer("weight_scale", torch.tensor(weight_scale, dtype=torch.float32, device=device))
        weight = (original.weight.detach().float() / self.weight_scale).clamp(-448, 448)
        self.register_buffer("weight_fp8", weight.to(torch.float8_e4m3fn).contiguous())
        self.register_buffer("bias", original.bias.detach().float().clone() if original.bias is not None else None)
        self._w_scale_vec = None

    def forward(self, x):
        n = self.weight_fp8.shape[0]
        if self._w_scale_vec is None or self._w_scale_vec.device != x.device:
            self._w_scale_vec = self.weight_scale.reshape(1).expand(n).contiguous().to(x.device)
        a, _ = norm_quant(x.float(), kind="none", fmt="e4m3", scale=float(self.input_scale))
        return scaled_gemm(a, self.weight_fp8, a_scale=float(self.input_scale), w_scale=self._w_scale_vec,
                           bias=self.bias, out_dtype=torch.float32)


class Int8SmoothQuantLinear(torch.nn.Module):
    """INT8 SmoothQuant linear with the reference's role spec (schema 1):
    ``smooth_scale`` [K], ``input_scale``, per-output ``weight_scale`` [N]
    (``build/unified_acoustic_export.py:104-112, 160-204``;
    ``scripts/export_weights.py:56-64``).  Weights are smoothed and quantized
    once; activations are divided by ``smooth`` inside the quant kernel."""

    def __init__(self, original, spec):
        super().__init__()
        w = original.weight.detach().float()
        device = w.device
        smooth = torch.as_tensor(spec["smooth_scale"], dtype=torch.float32, device=device)
        w = w * smooth[None, :]
        ws = torch.as_tensor(spec["weight_scale"], dtype=torch.float32, device=device).reshape(-1)
        if ws.numel() == 1:
            ws = ws.expand(w.shape[0]).contiguous()
        self.register_buffer("smooth_scale", smooth.contiguous())
        self.register_buffer("weight_scale", ws.contiguous())
        self.register_buffer("weight_q", (w / ws[:, None]).round().clamp(-128, 127).to(torch.int8).contiguous())
        self.register_buffer("bias", original.bias.detach().float().clone() if original.bias is not None else None)
        self.input_scale = float(spec["input_scale"])

    def forward(self, x, residual=None):
        a, _ = norm_quant(x, kind="none", fmt="int8", scale=self.input_scale, smooth=self.smooth_scale)
        return scaled_gemm(a, self.weight_q, a_scale=self.input_scale, w_scale=self.weight_scale,
                           bias=self.bias, residual=residual, out_dtype=torch.float32)


def fused_projection_residual(a_codes, w_codes, bias, residual, alpha: float, inv: float):
    """``FusedProjectionResidual`` plugin: ``z = acc*Alpha + bias + R``; returns
    (FP32 z, E4M3 codes of clamp(z * Inv))."""
    return scaled_gemm(a_codes, w_codes, a_scale=float(alpha), bias=bias, residual=residual,
                       out_dtype=torch.float32, dual_inv_scale=float(inv))


def i8_residual(q, w, a_scale: float, w_scale, bias, residual):
    """``i8_residual``: ``acc.to(f32) * (AS * WS[n]) + bias + R``, FP32 output."""
    return scaled_gemm(q, w, a_scale=float(a_scale), w_scale=w_scale, bias=bias, residual=residual,
                       out_dtype=torch.float32)


def int8_nonlinear_value(q, w, input_scale: float, weight_scale, bias, *, value=None, gate=None):
    """ZipVoice INT8 nonlinear-attention in_proj with its tanh/value/gate boundary
    (``zipvoice_int8_b*::OriginalInt8NonlinearValue*``): ``q`` [T, B, K] int8,
    ``w`` [3N, K] int8 (the three projections stacked), FP32 ``weight_scale`` and
    ``bias`` [3N], per-tensor ``input_scale``.  ``z_j = acc_j * (AS * WS[jN+n]) +
    bias[jN+n]``; returns ``value = tanh(z0) * z1`` as [1, B, T, N] and ``gate = z2``
    as [T, B, N], both FP32 (the plugin's output descriptors)."""
    if q.dtype != torch.int8 or w.dtype != torch.int8 or q.ndim != 3 or w.ndim != 2:
        raise ValueError("expected int8 q [T, B, K] and int8 w [3N, K]")
    steps, groups, k = q.shape
    if w.shape[1] != k or w.shape[0] % 3:
        raise ValueError("Input channels differ")
    n = w.shape[0] // 3
    weight_scale = _vec(weight_scale.reshape(-1), 3 * n, "weight_scale")
    bias = _vec(bias.reshape(-1), 3 * n, "bias")
    if value is None:
        value = torch.empty(1, groups, steps, n, device=q.device, dtype=torch.float32)
    if gate is None:
        gate = torch.empty(steps, groups, n, device=q.device, dtype=torch.float32)
    status = _lib.load().isp_int8_nonlinear_value(
        q.contiguous().data_ptr(), w.contiguous().data_ptr(), steps * groups, n, k, groups, float(input_scale),
        weight_scale.data_ptr(), bias.data_ptr(), value.data_ptr(), gate.data_ptr(), _lib.stream_handle(q.device))
    _lib.check(status, "isp_int8_nonlinear_value")
    return value, gate
