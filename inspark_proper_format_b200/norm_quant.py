"""Fused norm -> quantize op (torch-level wrapper over ``isp_norm_quant``).

An op the reference does not have as one call: it fuses the reference's
separate normalization (RMSNorm / Qwen RMSNorm / BiasNorm) and quantization
steps (static E4M3 ``_QDQ``, per-row ``_quantize``, INT8 SmoothQuant, NVFP4
dynamic block quantization) into one memory-bound pass.
"""
from __future__ import annotations

import torch

from . import _lib

KINDS = {"none": _lib.NORM_NONE, "rms_gptfast": _lib.NORM_RMS_GPTFAST,
         "rms_qwen": _lib.NORM_RMS_QWEN, "bias": _lib.NORM_BIAS}
FORMATS = {"e4m3": _lib.Q_E4M3_STATIC, "e4m3_row": _lib.Q_E4M3_ROW,
           "int8": _lib.Q_INT8_STATIC, "nvfp4": _lib.Q_NVFP4, "nvfp4_mma": _lib.Q_NVFP4_MMA}


def mma_scale_bytes(rows: int, k: int) -> int:
    """Bytes of NVFP4 block scales of an [rows, k] operand in the tensor-core
    layout (128-row x 4-block chunks of 512 bytes, rows padded to 128)."""
    return (rows + 127) // 128 * 128 * (k // 16)


def _param(t, k, name):
    if t is None:
        return None
    if t.dtype != torch.float32 or not t.is_cuda or t.numel() != k or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA FP32 tensor of {k} elements")
    return t


def norm_quant(x: torch.Tensor, *, kind: str = "rms_gptfast", fmt: str = "e4m3",
               gamma: torch.Tensor | None = None, bias: torch.Tensor | None = None,
               eps: float = 1e-6, log_scale: torch.Tensor | float | None = None,
               scale: float | None = None, smooth: torch.Tensor | None = None,
               global_scale: float | None = None, out: torch.Tensor | None = None,
               scales_out: torch.Tensor | None = None):
    """Normalize the rows of ``x`` ([..., K], BF16 or FP32) and quantize them.

    Returns ``(codes, scales)``:
      * ``e4m3``: float8_e4m3fn codes of ``clamp(y / scale)``, scales None;
      * ``e4m3_row``: codes and FP32 per-row scales ``max(amax/448, 1e-12)``;
      * ``int8``: int8 codes of ``clamp(rne(y / smooth / scale))``, scales None;
      * ``nvfp4``: uint8 [..., K/2] packed E2M1 (low nibble = even k) and
        float8_e4m3fn [..., K/16] block scales, with ``global_scale`` g;
      * ``nvfp4_mma``: the same codes, the block scales as a flat uint8 tensor
        in the tensor-core layout that ``nvfp4.nvfp4_gemm`` consumes
        (``mma_scale_bytes(M, K)`` bytes; K % 64 == 0).
    """
    if kind not in KINDS or fmt not in FORMATS:
        raise ValueError(f"unknown norm kind {kind!r} or format {fmt!r}")
    if x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda:
        raise ValueError("norm_quant expects a CUDA BF16 or FP32 tensor")
    x = x.contiguous()
    k = x.shape[-1]
    m = x.numel() // k if k else 0
    if k % 16:
        raise ValueError("the quantized dimension must be a multiple of 16")
    gamma = _param(gamma, k, "gamma")
    bias = _param(bias, k, "bias")
    smooth = _param(smooth, k, "smooth")
    out_mul = 1.0
    if kind == "bias":
        ls = log_scale if isinstance(log_scale, torch.Tensor) else torch.tensor(float(log_scale or 0.0))
        out_mul = float(ls.detach().float().exp())
    lead = x.shape[:-1]
    if fmt in ("nvfp4", "nvfp4_mma"):
        if global_scale is None:
            raise ValueError("nvfp4 needs the FP32 global scale")
        s = float(global_scale)
        codes = out if out is not None else torch.empty(*lead, k // 2, device=x.device, dtype=torch.uint8)
        if scales_out is not None:
            scales = scales_out
        elif fmt == "nvfp4":
            scales = torch.empty(*lead, k // 16, device=x.device, dtype=torch.float8_e4m3fn)
        else:
            scales = torch.zeros(mma_scale_bytes(m, k), device=x.device, dtype=torch.uint8)
    else:
        if fmt in ("e4m3", "int8"):
            if scale is None:
                raise ValueError(f"{fmt} needs a calibrated static scale")
            s = float(scale)
        else:
            s = 0.0
        dtype = torch.int8 if fmt == "int8" else torch.float8_e4m3fn
        codes = out if out is not None else torch.empty(*lead, k, device=x.device, dtype=dtype)
        scales = None
        if fmt == "e4m3_row":
            scales = scales_out if scales_out is not None else torch.empty(*lead, device=x.device,
                                                                          dtype=torch.float32)
    status = _lib.load().isp_norm_quant(
        x.data_ptr(), _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F32, m, k,
        _lib.ptr(gamma), _lib.ptr(bias), float(eps), out_mul, KINDS[kind], FORMATS[fmt], s,
        _lib.ptr(smooth), codes.data_ptr(), _lib.ptr(scales), _lib.stream_handle(x.device))
    _lib.check(status, "isp_norm_quant")
    return codes, scales


def quantize_fp8(x: torch.Tensor, input_scale: float) -> torch.Tensor:
    """``inspark_custom::fp8_quantize`` (``ops/tensorrt/cfm_gated_up_plugin.py:17-31``):
    FP32 activation -> E4M3 codes with a static scale; the plugin's int32
    view packs four codes per word (``codes.view(torch.int32)``)."""
    codes, _ = norm_quant(x, kind="none", fmt="e4m3", scale=input_scale)
    return codes


def adaln_quant(x: torch.Tensor, gamma: torch.Tensor, ada_w: torch.Tensor, ada_b: torch.Tensor, *,
                fmt: str = "e4m3", eps: float = 1e-6, scale: float | None = None,
                global_scale: float | None = None, smooth: torch.Tensor | None = None):
    """gpt_fast ``AdaptiveLayerNorm`` fused with the quantizer
    (``gpt_fast/model.py:18-32``): ``ada_w[b] * RMSNorm(x) + ada_b[b]`` for
    ``x`` [B, T, K] (or [B*T, K] with ``ada_w`` [B, K]), then ``fmt`` as in
    ``norm_quant``.  ``ada_w``/``ada_b`` are the split projection of each
    utterance's conditioning embedding, FP32 [B, K]."""
    if fmt not in FORMATS:
        raise ValueError(f"unknown format {fmt!r}")
    if x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda:
        raise ValueError("adaln_quant expects a CUDA BF16 or FP32 tensor")
    x = x.contiguous()
    k = x.shape[-1]
    m = x.numel() // k if k else 0
    ada_w = ada_w.float().reshape(-1, k).contiguous()
    ada_b = ada_b.float().reshape(-1, k).contiguous()
    groups = ada_w.shape[0]
    if ada_b.shape[0] != groups or groups == 0 or m % groups:
        raise ValueError("ada_w/ada_b must hold one [K] row per utterance and divide the rows evenly")
    gamma = _param(gamma, k, "gamma")
    smooth = _param(smooth, k, "smooth")
    lead = x.shape[:-1]
    scales = None
    if fmt in ("nvfp4", "nvfp4_mma"):
        if global_scale is None:
            raise ValueError("nvfp4 needs the FP32 global scale")
        s = float(global_scale)
        codes = torch.empty(*lead, k // 2, device=x.device, dtype=torch.uint8)
        scales = (torch.empty(*lead, k // 16, device=x.device, dtype=torch.float8_e4m3fn) if fmt == "nvfp4"
                  else torch.zeros(mma_scale_bytes(m, k), device=x.device, dtype=torch.uint8))
    else:
        s = float(scale) if fmt in ("e4m3", "int8") else 0.0
        if fmt in ("e4m3", "int8") and scale is None:
            raise ValueError(f"{fmt} needs a calibrated static scale")
        codes = torch.empty(*lead, k, device=x.device, dtype=torch.int8 if fmt == "int8" else torch.float8_e4m3fn)
        if fmt == "e4m3_row":
            scales = torch.empty(*lead, device=x.device, dtype=torch.float32)
    status = _lib.load().isp_adaln_quant(
        x.data_ptr(), _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F32, m, k, gamma.data_ptr(), float(eps),
        ada_w.data_ptr(), ada_b.data_ptr(), m // groups, FORMATS[fmt], s, _lib.ptr(smooth), codes.data_ptr(),
        _lib.ptr(scales), _lib.stream_handle(x.device))
    _lib.check(status, "isp_adaln_quant")
    return codes, scales


def adaptive_layer_norm_quant(module, x: torch.Tensor, embedding: torch.Tensor, **quant):
    """Drop-in for ``AdaptiveLayerNorm(x, embedding)`` followed by its Q/DQ: the
    module's own ``project_layer`` turns the [B, 1, K] embedding into the
    per-utterance (weight, bias); its ``norm`` supplies gamma and eps."""
    if embedding is None:
        return norm_quant(x, kind="rms_gptfast", gamma=module.norm.weight.detach().float(), eps=module.eps, **quant)
    with torch.no_grad():
        w, b = torch.split(module.project_layer(embedding).float(), module.d_model, dim=-1)
    return adaln_quant(x, module.norm.weight.detach().float().contiguous(), w.reshape(-1, module.d_model),
                       b.reshape(-1, module.d_model), eps=module.eps, **quant)
