"""Loader for the reference's exported quantized checkpoints (safetensors + JSON
role manifest), mapping every linear role onto this package's kernels.

Formats read unchanged:
  * FP8 / INT8 / BF16 roles (``scripts/export_weights.py:38-75``): per component
    ``<variant>/<component>.safetensors`` + ``<variant>/<component>.json`` with
    ``roles[role] = {precision, state_key, weight_scale, input_scale,
    [smooth_scale], weight_axis, weight_input_axis, stored_layout, ...}``; the
    state dict holds ``<key>`` (codes: float8_e4m3fn or int8, canonical [N, K];
    INT8 codes already multiplied by the smoothing factors before scaling),
    ``<key>.weight_scale`` [N], ``<key>.input_scale`` [], ``<key>.smooth_scale``
    [K] (INT8).
  * NVFP4 roles (``scripts/export_nvfp4_weights.py:25-46``): ``<key>`` uint8
    [N, K/2] (low nibble = even K), ``<key>.block_scale`` E4M3 [N, K/16],
    ``<key>.global_scale`` [], ``<key>.activation_global_scale`` [].
  * The role artifact itself (``quantization/unified.py:209-239``, schema 1) is
    validated by ``check_artifact`` with the reference's rules.
Biases are not role tensors: they stay under ``<key minus .weight>.bias`` in the
same state dict (non-role parameters keep their original dtype and values).
Convolution roles (3-D weights, codes in the module's own layout: Conv1d [CO, CI, KW],
ConvTranspose1d [CI, CO, KW]) run on the implicit-GEMM conv kernels
(``ExportedConv1d``); the manifest does not carry a convolution's stride, padding or
dilation, so ``build_roles`` maps a conv role only when the caller supplies that
geometry (from the model's module) and otherwise reports it.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import torch
from torch import nn

from . import conv, gemm, nvfp4
from .norm_quant import norm_quant

PRECISIONS = ("bf16", "fp8", "int8", "nvfp4")


def check_artifact(payload: dict, quant_format: str | None = None) -> dict:
    """The validation of ``load_artifact`` (``quantization/unified.py:209-239``)."""
    if payload.get("schema") != 1 or not payload.get("role_specs"):
        raise ValueError("Invalid unified quantization artifact")
    if quant_format and payload["scheme"] != quant_format:
        raise ValueError("Quantization artifact precision mismatch")
    for name, spec in payload["role_specs"].items():
        if spec.get("precision") not in PRECISIONS:
            raise ValueError(f"Invalid role precision: {name}")
        if spec["precision"] == "nvfp4":
            if not math.isfinite(spec["activation_amax"]) or spec["activation_amax"] <= 0 or spec["block_size"] != 16:
                raise ValueError(f"Invalid NVFP4 role: {name}")
        if spec["precision"] in ("fp8", "int8"):
            if not math.isfinite(spec["input_scale"]) or spec["input_scale"] <= 0:
                raise ValueError(f"Invalid activation scale: {name}")
            scales = spec["weight_scale"] if isinstance(spec["weight_scale"], list) else [spec["weight_scale"]]
            if not scales or any(not math.isfinite(v) or v <= 0 for v in scales):
                raise ValueError(f"Invalid weight scales: {name}")
            ia, oa = spec.get("weight_input_axis"), spec.get("weight_axis")
            if ia is not None or oa is not None:
                if type(ia) is not int or type(oa) is not int or {ia, oa} != {0, 1}:
                    raise ValueError(f"Invalid weight channel axes: {name}")
            if spec["precision"] == "int8":
                smooth = spec.get("smooth_scale")
                if not isinstance(smooth, list) or not smooth or any(not math.isfinite(v) or v <= 0 for v in smooth):
                    raise ValueError(f"Invalid smoothing scales: {name}")
    return payload


class ExportedLinear(nn.Module):
    """One exported linear role, run on this package's kernels.

    fp8:   x -> E4M3 with the calibrated input scale -> tcgen05 FP8 GEMM
           (``acc * input_scale * weight_scale[n] + bias``), the ``_QDQ`` +
           ``F.linear`` of the reference's export graph;
    int8:  x -> ``rne(x / smooth / input_scale)`` INT8 -> tcgen05 INT8 GEMM
           (``acc * (input_scale * weight_scale[n]) + bias``);
    nvfp4: x -> NVFP4 with the activation global scale -> block-scaled GEMM;
    bf16:  ``F.linear`` in BF16 (protected roles).
    The output dtype follows ``out_dtype`` (default: the input's)."""

    def __init__(self, role: str, meta: dict, state: dict, device="cuda"):
        super().__init__()
        self.role = role
        self.precision = meta["precision"]
        key = meta["state_key"]
        w = state[key]
        if w.ndim != 2:
            raise ValueError(f"{role}: {w.ndim}-D weight is a convolution role, not a linear one")
        bias_key = key[: -len(".weight")] + ".bias" if key.endswith(".weight") else None
        b = state.get(bias_key) if bias_key else None
        self.register_buffer("bias", None if b is None else b.detach().float().to(device).contiguous())
        self.out_features = w.shape[0]
        if self.precision == "fp8":
            self.weight = w.to(device).contiguous()
            self.weight_scale = state[key + ".weight_scale"].float().reshape(-1).to(device).contiguous()
            self.input_scale = float(state[key + ".input_scale"])
            self.in_features = w.shape[1]
        elif self.precision == "int8":
            self.weight = w.to(device).contiguous()
            self.weight_scale = state[key + ".weight_scale"].float().reshape(-1).to(device).contiguous()
            self.input_scale = float(state[key + ".input_scale"])
            self.smooth = state[key + ".smooth_scale"].float().reshape(-1).to(device).contiguous()
            self.in_features = w.shape[1]
        elif self.precision == "nvfp4":
            self.weight = nvfp4.NVFP4Weight.from_export(w.to(device), state[key + ".block_scale"].to(device),
                                                        state[key + ".global_scale"])
            self.activation_global = float(state[key + ".activation_global_scale"])
            self.in_features = self.weight.k
        elif self.precision == "bf16":
            self.weight = w.to(device).bfloat16().contiguous()
            self.in_features = w.shape[1]
        else:
            raise ValueError(f"{role}: unknown precision {self.precision!r}")
        if self.weight_scale_count() not in (0, self.out_features):
            raise ValueError(f"{role}: weight_scale does not match the output channels")

    def weight_scale_count(self) -> int:
        return self.weight_scale.numel() if self.precision in ("fp8", "int8") else 0

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        dtype = out_dtype or (x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32)
        if x.shape[-1] != self.in_features:
            raise ValueError("Input channels differ")
        if self.precision == "bf16":
            y = torch.nn.functional.linear(x.bfloat16(), self.weight,
                                           None if self.bias is None else self.bias.bfloat16())
            return y.to(dtype)
        xin = x if x.dtype in (torch.bfloat16, torch.float32) else x.float()
        if self.precision == "nvfp4":
            codes, scales = nvfp4.quantize_activation(xin, self.activation_global)
            return nvfp4.nvfp4_gemm(codes, scales, self.activation_global, self.weight, bias=self.bias,
                                    out_dtype=dtype)
        if self.precision == "fp8":
            codes, _ = norm_quant(xin, kind="none", fmt="e4m3", scale=self.input_scale)
        else:
            codes, _ = norm_quant(xin, kind="none", fmt="int8", scale=self.input_scale, smooth=self.smooth)
        return gemm.scaled_gemm(codes, self.weight, a_scale=self.input_scale, w_scale=self.weight_scale,
                                bias=self.bias, out_dtype=dtype)


class ExportedConv1d(nn.Module):
    """One exported convolution role on the implicit-GEMM conv kernels.

    geometry: ``stride``, ``padding``, ``dilation``, ``output_padding`` (default 0)
    and ``transposed`` of the model's Conv1d / ConvTranspose1d.  fp8 / int8 roles:
    static input quantization with the calibrated ``input_scale`` (INT8: x divided by
    ``smooth_scale`` first; the exporter already folded it into the codes), then
    ``acc * input_scale * weight_scale[co] + bias`` -- ``ExportWeightOp.forward`` for
    conv roles (``build/unified_acoustic_export.py:156-216``); bf16 roles run
    ``F.conv1d`` / ``F.conv_transpose1d`` in BF16."""

    def __init__(self, role: str, meta: dict, state: dict, geometry: dict, device="cuda"):
        super().__init__()
        self.role = role
        self.precision = meta["precision"]
        key = meta["state_key"]
        w = state[key]
        if w.ndim != 3:
            raise ValueError(f"{role}: {w.ndim}-D weight is not a convolution role")
        self.transposed = bool(geometry.get("transposed", False))
        self.stride = int(geometry.get("stride", 1))
        self.padding = int(geometry.get("padding", 0))
        self.dilation = int(geometry.get("dilation", 1))
        self.output_padding = int(geometry.get("output_padding", 0))
        ci, co = (w.shape[0], w.shape[1]) if self.transposed else (w.shape[1], w.shape[0])
        self.in_channels, self.out_channels, self.kernel_size = ci, co, w.shape[2]
        bias_key = key[: -len(".weight")] + ".bias" if key.endswith(".weight") else None
        b = state.get(bias_key) if bias_key else None
        self.register_buffer("bias", None if b is None else b.detach().float().to(device).contiguous())
        if self.precision == "bf16":
            self.weight = w.to(device).bfloat16().contiguous()
            return
        if self.precision not in ("fp8", "int8"):
            raise ValueError(f"{role}: unsupported convolution precision {self.precision!r}")
        out_axis = 1 if self.transposed else 0
        if int(meta.get("weight_axis", out_axis)) != out_axis:
            raise ValueError(f"{role}: weight scales must be per output channel")
        dense = w.permute(1, 0, 2) if self.transposed else w                     # [CO, CI, KW] codes
        codes_kn = dense.reshape(co, ci * self.kernel_size).t().contiguous().to(device)
        self.weight = conv.pack_folded(codes_kn.view(torch.uint8), co, ci, self.kernel_size, self.stride,
                                       self.dilation, self.padding, self.transposed)
        ws = state[key + ".weight_scale"].float().reshape(-1)
        self.weight_scale = (ws.expand(co) if ws.numel() == 1 else ws).to(device).contiguous()
        if self.weight_scale.numel() != co:
            raise ValueError(f"{role}: weight_scale does not match the output channels")
        self.input_scale = float(state[key + ".input_scale"])
        sm = state.get(key + ".smooth_scale") if self.precision == "int8" else None
        self.smooth = None if sm is None else sm.float().reshape(-1).to(device).contiguous()

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        dtype = out_dtype or (x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32)
        if x.ndim != 3 or x.shape[1] != self.in_channels:
            raise ValueError("Input channels changed")
        if self.precision == "bf16":
            bias = None if self.bias is None else self.bias.bfloat16()
            if self.transposed:
                y = torch.nn.functional.conv_transpose1d(x.bfloat16(), self.weight, bias, self.stride, self.padding,
                                                         self.output_padding, 1, self.dilation)
            else:
                y = torch.nn.functional.conv1d(x.bfloat16(), self.weight, bias, self.stride, self.padding,
                                               self.dilation)
            return y.to(dtype)
        return conv.run(x, self.weight, self.weight_scale, self.bias, ci=self.in_channels, co=self.out_channels,
                        kw=self.kernel_size, stride=self.stride, padding=self.padding, dilation=self.dilation,
                        transpose=self.transposed, output_padding=self.output_padding, code=self.precision,
                        in_scale=self.input_scale, smooth=self.smooth, out_dtype=dtype)


def build_roles(meta: dict, state: dict, device="cuda", conv_geometry: dict | None = None):
    """Map a component manifest (``meta['roles']``) and its state dict onto
    ExportedLinear / ExportedConv1d modules; ``conv_geometry`` = {role: geometry}
    for the convolution roles (see ExportedConv1d).  Returns ({role: module},
    {role: reason} for roles left unmapped, i.e. convolutions without geometry)."""
    roles, skipped = {}, {}
    for role, spec in meta["roles"].items():
        if spec["precision"] not in PRECISIONS:
            raise ValueError(f"Invalid role precision: {role}")
        w = state.get(spec["state_key"])
        if w is None:
            raise KeyError((role, spec["state_key"]))
        if w.ndim == 3:
            if conv_geometry and role in conv_geometry:
                roles[role] = ExportedConv1d(role, spec, state, conv_geometry[role], device)
            else:
                skipped[role] = "3-D weight (convolution role) without its stride / padding / dilation"
            continue
        if w.ndim != 2:
            skipped[role] = f"{w.ndim}-D weight"
            continue
        roles[role] = ExportedLinear(role, spec, state, device)
    return roles, skipped


def load_component_bytes(data: bytes, meta: dict, device="cuda", conv_geometry: dict | None = None):
    """``build_roles`` over a component's safetensors bytes."""
    from safetensors.torch import load
    return build_roles(meta, load(data), device, conv_geometry)


def load_component(safetensors_path, manifest_path=None, device="cuda", conv_geometry: dict | None = None):
    """Read one exported component (``<component>.safetensors`` and its
    ``<component>.json`` manifest beside it)."""
    safetensors_path = Path(safetensors_path)
    manifest_path = Path(manifest_path) if manifest_path else safetensors_path.with_suffix(".json")
    return load_component_bytes(safetensors_path.read_bytes(), json.loads(manifest_path.read_text()), device,
                                conv_geometry)
