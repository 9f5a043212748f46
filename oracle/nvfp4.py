"""Oracle for the NVFP4 (E2M1, 16-element K blocks, E4M3 block scales, FP32
global scale) GEMM and gated-up epilogue (numpy).

The reference runs NVFP4 through NVIDIA ModelOpt 0.47 quantizers and
TensorRT's native FP4 GEMM (``build/nvfp4_graph.py:73-87``,
``quantization/nvfp4.py:11-79``); neither is in the reference tree.  This
module restates the published two-level scheme recorded by the reference's
exporter (``scripts/export_nvfp4_weights.py:25-42``):

* weight global scale ``g_w = amax(W) / (6 * 448)``;
* activation global scale ``g_a = fp16(activation_amax) / (6 * 448)``
  (``scripts/export_nvfp4_weights.py:39``);
* block scale ``s_b = e4m3(amax_b / (6 * g))`` and codes
  ``e2m1(x / (s_b * g))`` (see ``normquant.quant_nvfp4``).

Parity against ModelOpt itself is unpinned.
"""
from __future__ import annotations

import numpy as np

from .formats import E4M3_MAX, e2m1_decode, e4m3_decode, e4m3_encode, unpack_nibbles
from .normquant import quant_nvfp4


def weight_global_scale(w: np.ndarray) -> np.float32:
    return np.float32(np.abs(np.asarray(w, np.float32)).max() / np.float32(6.0 * 448.0))


def activation_global_scale(activation_amax: float) -> np.float32:
    return np.float32(np.float32(np.float16(activation_amax)) / np.float32(6.0 * 448.0))


def quantize_weight(w: np.ndarray, global_scale=None):
    """[N, K] weight -> (packed uint8 [N, K/2], E4M3 block scales [N, K/16], g)."""
    w = np.asarray(w, np.float32)
    g = weight_global_scale(w) if global_scale is None else np.float32(global_scale)
    packed, scodes = quant_nvfp4(w, g)
    return packed, scodes, g


def dequantize(packed: np.ndarray, scodes: np.ndarray, g) -> np.ndarray:
    vals = e2m1_decode(unpack_nibbles(packed)).astype(np.float64)
    s = e4m3_decode(scodes).astype(np.float64)
    k = vals.shape[-1]
    vals = vals.reshape(vals.shape[:-1] + (k // 16, 16)) * s[..., None]
    return vals.reshape(vals.shape[:-2] + (k,)) * float(g)


def block_accumulate(a_packed, a_scodes, w_packed, w_scodes) -> np.ndarray:
    """sum over K of (e2m1_a * s_a_block) * (e2m1_w * s_w_block), exactly (float64)."""
    a = dequantize(a_packed, a_scodes, 1.0)
    w = dequantize(w_packed, w_scodes, 1.0)
    return a @ w.T


def nvfp4_gemm(a_packed, a_scodes, g_a, w_packed, w_scodes, g_w, bias=None):
    """``y = sum_blocks(e2m1_a e2m1_w s_a s_w) * (g_a * g_w) (+ bias)`` in FP32."""
    acc = block_accumulate(a_packed, a_scodes, w_packed, w_scodes).astype(np.float32)
    v = (acc * (np.float32(g_a) * np.float32(g_w))).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    return v


def gated_up_nvfp4(a_packed, a_scodes, g_a, w1, w3, out_global_scale):
    """NVFP4 gated-up: two block-scaled GEMMs sharing A, SwiGLU, then NVFP4
    requant of h with the calibrated global scale of the down projection's
    input.  ``w1``/``w3`` are (packed, scodes, g) triples.  Returns
    (packed h [M, N/2], block scales [M, N/16], FP32 h before requant)."""
    gate = nvfp4_gemm(a_packed, a_scodes, g_a, *w1)
    up = nvfp4_gemm(a_packed, a_scodes, g_a, *w3)
    sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-gate))).astype(np.float32)
    h = ((gate * sig).astype(np.float32) * up).astype(np.float32)
    packed, scodes = quant_nvfp4(h, out_global_scale)
    return packed, scodes, h


def sf_to_mma_layout(sf: np.ndarray) -> np.ndarray:
    """Block scales [R, K/16] (row-major, ModelOpt order) -> the tensor-core
    layout: 128-row x 4-block chunks of 512 bytes, K-chunks first, with byte
    ((r//128) * (K/64) + k16//4) * 512 + (r%32)*16 + ((r%128)//32)*4 + k16%4.
    Rows are padded to a multiple of 128 with zero bytes."""
    sf = np.asarray(sf, np.uint8)
    r, kb = sf.shape
    if kb % 4:
        raise ValueError("K must be a multiple of 64")
    rb = (r + 127) // 128
    out = np.zeros(rb * 128 * kb, np.uint8)
    rows = np.arange(r)[:, None]
    ks = np.arange(kb)[None, :]
    off = ((rows // 128) * (kb // 4) + ks // 4) * 512 + (rows % 32) * 16 + ((rows % 128) // 32) * 4 + ks % 4
    out[off] = sf
    return out


def sf_from_mma_layout(tiled: np.ndarray, r: int, kb: int) -> np.ndarray:
    rows = np.arange(r)[:, None]
    ks = np.arange(kb)[None, :]
    off = ((rows // 128) * (kb // 4) + ks // 4) * 512 + (rows % 32) * 16 + ((rows % 128) // 32) * 4 + ks % 4
    return np.asarray(tiled, np.uint8)[off]


def e4m3_static(h: np.ndarray, scale: float) -> np.ndarray:
    return e4m3_encode(np.clip((h / np.float32(scale)).astype(np.float32), -E4M3_MAX, E4M3_MAX))
