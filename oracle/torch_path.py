"""The reference's CPU PyTorch path for the headline workload, restated with
the same torch operators — TEST/BASELINE INFRASTRUCTURE ONLY.

Used by ``bench.py`` as the timed CPU baseline (``cpu_baseline`` and
``--impl reference``): the reference cannot be installed on the GPU box, so
its eager path is restated here op for op:

* gpt_fast ``RMSNorm`` (``models/indextts2/upstream/s2mel/modules/gpt_fast/model.py:250-258``);
* static E4M3 ``_QDQ`` (``build/unified_acoustic_export.py:27-33``);
* ``ExportWeightOp.forward`` linear on dequantized operands
  (``build/unified_acoustic_export.py:153-204``), FP32 ``F.linear``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = (xf * torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)).type_as(x)
    return y * weight


def qdq_e4m3(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return (x.float() / scale).clamp(-448, 448).to(torch.float8_e4m3fn).float() * scale


class FP8Layer:
    """One cfg-2 layer: RMSNorm -> E4M3 Q/DQ -> the ten projections, each on Q/DQ'd inputs."""

    def __init__(self, weights, scales, bias=None):
        # weights: list of (W_dequantized FP32 [N, K]); scales: activation scales per GEMM input
        self.weights = weights
        self.scales = scales
        self.bias = bias

    def outputs(self, x, gamma, eps, norm_scale):
        """FP32 outputs of the seven projections whose results leave the layer: the
        three FF outputs, attention in and out, and the convolution output (the
        hidden FF / convolution activations pass through their own Q/DQ)."""
        a = qdq_e4m3(rms_norm(x, gamma, eps), norm_scale)
        w = self.weights
        outs = []
        for f in range(3):
            h = F.linear(a, w[2 * f])
            outs.append(F.linear(qdq_e4m3(h, self.scales[f]), w[2 * f + 1]))
        outs.append(F.linear(a, w[6]))
        outs.append(F.linear(a, w[7]))
        c1 = F.linear(a, w[8])
        outs.append(F.linear(qdq_e4m3(c1, self.scales[3]), w[9]))
        return outs

    def __call__(self, x, gamma, eps, norm_scale):
        return self.outputs(x, gamma, eps, norm_scale)[-1].bfloat16()
