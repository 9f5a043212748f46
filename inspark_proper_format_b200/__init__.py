"""B200 (sm_100a) quantized-linear hot path of the InSpark TTS runtime.

Torch-level ops over the C ABI in ``include/isp_b200.h``:
norm->quantize, W8A8 FP8/INT8 scaled GEMMs with fused epilogues, the CFM
gated-up SwiGLU and the BigVGAN anti-aliased Snake FIR.  Every op runs a
hand-written CUDA kernel; there is no CPU fallback.
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
