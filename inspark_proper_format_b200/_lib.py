"""ctypes binding of ``libisp_b200.so`` (the C ABI declared in include/isp_b200.h).

The library is built in-tree by ``inspark_proper_format_b200.build``.  There is
no fallback: if the shared object is missing, or the current GPU is not an
sm_100 part, every op raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "libisp_b200.so"

ISP_OK, ISP_ERR_SHAPE, ISP_ERR_ALIGN, ISP_ERR_DTYPE, ISP_ERR_ARCH, ISP_ERR_LAUNCH, ISP_ERR_TIMEOUT, ISP_ERR_ARG = range(8)
BF16, F32, F16, E4M3, I8, E2M1, I32 = range(7)
NORM_NONE, NORM_RMS_GPTFAST, NORM_RMS_QWEN, NORM_BIAS = range(4)
Q_E4M3_STATIC, Q_E4M3_ROW, Q_INT8_STATIC, Q_NVFP4, Q_NVFP4_MMA = range(5)

_vp, _i, _i64, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float

# name -> (restype, argtypes); the single source of the exported symbol list.
SIGNATURES = {
    "isp_version": (_i, []),
    "isp_status_string": (ctypes.c_char_p, [_i]),
    "isp_device_check": (_i, []),
    "isp_read_device_error": (_i, [ctypes.POINTER(_i), _i, _vp]),
    "isp_wait_selftest": (_i, [_i64, _vp]),
    "isp_norm_quant": (_i, [_vp, _i, _i64, _i, _vp, _vp, _f, _f, _i, _i, _f, _vp, _vp, _vp, _vp]),
    "isp_adaln_quant": (_i, [_vp, _i, _i64, _i, _vp, _f, _vp, _vp, _i64, _i, _f, _vp, _vp, _vp, _vp]),
    "isp_conv1d_geometry": (_i, [_i, _i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "isp_conv1d_pack_weight": (_i, [_vp, _i64, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp]),
    "isp_conv1d_quant": (_i, [_vp, _i, _i64, _i, _i64, _i, _vp, _f, _vp, _i, _vp, _i, _vp]),
    "isp_conv1d": (_i, [_vp, _i, _i64, _i, _i64, _vp, _i, _i, _i, _i, _i, _i, _i, _i64, _f, _vp, _vp, _vp, _vp,
                        _i, _vp]),
    "isp_conv1d_dynamic_noalloc": (_i, [_vp, _i, _i64, _i, _i64, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _i64,
                                        _vp, _vp, _vp, _i, _vp]),
    "isp_fir_snake": (_i, [_vp, _i64, _i, _i64, _vp, _vp, _vp, _vp, _vp, _i, _vp, _f, _vp]),
    "isp_scaled_gemm": (_i, [_vp, _vp, _i, _i64, _i, _i, _f, _vp, _vp, _vp, _vp, _i, _vp, _i, _f, _vp, _f, _vp]),
    "isp_gated_up": (_i, [_vp, _vp, _vp, _i, _i64, _i, _i, _vp, _vp, _f, _vp, _i, _vp]),
    "isp_int8_nonlinear_value": (_i, [_vp, _vp, _i64, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _vp]),
    "isp_nvfp4_scales_to_mma": (_i, [_vp, _i64, _i, _vp, _vp]),
    "isp_nvfp4_gemm": (_i, [_vp, _vp, _vp, _vp, _i64, _i, _i, _f, _vp, _vp, _i, _vp, _i, _vp]),
    "isp_nvfp4_gated_up": (_i, [_vp, _vp, _vp, _vp, _i64, _i, _i, _f, _f, _f, _vp, _vp, _vp]),
}

_LIB = None


class IspError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


def load() -> ctypes.CDLL:
    """Load the in-tree shared object and bind every exported symbol."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"CUDA library {LIB_PATH.name} is not built; run inspark_proper_format_b200.build.build() "
            "(this package has no CPU fallback)")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        try:
            fn = getattr(lib, name)
        except AttributeError:   # completeness is enforced by tests/test_abi_exports.py
            continue
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def status_string(status: int) -> str:
    try:
        return load().isp_status_string(status).decode()
    except Exception:  # library missing: still produce a message
        return "status"


def check(status: int, what: str) -> None:
    """Map a status code to the exception class the reference raises."""
    if status == ISP_OK:
        return
    if status in (ISP_ERR_SHAPE, ISP_ERR_DTYPE, ISP_ERR_ALIGN, ISP_ERR_ARG):
        raise ValueError(f"{what}: {status_string(status)}")
    raise IspError(status, what)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def read_device_error(clear: bool = True, stream=None) -> int:
    """Read (and optionally reset) the device error word of the current device."""
    out = ctypes.c_int(0)
    check(load().isp_read_device_error(ctypes.byref(out), int(clear), stream if stream is not None else stream_handle()),
          "isp_read_device_error")
    return out.value
