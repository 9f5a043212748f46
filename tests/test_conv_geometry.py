"""CPU checks of the implicit-conv geometry (host code of the C ABI, no GPU):
the phase-folded window covers exactly the reference's gather positions, and
bad geometries are rejected before any device work."""
import ctypes

import numpy as np
import pytest

from oracle import conv as oconv


@pytest.fixture(scope="module")
def lib():
    from inspark_proper_format_b200 import _lib, build
    build.build()
    return _lib.load()


def folded_window(kw, stride, dilation, padding, transpose):
    """Restatement: Conv1d is one phase over all taps; ConvTranspose1d folds the
    stride's phases into columns and spans the input offsets R = (r + padding -
    k * dilation) / stride that any (phase r, tap k) pair reads."""
    if not transpose:
        return 1, kw, 0
    offsets = [(r + padding - k * dilation) // stride for r in range(stride) for k in range(kw)
               if (r + padding - k * dilation) % stride == 0]
    if not offsets:
        return stride, 1, 0
    return stride, max(offsets) - min(offsets) + 1, min(offsets)


GEOMS = [(3, 1, 5, 5, False), (7, 1, 1, 3, False), (4, 2, 1, 1, False), (16, 8, 1, 4, True), (3, 2, 2, 1, True),
         (5, 3, 1, 1, True), (12, 6, 1, 3, True), (11, 5, 1, 3, True), (4, 4, 2, 0, True), (1, 1, 1, 0, False),
         (8, 4, 1, 2, True), (7, 3, 2, 0, True)]


@pytest.mark.parametrize("g", GEOMS)
def test_geometry_matches_restatement(lib, g):
    phases, taps = ctypes.c_int(), ctypes.c_int()
    assert lib.isp_conv1d_geometry(*g[:4], int(g[4]), ctypes.byref(phases), ctypes.byref(taps)) == 0
    assert (phases.value, taps.value) == folded_window(*g)[:2]


@pytest.mark.parametrize("g", [g for g in GEOMS if g[4]])
def test_folded_window_covers_every_gather_position(g):
    """Every (output time, tap, input row) triple that ``ops/triton/fp8_conv.py:
    31-33`` reads is formed exactly once by some (phase, window slot) of the
    folded GEMM, with the tap the weight packing assigns to that pair."""
    kw, s, dil, pad, _ = g
    _, slots, r_min = folded_window(*g)
    t_out = 64
    seen = []
    for r in range(s):
        for j in range(slots):
            num = r + pad - (r_min + j) * s
            if num < 0 or num % dil or num // dil >= kw:
                continue                       # zero weight in this (phase, slot)
            k = num // dil
            for q in range((t_out - r + s - 1) // s):
                seen.append((q * s + r, k, q + r_min + j))
    expected = set()
    for t in range(t_out):
        for k in range(kw):
            num = t + pad - k * dil
            if num % s == 0:
                expected.add((t, k, num // s))
    assert len(seen) == len(set(seen)) and set(seen) == expected


def test_geometry_limits_and_host_validation(lib):
    p, t = ctypes.c_int(), ctypes.c_int()
    assert lib.isp_conv1d_geometry(129, 1, 1, 0, 0, ctypes.byref(p), ctypes.byref(t)) == 1     # > 128 slots
    assert lib.isp_conv1d_geometry(0, 1, 1, 0, 0, ctypes.byref(p), ctypes.byref(t)) == 1
    assert lib.isp_conv1d_geometry(3, 0, 1, 0, 0, ctypes.byref(p), ctypes.byref(t)) == 1
    assert lib.isp_conv1d_geometry(3, 1, 1, 0, 0, None, None) == 7
    # NULL operands, wrong dtypes and a wrong output length fail on the host
    assert lib.isp_conv1d(None, 3, 1, 128, 10, None, 8, 3, 1, 1, 1, 0, 0, 10, 1.0, None, None, None, None, 1,
                          None) == 7
    buf = ctypes.create_string_buffer(64)
    ptr = ctypes.addressof(buf)
    assert lib.isp_conv1d(ptr, 4, 1, 128, 10, ptr, 8, 3, 1, 1, 1, 0, 0, 10, 0.0, ptr, ptr, None, ptr, 1,
                          None) == 7       # dynamic scale with INT8 codes
    assert lib.isp_conv1d(ptr, 3, 1, 128, 10, ptr, 8, 3, 1, 1, 1, 0, 0, 11, 1.0, None, ptr, None, ptr, 1,
                          None) == 1       # T_out != (10 + 2 - 2 - 1) / 1 + 1
    assert lib.isp_conv1d_quant(ptr, 1, 1, 8, 10, 1, None, 0.0, ptr, 4, ptr, 128, None) == 7   # INT8 dynamic
    assert lib.isp_conv1d_quant(ptr, 1, 1, 8, 10, 1, None, 1.0, None, 3, ptr, 100, None) == 1  # C_pad % 128


def test_out_length_matches_oracle():
    from inspark_proper_format_b200.conv import out_length
    for t in (1, 7, 100):
        for g in GEOMS:
            kw, s, dil, pad, tr = g
            assert out_length(t, kw, s, pad, dil, tr, 0) == oconv.conv_out_length(t, kw, s, pad, dil, tr, 0)
    assert [out_length(10, 3, 2, 1, 1, True, op) for op in (0, 1)] == [19, 20]   # 9*2 - 2 + 2 + op + 1
