"""Failure detection on the GPU without a fault: a bounded device-side wait that
runs out (a barrier nothing arrives on, 2 ms limit) must come back as
ISP_ERR_TIMEOUT in the device error word, leave the context usable and free its
TMEM, so the next kernel (a tcgen05 GEMM that allocates TMEM) runs and matches
the oracle."""
import numpy as np
import pytest
import torch

from oracle import gemm as og

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_stays_usable():
    from inspark_proper_format_b200 import _lib
    from inspark_proper_format_b200.gemm import scaled_gemm
    lib = _lib.load()
    torch.cuda.synchronize()
    assert _lib.read_device_error(clear=True) == 0
    for _ in range(2):                                   # twice: the cleanup leaves nothing behind
        assert lib.isp_wait_selftest(2_000_000, _lib.stream_handle()) == _lib.ISP_OK
        assert _lib.read_device_error(clear=True) == _lib.ISP_ERR_TIMEOUT
        assert _lib.read_device_error(clear=True) == 0   # the read above cleared it
    g = np.random.default_rng(5)
    a = g.integers(-127, 128, (300, 512), dtype=np.int8)
    w = g.integers(-127, 128, (256, 512), dtype=np.int8)
    ws = (g.random(256) * 1e-3).astype(np.float32)
    y = scaled_gemm(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), a_scale=0.01,
                    w_scale=torch.from_numpy(ws).cuda(), out_dtype=torch.float32)
    np.testing.assert_array_equal(y.cpu().numpy(), og.int8_gemm(a, w, np.float32(0.01), ws))
    assert _lib.read_device_error(clear=True) == 0
