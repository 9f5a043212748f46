"""GPU: isp_conv1d_dynamic_noalloc (per-utterance maxima in a static device array)
against the caller-scratch path (isp_conv1d_quant with a caller amax buffer, then
isp_conv1d).  Collected last on purpose: it must pass alone and after every other
GPU test (the static array keeps no state between calls)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup():
    from inspark_proper_format_b200 import _lib, conv
    from inspark_proper_format_b200.gemm import pack_weight
    g = torch.Generator(device="cuda").manual_seed(3)
    ci, co, kw, s, pad, dil, tr = 256, 128, 8, 4, 2, 1, True          # ConvTranspose1d, 4 folded phases
    w = torch.randn(ci, co, kw, device="cuda", generator=g) * 0.05
    packed, scales = pack_weight(w.permute(1, 0, 2).reshape(co, ci * kw))
    folded = conv.pack_folded(packed.view(torch.uint8), co, ci, kw, s, dil, pad, tr)
    bias = torch.randn(co, device="cuda", generator=g) * 0.1
    return _lib, conv, g, (ci, co, kw, s, pad, dil, tr), folded, scales, bias


def test_noalloc_matches_caller_scratch_path_two_calls():
    _lib, conv, g, (ci, co, kw, s, pad, dil, tr), folded, scales, bias = _setup()
    lib = _lib.load()
    c_pad = folded.shape[-1]
    # two calls in a row with different batch sizes and per-utterance scales: the
    # second must not see the first call's maxima
    for b, t, gain in ((3, 200, 4.0), (2, 333, 0.25)):
        x = torch.randn(b, ci, t, device="cuda", generator=g) * gain
        x[-1] *= 3.0
        ref = conv.run(x, folded, scales, bias, ci=ci, co=co, kw=kw, stride=s, padding=pad, dilation=dil,
                       transpose=tr)
        t_out = conv.out_length(t, kw, s, pad, dil, tr)
        xq = torch.empty(b, t, c_pad, device="cuda", dtype=torch.uint8)
        y = torch.empty(b, co, t_out, device="cuda")
        st = lib.isp_conv1d_dynamic_noalloc(x.data_ptr(), _lib.F32, b, ci, t, xq.data_ptr(), c_pad, folded.data_ptr(),
                                            co, kw, s, dil, pad, 0, int(tr), t_out, scales.data_ptr(),
                                            bias.data_ptr(), y.data_ptr(), _lib.F32, _lib.stream_handle(x.device))
        _lib.check(st, "isp_conv1d_dynamic_noalloc")
        torch.testing.assert_close(y, ref, rtol=1e-6, atol=1e-6)
    assert _lib.read_device_error(clear=True) == 0


def test_noalloc_strided_conv1d_bf16_two_calls():
    """The Conv1d branch: stride 2 (codes padded to a whole number of stride rows,
    T odd), BF16 input and output, two calls with different batches."""
    from inspark_proper_format_b200 import _lib, conv
    from inspark_proper_format_b200.gemm import pack_weight
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(9)
    ci, co, kw, s, pad, dil, tr = 192, 96, 4, 2, 1, 1, False
    w = torch.randn(co, ci, kw, device="cuda", generator=g) * 0.05
    packed, scales = pack_weight(w.reshape(co, ci * kw))
    folded = conv.pack_folded(packed.view(torch.uint8), co, ci, kw, s, dil, pad, tr)
    bias = torch.randn(co, device="cuda", generator=g) * 0.1
    c_pad = folded.shape[-1]
    for b, t, gain in ((4, 301, 2.0), (1, 77, 0.5)):
        x = (torch.randn(b, ci, t, device="cuda", generator=g) * gain).bfloat16()
        ref = conv.run(x, folded, scales, bias, ci=ci, co=co, kw=kw, stride=s, padding=pad, dilation=dil,
                       transpose=tr)
        t_out = conv.out_length(t, kw, s, pad, dil, tr)
        t_rows = (t + s - 1) // s * s
        xq = torch.empty(b, t_rows, c_pad, device="cuda", dtype=torch.uint8)
        y = torch.empty(b, co, t_out, device="cuda", dtype=torch.bfloat16)
        st = lib.isp_conv1d_dynamic_noalloc(x.data_ptr(), _lib.BF16, b, ci, t, xq.data_ptr(), c_pad,
                                            folded.data_ptr(), co, kw, s, dil, pad, 0, int(tr), t_out,
                                            scales.data_ptr(), bias.data_ptr(), y.data_ptr(), _lib.BF16,
                                            _lib.stream_handle(x.device))
        _lib.check(st, "isp_conv1d_dynamic_noalloc")
        assert ref.dtype == torch.bfloat16
        torch.testing.assert_close(y, ref, rtol=0, atol=0)        # same kernels, same scales: identical
    assert _lib.read_device_error(clear=True) == 0


def test_noalloc_rejects_batches_beyond_the_scratch():
    _lib, conv, g, (ci, co, kw, s, pad, dil, tr), folded, scales, bias = _setup()
    dummy = torch.empty(16, device="cuda")
    p = dummy.data_ptr()
    st = _lib.load().isp_conv1d_dynamic_noalloc(p, _lib.F32, 8193, ci, 10, p, folded.shape[-1], p, co, kw, s, dil,
                                                pad, 0, int(tr), conv.out_length(10, kw, s, pad, dil, tr), p, None, p,
                                                _lib.F32, _lib.stream_handle(dummy.device))
    assert st == _lib.ISP_ERR_SHAPE
