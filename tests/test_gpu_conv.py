"""GPU parity: quantized learned Conv1d / ConvTranspose1d as the phase-folded
implicit GEMM on tcgen05, against the oracle and the reference fixtures
(``ops/triton/fp8_conv.conv1d`` through Triton's interpreter; ``ExportWeightOp``
conv roles)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import conv as oconv
from oracle import gemm as og
from oracle.formats import bf16_round

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def C():
    from inspark_proper_format_b200 import _lib, conv
    yield conv
    assert _lib.read_device_error(clear=True) == 0, "a bounded device wait expired"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def packed_dev(packed_u8):
    return torch.from_numpy(np.ascontiguousarray(packed_u8)).cuda().view(torch.float8_e4m3fn)


@pytest.mark.parametrize("name", ["dilated", "strided", "deconv", "deconv_ragged", "bf16"])
def test_matrix_conv_matches_triton_reference_fixture(C, name):
    """Same packed weight, scales and inputs as the reference's FP8 conv kernel."""
    d = np.load(GOLDEN / "conv_matrix_fp8.npz")
    tr, ci, co, kw, s, pad, dil, op, bf = (int(v) for v in d[f"{name}_geom"])
    x = torch.from_numpy(d[f"{name}_x"]).cuda()
    if bf:
        x = x.bfloat16()
    bias = torch.from_numpy(d[f"{name}_bias"]).cuda() if f"{name}_bias" in d.files else None
    y = C.conv1d(x, packed_dev(d[f"{name}_packed"]), torch.from_numpy(d[f"{name}_scales"]).cuda(), bias, ci, co, kw,
                 s, pad, dil, bool(tr), op)
    assert y.dtype == x.dtype and tuple(y.shape) == d[f"{name}_y"].shape
    got = y.float().cpu().numpy()
    if bf:
        ref32 = oconv.matrix_conv1d(d[f"{name}_x"], d[f"{name}_packed"], d[f"{name}_scales"], d[f"{name}_bias"], ci,
                                    co, kw, s, pad, dil, bool(tr), op)
        assert np.all(np.abs(got - ref32) <= np.abs(ref32) * 2.0 ** -8 + 1e-6)   # one BF16 rounding
    else:
        assert rel_l2(got, d[f"{name}_y"]) < 1e-6     # exact products; FP32 sums in another order


# (transpose, ci, co, kw, stride, padding, dilation, output_padding, batch, t)
GEOMETRIES = [
    (False, 128, 128, 3, 1, 5, 5, 0, 2, 700),        # BigVGAN resblock conv (dilation 5), stationary B
    (False, 512, 256, 7, 1, 3, 1, 0, 2, 300),        # conv_pre-like, streaming B (K = 3584)
    (True, 256, 128, 16, 8, 4, 1, 0, 2, 90),         # upsampling ConvTranspose1d, 8 phases, window 3
    (True, 200, 40, 5, 3, 1, 1, 2, 3, 61),           # ragged phases, C and CO unaligned, output_padding
    (True, 200, 40, 5, 3, 1, 1, 1, 3, 61),           # the same through the strided TMA store (T_out = 184)
    (False, 96, 72, 4, 2, 1, 1, 0, 3, 259),          # strided Conv1d (A view of 2 x C_pad columns)
    (True, 64, 48, 4, 2, 1, 1, 0, 2, 512),           # ConvTranspose1d stride 2 through the TMA store
    (True, 128, 80, 7, 3, 0, 2, 0, 2, 100),          # dilated ConvTranspose1d, non-power-of-2 stride
    (False, 64, 300, 1, 1, 0, 1, 0, 1, 1000),        # pointwise, two channel tiles
]


@pytest.mark.parametrize("geom", GEOMETRIES, ids=lambda g: "x".join(map(str, g[:8])))
def test_matrix_conv_geometries_vs_oracle(C, geom):
    tr, ci, co, kw, s, pad, dil, op, b, t = geom
    g = np.random.default_rng(hash(geom) % 2**32)
    w = (g.standard_normal((ci, co, kw) if tr else (co, ci, kw)) * 0.05).astype(np.float32)
    dense = np.transpose(w, (1, 0, 2)) if tr else w
    packed, scales = og.pack_weight(dense.reshape(co, ci * kw))
    bias = (g.standard_normal(co) * 0.1).astype(np.float32)
    x = g.standard_normal((b, ci, t)).astype(np.float32)
    x[:, g.choice(ci, 2, replace=False)] *= 8.0
    x[1 % b] *= 0.25                                  # utterances with different scales
    ref = oconv.matrix_conv1d(x, packed, scales, bias, ci, co, kw, s, pad, dil, tr, op)
    y = C.conv1d(torch.from_numpy(x).cuda(), packed_dev(packed), torch.from_numpy(scales).cuda(),
                 torch.from_numpy(bias).cuda(), ci, co, kw, s, pad, dil, tr, op)
    assert tuple(y.shape) == ref.shape
    assert rel_l2(y.cpu().numpy(), ref) < 1e-5


def test_matrix_conv_bf16_and_f16_inputs(C):
    tr, ci, co, kw, s, pad, dil = False, 160, 96, 3, 1, 3, 3
    g = np.random.default_rng(7)
    w = (g.standard_normal((co, ci, kw)) * 0.05).astype(np.float32)
    packed, scales = og.pack_weight(w.reshape(co, ci * kw))
    for t in (333, 336):                             # per-element and tensor-map output stores
        x = bf16_round(g.standard_normal((2, ci, t)).astype(np.float32))
        ref32 = oconv.matrix_conv1d(x, packed, scales, None, ci, co, kw, s, pad, dil, tr)
        _check_half_outputs(C, x, packed, scales, ref32, ci, co, kw, s, pad, dil, tr)


def _check_half_outputs(C, x, packed, scales, ref32, ci, co, kw, s, pad, dil, tr):
    for dt in (torch.bfloat16, torch.float16):
        y = C.conv1d(torch.from_numpy(x).cuda().to(dt), packed_dev(packed), torch.from_numpy(scales).cuda(), None, ci,
                     co, kw, s, pad, dil, tr, 0)
        assert y.dtype == dt
        ulp = 2.0 ** -8 if dt == torch.bfloat16 else 2.0 ** -11
        got = y.float().cpu().numpy()
        assert np.mean(np.abs(got - ref32) <= np.abs(ref32) * ulp + 1e-6) > 0.999


def test_dynamic_amax_is_per_utterance_max(C):
    from inspark_proper_format_b200 import _lib
    x = torch.randn(3, 50, 77, device="cuda")
    x[2] *= 5
    xq = torch.empty(3, 77, 128, device="cuda", dtype=torch.uint8)
    amax = torch.full((3,), 123.0, device="cuda")
    st = _lib.load().isp_conv1d_quant(x.data_ptr(), _lib.F32, 3, 50, 77, 1, None, 0.0, amax.data_ptr(), _lib.E4M3,
                                      xq.data_ptr(), 128, _lib.stream_handle(x.device))
    _lib.check(st, "isp_conv1d_quant")
    assert torch.equal(amax, x.abs().amax(dim=(1, 2)))
    # channels past C and the codes themselves
    scale = np.maximum(amax.cpu().numpy() / np.float32(448), np.float32(1e-12)).astype(np.float32)
    codes = oconv.quantize_input(x.cpu().numpy() / scale[:, None, None] * 1.0, 1.0)
    assert np.array_equal(xq[:, :, :50].cpu().numpy(), np.transpose(codes, (0, 2, 1)))
    assert int(xq[:, :, 50:].count_nonzero()) == 0


def test_export_conv_roles_match_reference_fixture(C):
    """``ExportWeightOp`` FP8 Conv1d (dilated, padded) and ConvTranspose1d
    (zero-insertion rewrite) with the fixture's calibrated scales."""
    d = np.load(GOLDEN / "conv_fp8_export.npz")
    conv = torch.nn.Conv1d(64, 48, 7, padding=int(d["padding"]), dilation=int(d["dilation"]))
    deconv = torch.nn.ConvTranspose1d(32, 24, 8, stride=int(d["stride_d"]), padding=int(d["padding_d"]))
    with torch.no_grad():
        conv.weight.copy_(torch.from_numpy(d["w"]))
        conv.bias.copy_(torch.from_numpy(d["bias"]))
        deconv.weight.copy_(torch.from_numpy(d["wd"]))
        deconv.bias.copy_(torch.from_numpy(d["biasd"]))
    qc = C.QuantConv1d(conv.cuda(), {"precision": "fp8", "input_scale": float(d["in_scale"]),
                                     "weight_scale": d["w_scale"].tolist(), "weight_axis": 0})
    qd = C.QuantConv1d(deconv.cuda(), {"precision": "fp8", "input_scale": float(d["in_scale_d"]),
                                       "weight_scale": d["w_scale_d"].tolist(), "weight_axis": 1,
                                       "conv_transpose_rewrite": "zero_insert_conv"})
    yc = qc(torch.from_numpy(d["x"]).cuda()).cpu().numpy()
    yd = qd(torch.from_numpy(d["xd"]).cuda()).cpu().numpy()
    assert yc.shape == d["y"].shape and yd.shape == d["yd"].shape
    assert rel_l2(yc, d["y"]) < 1e-5
    assert rel_l2(yd, d["yd"]) < 1e-5


@pytest.mark.parametrize("t", [150, 160])            # scalar and float4 input loads
def test_export_int8_smoothquant_conv_vs_oracle(C, t):
    ci, co, kw, pad, dil = 136, 64, 5, 4, 2
    g = np.random.default_rng(11)
    conv = torch.nn.Conv1d(ci, co, kw, padding=pad, dilation=dil)
    with torch.no_grad():
        conv.weight.copy_(torch.from_numpy((g.standard_normal((co, ci, kw)) * 0.05).astype(np.float32)))
    x = g.standard_normal((2, ci, t)).astype(np.float32)
    x[:, :3] *= 12
    smooth = np.sqrt(np.abs(x).max(axis=(0, 2)) / 4).astype(np.float32) + np.float32(0.5)
    in_scale = float(np.abs(x / smooth[None, :, None]).max() / 127)
    w_s = (np.abs(conv.weight.detach().numpy() * smooth[None, :, None]).max(axis=(1, 2)) / 127).astype(np.float32)
    q = C.QuantConv1d(conv.cuda(), {"precision": "int8", "input_scale": in_scale, "weight_scale": w_s.tolist(),
                                    "smooth_scale": smooth.tolist()})
    ref = oconv.fp8_conv1d(x, conv.weight.detach().cpu().numpy(), conv.bias.detach().cpu().numpy(), in_scale, w_s,
                           dilation=dil, padding=pad, fmt="int8", smooth=smooth)
    y = q(torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_l2(y, ref) < 1e-6      # integer accumulation is exact


def test_export_deconv_static_vs_zero_insertion_oracle(C):
    """The phase-folded ConvTranspose1d equals the reference's zero-insertion
    rewrite (same code products), including output_padding."""
    ci, co, kw, s, pad, op = 128, 96, 12, 6, 3, 2
    g = np.random.default_rng(5)
    deconv = torch.nn.ConvTranspose1d(ci, co, kw, stride=s, padding=pad, output_padding=op)
    with torch.no_grad():
        deconv.weight.copy_(torch.from_numpy((g.standard_normal((ci, co, kw)) * 0.05).astype(np.float32)))
    x = g.standard_normal((2, ci, 40)).astype(np.float32)
    in_scale = float(np.abs(x).max() / 448)
    w_s = (np.abs(deconv.weight.detach().numpy()).max(axis=(0, 2)) / 448).astype(np.float32)
    q = C.QuantConv1d(deconv.cuda(), {"precision": "fp8", "input_scale": in_scale, "weight_scale": w_s.tolist(),
                                      "weight_axis": 1, "conv_transpose_rewrite": "zero_insert_conv"})
    ref = oconv.fp8_conv_transpose1d(x, deconv.weight.detach().cpu().numpy(), deconv.bias.detach().cpu().numpy(),
                                     in_scale, w_s, stride=s, padding=pad, output_padding=op)
    y = q(torch.from_numpy(x).cuda(), out_dtype=torch.float32).cpu().numpy()
    assert y.shape == ref.shape
    assert rel_l2(y, ref) < 1e-5


def test_fp8_matrix_conv_module(C):
    mod = torch.nn.ConvTranspose1d(64, 32, 4, stride=2, padding=1).cuda()
    m = C.FP8MatrixConv(mod)
    x = torch.randn(2, 64, 45, device="cuda")
    y = m(x)
    packed = m.weight.view(torch.uint8).cpu().numpy()
    ref = oconv.matrix_conv1d(x.cpu().numpy(), packed, m.scales.cpu().numpy(), m.bias.detach().cpu().numpy(), 64, 32,
                              4, 2, 1, 1, True)
    assert rel_l2(y.detach().cpu().numpy(), ref) < 1e-5
    # two calls in a row reuse the cached folded weight
    assert torch.equal(m(x), y)


def test_export_int8_smoothquant_deconv_vs_oracle(C):
    """INT8 SmoothQuant ConvTranspose1d role (smoothing on the CI axis of the
    [CI, CO, KW] weight, input divided before the zero insertion): exact integer
    products, so the folded phases match the zero-insertion oracle to FP32 rounding."""
    ci, co, kw, s, pad = 144, 48, 8, 4, 2
    g = np.random.default_rng(13)
    deconv = torch.nn.ConvTranspose1d(ci, co, kw, stride=s, padding=pad)
    with torch.no_grad():
        deconv.weight.copy_(torch.from_numpy((g.standard_normal((ci, co, kw)) * 0.05).astype(np.float32)))
    x = g.standard_normal((2, ci, 37)).astype(np.float32)
    x[:, :4] *= 15
    smooth = (np.sqrt(np.abs(x).max(axis=(0, 2))) + 0.5).astype(np.float32)
    in_scale = float(np.abs(x / smooth[None, :, None]).max() / 127)
    wsm = deconv.weight.detach().numpy() * smooth[:, None, None]
    w_s = (np.abs(wsm).max(axis=(0, 2)) / 127).astype(np.float32)
    q = C.QuantConv1d(deconv.cuda(), {"precision": "int8", "input_scale": in_scale, "weight_scale": w_s.tolist(),
                                      "weight_axis": 1, "smooth_scale": smooth.tolist(),
                                      "conv_transpose_rewrite": "zero_insert_conv"})
    ref = oconv.fp8_conv_transpose1d(x, deconv.weight.detach().cpu().numpy(), deconv.bias.detach().cpu().numpy(),
                                     in_scale, w_s, stride=s, padding=pad, fmt="int8", smooth=smooth)
    y = q(torch.from_numpy(x).cuda()).cpu().numpy()
    assert y.shape == ref.shape
    assert rel_l2(y, ref) < 1e-6


def test_dynamic_conv_nan_input_like_reference(C):
    """A NaN input element: the reference's ``tl.max`` / ``tl.maximum`` (maxnum)
    drop it from the utterance's scale, so every other output keeps its value and
    only outputs whose window covers the NaN are NaN (same NaN mask as the oracle)."""
    ci, co, kw = 64, 48, 3
    g = torch.Generator().manual_seed(77)
    w = torch.randn(co, ci, kw, generator=g) * 0.05
    packed, scales = og.pack_weight(w.reshape(co, ci * kw).numpy())
    x = torch.randn(2, ci, 90, generator=g)
    x[0, 5, 40] = float("nan")
    y = C.conv1d(x.cuda(), packed_dev(packed), torch.from_numpy(scales).cuda(), None, ci, co, kw, 1, 1, 1, False, 0)
    ref = oconv.matrix_conv1d(x.numpy(), packed, scales, None, ci, co, kw, 1, 1, 1, False)
    got = y.cpu().numpy()
    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
    assert np.isnan(ref).sum() == co * kw                     # 3 output times x every channel of utterance 0
    ok = ~np.isnan(ref)
    assert rel_l2(got[ok], ref[ok]) < 1e-6
