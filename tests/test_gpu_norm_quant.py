"""GPU parity: fused norm->quantize kernel vs the oracle (and the golden fixtures)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import normquant as onq
from oracle.formats import bf16_round, bits_to_bf16

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def nq():
    from inspark_proper_format_b200.norm_quant import norm_quant
    return norm_quant


def _acts(m, k, outliers, factor, seed, bf16=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    idx = torch.randperm(k, generator=g)[:outliers]
    x[:, idx] *= factor
    return x.bfloat16() if bf16 else x


KIND = {"rms_gptfast": onq.NORM_RMS_GPTFAST, "rms_qwen": onq.NORM_RMS_QWEN, "bias": onq.NORM_BIAS,
        "none": onq.NORM_NONE}


def _oracle(x, kind, fmt, **kw):
    xf = x.float().numpy()
    return onq.norm_quant(xf, KIND[kind], {"e4m3": onq.Q_E4M3_STATIC, "e4m3_row": onq.Q_E4M3_ROW,
                                           "int8": onq.Q_INT8_STATIC, "nvfp4": onq.Q_NVFP4}[fmt],
                          input_is_bf16=x.dtype == torch.bfloat16, **kw)


@pytest.mark.parametrize("kind", ["rms_gptfast", "rms_qwen", "bias", "none"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("m,k", [(1, 16), (3, 48), (37, 512), (300, 1280), (129, 4096)])
def test_norm_e4m3_static_bit_exact(nq, kind, dtype, m, k):
    x = _acts(m, k, 4, 20.0, m * 7 + k, bf16=dtype == torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    gamma = torch.rand(k, generator=g) * 0.2 + 0.9
    bias = torch.randn(k, generator=g) * 0.1
    scale = 0.0137
    codes, _ = nq(x.cuda(), kind=kind, fmt="e4m3", gamma=gamma.cuda(), bias=bias.cuda(), eps=1e-6,
                  log_scale=torch.tensor(0.3), scale=scale)
    ref, _ = _oracle(x, kind, "e4m3", gamma=gamma.numpy(), bias=bias.numpy(), eps=1e-6,
                     log_scale_exp=float(torch.tensor(0.3).exp()), scale=scale)
    np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), ref)


@pytest.mark.parametrize("m,k", [(1, 512), (255, 512), (1000, 1536)])
def test_row_dynamic_e4m3(nq, m, k):
    x = _acts(m, k, 4, 20.0, 3)
    codes, s = nq(x.cuda(), kind="none", fmt="e4m3_row")
    ref, rs = _oracle(x, "none", "e4m3_row")
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), ref)


@pytest.mark.parametrize("smooth_on", [True, False])
@pytest.mark.parametrize("m,k", [(64, 1280), (17, 5120), (5, 512)])
def test_int8_smoothquant(nq, smooth_on, m, k):
    x = _acts(m, k, 8, 30.0, 5)
    g = torch.Generator().manual_seed(2)
    smooth = torch.rand(k, generator=g) * 3 + 0.2 if smooth_on else None
    gamma = torch.rand(k, generator=g) * 0.2 + 0.9
    kind = "rms_gptfast" if k <= 4096 else "none"
    codes, _ = nq(x.cuda(), kind=kind, fmt="int8", gamma=gamma.cuda(),
                  smooth=None if smooth is None else smooth.cuda(), scale=1.0 / 127)
    ref, _ = _oracle(x, kind, "int8", gamma=gamma.numpy(), smooth=None if smooth is None else smooth.numpy(),
                     scale=np.float32(1.0 / 127))
    np.testing.assert_array_equal(codes.cpu().numpy(), ref)


@pytest.mark.parametrize("m,k", [(1, 16), (64, 512), (333, 2048)])
def test_nvfp4_block_quant(nq, m, k):
    x = _acts(m, k, 4, 20.0, 9)
    gs = float(np.float32(np.abs(x.float().numpy()).max() * 0.7 / (6 * 448)))
    x[0, :16] = 0  # an all-zero block takes the scale-1.0 rule
    packed, sf = nq(x.cuda(), kind="rms_qwen", fmt="nvfp4", gamma=torch.ones(k).cuda(), global_scale=gs)
    ref_p, ref_s = _oracle(x, "rms_qwen", "nvfp4", gamma=np.ones(k, np.float32), global_scale=gs)
    np.testing.assert_array_equal(sf.view(torch.uint8).cpu().numpy(), ref_s)
    np.testing.assert_array_equal(packed.cpu().numpy(), ref_p)


def test_golden_gptfast_front_end(nq):
    d = np.load(GOLDEN / "normquant_gptfast_e4m3.npz")
    x = torch.from_numpy(bits_to_bf16(d["x_bf16"])).bfloat16()
    codes, _ = nq(x.cuda(), kind="rms_gptfast", fmt="e4m3", gamma=torch.from_numpy(d["gamma"]).cuda(),
                  eps=float(d["eps"]), scale=float(d["scale"]))
    got = codes.view(torch.uint8).cpu().numpy()
    assert np.mean(got != d["codes"]) < 1e-4  # reference FP32 row-sum order, documented
    dq = (codes.float().cpu().numpy() * d["scale"]).astype(np.float32)
    assert np.mean(dq != d["qdq"]) < 1e-4


def test_golden_biasnorm_front_end(nq):
    d = np.load(GOLDEN / "normquant_biasnorm_e4m3.npz")
    x = torch.from_numpy(d["x"])
    codes, _ = nq(x.cuda(), kind="bias", fmt="e4m3", bias=torch.from_numpy(d["bias"]).cuda(),
                  log_scale=float(np.log(d["log_scale_exp"])), scale=float(d["scale"]))
    assert np.mean(codes.view(torch.uint8).cpu().numpy() != d["codes"]) < 1e-3


def test_full_size_config1_properties(nq):
    """Config-1 front end at full size: codes decode within half an E4M3 step."""
    x = _acts(3040, 512, 4, 20.0, 0)
    gamma = torch.rand(512, generator=torch.Generator().manual_seed(1)) * 0.2 + 0.9
    y = onq.rms_norm_gptfast(x.float().numpy(), gamma.numpy(), 1e-6, True)
    scale = float(np.abs(y).max() / 448)
    codes, _ = nq(x.cuda(), kind="rms_gptfast", fmt="e4m3", gamma=gamma.cuda(), scale=scale)
    ref = onq.quant_e4m3_static(y, scale)
    np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), ref)


def test_errors_are_reported_before_launch(nq):
    x = torch.randn(4, 24, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        nq(x, kind="none", fmt="e4m3", scale=1.0)          # K % 16 != 0
    with pytest.raises(ValueError):
        nq(torch.randn(4, 32, device="cuda").bfloat16(), kind="rms_gptfast", fmt="e4m3", scale=1.0)  # no gamma


def test_golden_adaptive_layer_norm(nq):
    """AdaLN (gpt_fast AdaptiveLayerNorm) fused with static E4M3, against the reference fixture."""
    from inspark_proper_format_b200.norm_quant import adaln_quant
    d = np.load(GOLDEN / "normquant_adaln_e4m3.npz")
    x = torch.from_numpy(bits_to_bf16(d["x_bf16"])).bfloat16()
    codes, _ = adaln_quant(x.cuda(), torch.from_numpy(d["gamma"]).cuda(), torch.from_numpy(d["ada_w"]).cuda(),
                           torch.from_numpy(d["ada_b"]).cuda(), eps=float(d["eps"]), scale=float(d["scale"]))
    got = codes.view(torch.uint8).cpu().numpy()
    assert np.mean(got != d["codes"]) < 1e-4      # reference FP32 row-sum order, documented
    ref = onq.quant_e4m3_static(onq.adaptive_layer_norm(bits_to_bf16(d["x_bf16"]), d["gamma"], float(d["eps"]),
                                                        d["ada_w"], d["ada_b"], int(d["rows_per_group"]), True),
                                float(d["scale"]))
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("fmt", ["e4m3", "nvfp4"])
@pytest.mark.parametrize("b,t,k", [(3, 50, 512), (2, 7, 1280)])
def test_adaln_bit_exact(nq, fmt, b, t, k):
    from inspark_proper_format_b200.norm_quant import adaln_quant
    g = torch.Generator().manual_seed(b * t + k)
    x = torch.randn(b * t, k, generator=g).bfloat16()
    gamma = torch.rand(k, generator=g) * 0.2 + 0.9
    w = torch.randn(b, k, generator=g) * 0.1 + 1.0
    bb = torch.randn(b, k, generator=g) * 0.1
    y = onq.adaptive_layer_norm(x.float().numpy(), gamma.numpy(), 1e-6, w.numpy(), bb.numpy(), t, True)
    if fmt == "e4m3":
        scale = float(np.abs(y).max() / 448)
        codes, _ = adaln_quant(x.cuda(), gamma.cuda(), w.cuda(), bb.cuda(), scale=scale)
        np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), onq.quant_e4m3_static(y, scale))
    else:
        gs = float(np.float32(np.abs(y).max() / (6 * 448)))
        codes, sf = adaln_quant(x.cuda(), gamma.cuda(), w.cuda(), bb.cuda(), fmt="nvfp4", global_scale=gs)
        rp, rs = onq.quant_nvfp4(y, gs)
        np.testing.assert_array_equal(codes.cpu().numpy(), rp)
        np.testing.assert_array_equal(sf.view(torch.uint8).cpu().numpy(), rs)


def _near_tie_inputs(m, k, s, grid_values, seed):
    """FP32 x = RN(v * s) for values v at or next to the rounding boundaries of the
    code grid, plus 1-ulp neighbours, so x / s lands within an FP32 ulp of a tie:
    the cases where a quotient off by one ulp would change the code."""
    g = np.random.default_rng(seed)
    v = g.choice(grid_values, size=(m, k)).astype(np.float64)
    x = (v * np.float64(s)).astype(np.float32)
    step = g.integers(-2, 3, size=(m, k)).astype(np.int32)
    x = (x.view(np.int32) + step).view(np.float32)          # walk up to 2 ulps either way
    return x


@pytest.mark.parametrize("k", [512, 1280])
def test_quotient_rounding_at_e4m3_ties(nq, k):
    """E4M3 codes of x / s where x / s sits on or beside E4M3 midpoints (5
    significant bits) across the normal and subnormal E4M3 ranges: bit-exact."""
    mids = np.array([(2 * m + 1) / 2 * 2.0 ** e for m in range(8, 16) for e in range(-9, 6)] +
                    [(2 * m + 1) / 2 * 2.0 ** -9 for m in range(0, 8)], np.float64)
    grid = np.concatenate([mids, -mids])
    for seed, s in enumerate((0.0137, 3.0e-3, 0.71, 1.7e-5)):
        x = _near_tie_inputs(64, k, s, grid, seed)
        codes, _ = nq(torch.from_numpy(x).cuda(), kind="none", fmt="e4m3", scale=s)
        ref = onq.quant_e4m3_static(x, s)
        np.testing.assert_array_equal(codes.view(torch.uint8).cpu().numpy(), ref)


def test_quotient_rounding_at_int8_ties(nq):
    """INT8 codes of x / s with x / s on or beside k + 1/2: bit-exact."""
    grid = np.array([k + 0.5 for k in range(-130, 130)], np.float64)
    for seed, s in enumerate((0.0137, 3.1e-3, 1.3)):
        x = _near_tie_inputs(64, 512, s, grid, seed + 10)
        codes, _ = nq(torch.from_numpy(x).cuda(), kind="none", fmt="int8", scale=s)
        ref = onq.quant_int8_static(x, s, None)
        np.testing.assert_array_equal(codes.view(torch.int8).cpu().numpy(), ref)
