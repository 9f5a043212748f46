"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures in ``tests/golden`` were written by ``tests/golden/make_golden.py``
from the reference's own PyTorch modules; this suite needs neither the
reference nor a GPU.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import fir, formats, gemm, normquant
from oracle.formats import bits_to_bf16, e4m3_decode

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / f"{name}.npz")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_manifest_pins_fixture_bytes():
    lines = (GOLDEN / "MANIFEST.sha256").read_text().split("\n")
    entries = [line.split() for line in lines if line.strip()]
    assert len(entries) >= 9
    for digest, name in entries:
        assert hashlib.sha256((GOLDEN / name).read_bytes()).hexdigest() == digest, name


def test_gptfast_rmsnorm_then_static_e4m3():
    d = load("normquant_gptfast_e4m3")
    x = bits_to_bf16(d["x_bf16"])
    y = normquant.rms_norm_gptfast(x, d["gamma"], float(d["eps"]), True)
    # Row statistic rounding may differ from torch's FP32 running sum on rare rows.
    assert np.mean(y != d["y"]) < 1e-4
    codes, _ = normquant.norm_quant(x, normquant.NORM_RMS_GPTFAST, normquant.Q_E4M3_STATIC,
                                    gamma=d["gamma"], eps=float(d["eps"]), scale=float(d["scale"]))
    assert np.mean(codes != d["codes"]) < 1e-4
    # Given the reference's own normalized values the quantizer is bit-exact.
    exact = normquant.quant_e4m3_static(d["y"], float(d["scale"]))
    np.testing.assert_array_equal(exact, d["codes"])
    np.testing.assert_array_equal((e4m3_decode(exact) * d["scale"]).astype(np.float32), d["qdq"])


def test_adaptive_layer_norm_then_static_e4m3():
    d = load("normquant_adaln_e4m3")
    x = bits_to_bf16(d["x_bf16"])
    y = normquant.adaptive_layer_norm(x, d["gamma"], float(d["eps"]), d["ada_w"], d["ada_b"],
                                      int(d["rows_per_group"]), True)
    assert np.mean(y != d["y"]) < 1e-4           # rare rows: torch's FP32 running row sum
    np.testing.assert_allclose(y, d["y"], rtol=1e-5, atol=1e-6)
    exact = normquant.quant_e4m3_static(d["y"], float(d["scale"]))
    np.testing.assert_array_equal(exact, d["codes"])


def test_qwen_rmsnorm_then_static_e4m3():
    d = load("normquant_qwen_e4m3")
    x = bits_to_bf16(d["x_bf16"])
    y = normquant.rms_norm_qwen(x, d["gamma"], float(d["eps"]), True)
    assert np.mean(y != bits_to_bf16(d["y_bf16"])) < 1e-4
    exact = normquant.quant_e4m3_static(bits_to_bf16(d["y_bf16"]), float(d["scale"]))
    np.testing.assert_array_equal(exact, d["codes"])


def test_biasnorm_then_static_e4m3():
    d = load("normquant_biasnorm_e4m3")
    y = normquant.bias_norm(d["x"], d["bias"], float(d["log_scale_exp"]), False)
    np.testing.assert_allclose(y, d["y"], rtol=2e-6, atol=1e-7)
    codes = normquant.quant_e4m3_static(d["y"], float(d["scale"]))
    np.testing.assert_array_equal(codes, d["codes"])
    mine = normquant.quant_e4m3_static(y, float(d["scale"]))
    assert np.mean(mine != d["codes"]) < 1e-3


def test_pack_weight_matches_reference():
    d = load("pack_weight")
    packed, scale = gemm.pack_weight(d["w"])
    np.testing.assert_array_equal(scale, d["scale"])
    np.testing.assert_array_equal(packed, d["packed"])
    # The per-row dynamic quantizer is the same rule applied to rows.
    codes, s = normquant.quant_e4m3_row(d["w"])
    np.testing.assert_array_equal(s, d["scale"])
    np.testing.assert_array_equal(codes.T, d["packed"][:, :codes.shape[0]])


def test_fp8_linear_export_weight_op():
    d = load("fp8_linear_export")
    a_codes = normquant.quant_e4m3_static(d["a"], float(d["input_scale"]))
    np.testing.assert_array_equal(a_codes, d["a_codes"])
    w_scale = np.maximum((np.abs(d["w"]).max(1) / np.float32(448)).astype(np.float32), np.float32(1e-12))
    np.testing.assert_array_equal(w_scale.astype(np.float32), d["weight_scale"])
    w_codes = formats.e4m3_quantize(d["w"], w_scale[:, None])
    np.testing.assert_array_equal(w_codes, d["w_codes"])
    out = gemm.fp8_gemm(a_codes, w_codes, d["input_scale"], d["weight_scale"], d["bias"])
    assert rel_l2(out, d["out"]) < 1e-6


def test_fp8_linear_zipvoice():
    d = load("fp8_linear_zipvoice")
    a_codes = normquant.quant_e4m3_static(d["a"], float(d["input_scale"]))
    n = d["weight_fp8"].shape[0]
    w_scale = np.full(n, d["weight_scale"], np.float32)
    out = gemm.fp8_gemm(a_codes, d["weight_fp8"], d["input_scale"], w_scale, d["bias"])
    assert rel_l2(out, d["out"]) < 1e-6


def test_int8_smoothquant():
    d = load("int8_smoothquant")
    qa = normquant.quant_int8_static(d["a"], float(d["input_scale"]), d["smooth"])
    np.testing.assert_array_equal(qa, d["a_q"])
    out = gemm.int8_gemm(d["a_q"], d["w_q"], float(d["input_scale"]), d["weight_scale"], d["bias"])
    assert rel_l2(out, d["out"]) < 1e-6


def test_gated_up_swiglu_requant():
    d = load("gated_up")
    a_codes = normquant.quant_e4m3_static(d["x"], float(d["input_scale"]))
    w1c = formats.e4m3_quantize(d["w1"], d["w1_scale"][:, None])
    w3c = formats.e4m3_quantize(d["w3"], d["w3_scale"][:, None])
    s1 = (d["w1_scale"] * d["input_scale"]).astype(np.float32)
    s3 = (d["w3_scale"] * d["input_scale"]).astype(np.float32)
    out, q = gemm.gated_up(a_codes, w1c, w3c, s1, s3, float(d["output_scale"]))
    # The reference requantizes by division, the gated-up kernel by the
    # reciprocal; both agree except on codes sitting at a rounding tie.
    assert np.mean(out != d["out"]) < 2e-3
    assert rel_l2(out, d["out"]) < 1e-3


@pytest.mark.parametrize("t", [1, 2, 5, 12, 301, 1000])
def test_fir_snake_matches_activation1d(t):
    d = load("fir")
    f_up, f_down = fir.bigvgan_filters()
    np.testing.assert_allclose(f_up, d["filter"], atol=5e-8)
    y = fir.alias_free_snake(d[f"x_{t}"], d["up"], d["down"], d["alpha"], fir.snake_inverse_beta(d["alpha"]))
    np.testing.assert_allclose(y, d[f"y_{t}"], atol=1e-6, rtol=1e-5)
    assert rel_l2(y, d[f"y_{t}"]) < 1e-6


def test_fir_static_alias_free_and_snakebeta():
    d = load("fir")
    y = fir.alias_free_snake(d["x_1000"], d["up"], d["down"], d["alpha"], fir.snake_inverse_beta(d["alpha"]))
    assert rel_l2(y, d["y_static_1000"]) < 1e-6
    alpha = np.exp(d["log_alpha"]).astype(np.float32)
    inv_beta = (np.float32(1) / (np.exp(d["log_beta"]).astype(np.float32) + np.float32(1e-9))).astype(np.float32)
    y = fir.alias_free_snake(d["x_301"], d["up"], d["down"], alpha, inv_beta)
    assert rel_l2(y, d["y_beta_301"]) < 1e-6


def test_conv_oracle_matches_export_weight_op():
    """Quantized learned Conv1d and ConvTranspose1d (zero-insertion rewrite) of the
    reference's export graph, against the oracle's exact-sum restatement."""
    from oracle import conv as oconv
    d = load("conv_fp8_export")
    y = oconv.fp8_conv1d(d["x"], d["w"], d["bias"], d["in_scale"], d["w_scale"], dilation=int(d["dilation"]),
                         padding=int(d["padding"]))
    assert y.shape == d["y"].shape
    assert np.linalg.norm(y - d["y"]) / np.linalg.norm(d["y"]) < 1e-6      # torch's FP32 conv sum order
    yd = oconv.fp8_conv_transpose1d(d["xd"], d["wd"], d["biasd"], d["in_scale_d"], d["w_scale_d"],
                                    stride=int(d["stride_d"]), padding=int(d["padding_d"]))
    assert yd.shape == d["yd"].shape
    assert np.linalg.norm(yd - d["yd"]) / np.linalg.norm(d["yd"]) < 1e-6


CONV_MATRIX_CASES = ("dilated", "strided", "deconv", "deconv_ragged", "bf16")


@pytest.mark.parametrize("name", CONV_MATRIX_CASES)
def test_matrix_conv_oracle_matches_triton_reference(name):
    """``ops/triton/fp8_conv.conv1d`` (run by Triton's CPU interpreter on exact
    E4M3 inputs) against the oracle's gather-form restatement: every geometry,
    dynamic per-utterance scales, the packed [K, N] weight."""
    from oracle import conv as oconv
    d = load("conv_matrix_fp8")
    tr, ci, co, kw, s, pad, dil, op, bf = (int(v) for v in d[f"{name}_geom"])
    bias = d[f"{name}_bias"] if f"{name}_bias" in d.files else None
    y = oconv.matrix_conv1d(d[f"{name}_x"], d[f"{name}_packed"], d[f"{name}_scales"], bias, ci, co, kw, s, pad, dil,
                            bool(tr), op)
    ref = d[f"{name}_y"]
    assert y.shape == ref.shape
    if bf:
        # the interpreter's BF16 store truncates; the FP32 value before it must agree
        assert np.array_equal((y.view(np.uint32) & 0xFFFF0000).view(np.float32), ref)
    else:
        assert rel_l2(y, ref) < 1e-6                                      # FP32 dot order of the interpreter


def test_matrix_conv_weight_packing_is_pack_weight():
    """The packed conv weight is ``pack_weight`` of the [CO, CI * KW] matrix
    (ConvTranspose1d: of weight.permute(1, 0, 2))."""
    d = load("conv_matrix_fp8")
    for name in CONV_MATRIX_CASES:
        tr, ci, co, kw = (int(v) for v in d[f"{name}_geom"][:4])
        w = d[f"{name}_w"]
        dense = np.transpose(w, (1, 0, 2)) if tr else w
        packed, scales = gemm.pack_weight(dense.reshape(co, ci * kw))
        assert np.array_equal(packed, d[f"{name}_packed"]), name
        assert np.array_equal(scales, d[f"{name}_scales"]), name


def test_fp8_linear_oracle_matches_triton_reference():
    """``ops/triton/fp8.linear`` (dynamic per-row scale; single and split-K
    tiles) on exact E4M3 inputs against ``oracle.gemm.fp8_linear``."""
    d = load("fp8_linear_triton")
    y = gemm.fp8_linear(d["x"], d["packed"], d["scales"], d["bias"], out_bf16=False)
    for split in (1, 3):
        assert rel_l2(y, d[f"y_split{split}"]) < 1e-6
