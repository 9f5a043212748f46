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
    # torch sums the 512 squares in FP32 in its own vectorized order; the oracle (and
    # the kernel) round the exact sum once.  The normalized values differ by one ulp
    # in 29 of the 192 rows; not one of the 98304 codes differs.
    mine = normquant.quant_e4m3_static(y, float(d["scale"]))
    assert np.count_nonzero(mine != d["codes"]) == 0
    assert np.count_nonzero((y != d["y"]).any(axis=1)) <= 32


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


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_fir_quant_oracle_matches_triton_reference(case):
    """``deployment/multibatch/fir_quant_kernel.py`` (run by Triton's CPU
    interpreter: log-scale Snake, FP32 FIR, then the signed INT8 rule
    ``rint(div_rn(div_rn(y, smooth), scale))``) against ``oracle.fir``."""
    d = load("fir_quant")
    alpha = np.exp(d[f"{case}_log_alpha"]).astype(np.float32)
    inv_beta = (np.float32(1) / (np.exp(d[f"{case}_log_beta"]).astype(np.float32) + np.float32(1e-9))).astype(np.float32)
    q = fir.alias_free_snake_int8(d[f"{case}_x"], d["up"], d["down"], alpha, inv_beta, d[f"{case}_smooth"],
                                  float(d[f"{case}_scale"][0]))
    ref = d[f"{case}_q"]
    assert q.shape == ref.shape
    # the kernel divides sin^2 by (beta + 1e-9) where the oracle multiplies by its
    # reciprocal: FP32 values on an INT8 rounding tie may land on either side
    assert np.count_nonzero(q != ref) <= max(1, q.size // 10000)
    assert np.abs(q.astype(int) - ref.astype(int)).max() <= 1


@pytest.mark.parametrize("case,groups", [("b1", 1), ("b16", 16)])
def test_int8_nonlinear_value_oracle_matches_triton_reference(case, groups):
    """``int8_nonlinear_value`` (b1 and the 16-group variant, run by Triton's CPU
    interpreter) against ``oracle.gemm.int8_nonlinear_value``: the gate (z2) is
    bit-exact; value = tanh(z0) * z1 within 2 ulps (both sides use numpy's tanh
    here; the GPU kernel uses CUDA's tanhf)."""
    d = load("int8_nonlinear_value")
    q = d[f"{case}_q"]
    value, gate = gemm.int8_nonlinear_value(q.reshape(-1, q.shape[-1]), d["w"], float(d[f"{case}_as"][0]),
                                            d[f"{case}_ws"], d[f"{case}_bias"], groups)
    np.testing.assert_array_equal(gate, d[f"{case}_gate"].reshape(gate.shape))
    ref = d[f"{case}_value"].reshape(value.shape)
    np.testing.assert_array_max_ulp(value, ref, maxulp=2)


def test_cpu_reference_arm_is_the_reference_eager_layer():
    """``oracle/torch_path.FP8Layer`` (the arithmetic ``bench.py --impl reference``
    times) against the same layer built from the reference's own RMSNorm, _QDQ and
    FP8 ExportWeightOp modules: all seven layer outputs bit-identical."""
    import torch

    from oracle.torch_path import FP8Layer
    d = load("fp8_layer_eager")
    x = torch.from_numpy(d["x_bits"].view(np.int16)).view(torch.bfloat16)
    layer = FP8Layer([torch.from_numpy(d[f"wq{i}"]) for i in range(10)],
                     [torch.tensor(float(v)) for v in d["act_scales"]])
    outs = layer.outputs(x, torch.from_numpy(d["gamma"]), 1e-6, torch.tensor(float(d["norm_scale"])))
    for i, o in enumerate(outs):
        np.testing.assert_array_equal(o.numpy(), d[f"y{i}"], err_msg=f"output {i}")
    # the weights the bench quantizes itself ((w / s).clamp.to(e4m3) * s) are the folded ones
    for i in range(10):
        w = torch.from_numpy(d[f"w{i}"])
        s = (w.abs().amax(1) / 448).clamp_min(1e-12)
        wq = (w / s[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s[:, None]
        np.testing.assert_array_equal(wq.numpy(), d[f"wq{i}"])


def test_fir_torch_f64_matches_activation1d():
    """The float64 torch restatement the full-size GPU FIR test uses as its
    reference, against the reference's Activation1d(Snake) outputs."""
    import torch

    from fir_torch_f64 import activation1d_f64
    d = load("fir")
    for t in (1, 2, 5, 12, 301, 1000):
        x = torch.from_numpy(d[f"x_{t}"])
        alpha = torch.from_numpy(d["alpha"])
        ib = torch.from_numpy(fir.snake_inverse_beta(d["alpha"]))
        y = activation1d_f64(x, torch.from_numpy(d["filter"]), alpha, ib).numpy()
        assert y.shape == d[f"y_{t}"].shape
        assert rel_l2(y, d[f"y_{t}"]) < 1e-6, t
