"""GPU parity: tcgen05 W8A8 GEMMs (FP8 / INT8, all epilogues) vs the oracle."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import normquant as onq
from oracle.formats import e4m3_decode, e4m3_encode

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def G():
    from inspark_proper_format_b200 import _lib, gemm
    yield gemm
    assert _lib.read_device_error(clear=True) == 0, "a bounded device wait expired"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def fp8_operands(m, n, k, seed):
    g = np.random.default_rng(seed)
    a = g.standard_normal((m, k)).astype(np.float32)
    a[:, g.choice(k, 4, replace=False)] *= 20
    w = (g.standard_normal((n, k)) * 0.02).astype(np.float32)
    a_scale = np.float32(np.abs(a).max() / 448)
    w_scale = np.maximum((np.abs(w).max(1) / np.float32(448)).astype(np.float32), np.float32(1e-12))
    a_codes = onq.quant_e4m3_static(a, a_scale)
    w_codes = e4m3_encode(np.clip((w / w_scale[:, None]).astype(np.float32), -448, 448))
    bias = (g.standard_normal(n) * 0.1).astype(np.float32)
    return a_codes, w_codes, a_scale, w_scale, bias


def dev_codes(c):
    return torch.from_numpy(c).cuda().view(torch.float8_e4m3fn)


SHAPES = [(1, 16, 16), (7, 32, 48), (128, 256, 128), (129, 272, 144), (300, 1536, 512), (3040, 1536, 512),
          (555, 512, 1536), (64, 3840, 1280), (1000, 1024, 512), (260, 528, 1040)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_fp8_scaled_gemm(G, m, n, k, out):
    a, w, sa, sw, bias = fp8_operands(m, n, k, m + n + k)
    dtype = torch.bfloat16 if out == "bf16" else torch.float32
    y = G.scaled_gemm(dev_codes(a), dev_codes(w), a_scale=float(sa), w_scale=torch.from_numpy(sw).cuda(),
                      bias=torch.from_numpy(bias).cuda(), out_dtype=dtype)
    ref = og.fp8_gemm(a, w, sa, sw, bias, out="f32")
    got = y.float().cpu().numpy()
    if out == "f32":
        assert rel_l2(got, ref) < 1e-6
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5 * np.abs(ref).max())
    else:
        assert rel_l2(got, og._emit(ref, "bf16", None)) < 5e-4
        np.testing.assert_allclose(got, ref, rtol=8e-3, atol=1e-3 * np.abs(ref).max())


@pytest.mark.parametrize("m,n,k", [(300, 1536, 512), (129, 256, 128)])
def test_fp8_gemm_row_scales_f16_and_requant(G, m, n, k):
    a, w, sa, sw, bias = fp8_operands(m, n, k, 11)
    rows = (np.random.default_rng(1).random(m).astype(np.float32) + 0.5) * sa
    y = G.scaled_gemm(dev_codes(a), dev_codes(w), a_scale_rows=torch.from_numpy(rows).cuda(),
                      w_scale=torch.from_numpy(sw).cuda(), out_dtype=torch.float16)
    ref = og.fp8_gemm(a, w, rows, sw, None, out="f32")
    assert rel_l2(y.float().cpu().numpy(), ref) < 1e-3
    inv = np.float32(448.0 / np.abs(ref).max())
    q = G.scaled_gemm(dev_codes(a), dev_codes(w), a_scale_rows=torch.from_numpy(rows).cuda(),
                      w_scale=torch.from_numpy(sw).cuda(), out_dtype=torch.float8_e4m3fn, out_inv_scale=float(inv))
    qref = e4m3_encode(np.clip((ref * inv).astype(np.float32), -448, 448))
    got = q.view(torch.uint8).cpu().numpy()
    assert np.mean(got != qref) < 5e-3           # accumulation-order ties only
    assert rel_l2(e4m3_decode(got), e4m3_decode(qref)) < 1e-2


@pytest.mark.parametrize("res_dtype", [torch.float32, torch.bfloat16])
def test_residual_dual_output(G, res_dtype):
    m, n, k = 777, 512, 512
    a, w, sa, sw, bias = fp8_operands(m, n, k, 5)
    alpha = np.float32(sa * sw.mean())
    r = np.random.default_rng(2).standard_normal((m, n)).astype(np.float32)
    rt = torch.from_numpy(r).to(res_dtype)
    r_used = rt.float().numpy()
    inv = np.float32(30.0)
    y, q = G.fused_projection_residual(dev_codes(a), dev_codes(w), torch.from_numpy(bias).cuda(), rt.cuda(),
                                       float(alpha), float(inv))
    zref, qref = og.residual_dual(a, w, alpha, bias, r_used, inv)
    assert rel_l2(y.cpu().numpy(), zref) < 1e-6
    got = q.view(torch.uint8).cpu().numpy()
    assert np.mean(got != qref) < 1e-3


@pytest.mark.parametrize("m,n,k", [(64, 3840, 1280), (64, 1280, 5120), (333, 1280, 1280), (16384 // 16, 5120, 1280)])
def test_int8_gemm_bit_exact(G, m, n, k):
    g = np.random.default_rng(m + n)
    qa = g.integers(-128, 128, (m, k), dtype=np.int64).astype(np.int8)
    qw = g.integers(-127, 128, (n, k), dtype=np.int64).astype(np.int8)
    sa = np.float32(1 / 127)
    sw = (g.random(n).astype(np.float32) * 1e-3 + 1e-4).astype(np.float32)
    bias = (g.standard_normal(n) * 0.1).astype(np.float32)
    r = g.standard_normal((m, n)).astype(np.float32)
    y = G.i8_residual(torch.from_numpy(qa).cuda(), torch.from_numpy(qw).cuda(), float(sa), torch.from_numpy(sw).cuda(),
                      torch.from_numpy(bias).cuda(), torch.from_numpy(r).cuda())
    ref = og.int8_gemm(qa, qw, sa, sw, bias, r)
    np.testing.assert_array_equal(y.cpu().numpy(), ref)


def test_int8_smoothquant_golden(G):
    d = np.load(GOLDEN / "int8_smoothquant.npz")
    y = G.scaled_gemm(torch.from_numpy(d["a_q"]).cuda(), torch.from_numpy(d["w_q"]).cuda(),
                      a_scale=float(d["input_scale"]), w_scale=torch.from_numpy(d["weight_scale"]).cuda(),
                      bias=torch.from_numpy(d["bias"]).cuda(), out_dtype=torch.float32)
    assert rel_l2(y.cpu().numpy(), d["out"]) < 1e-6
    # the full module path: smooth + quantize + GEMM
    lin = torch.nn.Linear(d["w"].shape[1], d["w"].shape[0]).cuda()
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(d["w"]))
        lin.bias.copy_(torch.from_numpy(d["bias"]))
    spec = dict(smooth_scale=d["smooth"].tolist(), input_scale=float(d["input_scale"]),
                weight_scale=d["weight_scale"].tolist())
    mod = G.Int8SmoothQuantLinear(lin, spec)
    assert rel_l2(mod(torch.from_numpy(d["a"]).cuda()).cpu().numpy(), d["out"]) < 1e-6


def test_fp8_linear_export_golden(G):
    d = np.load(GOLDEN / "fp8_linear_export.npz")
    y = G.scaled_gemm(dev_codes(d["a_codes"]), dev_codes(d["w_codes"]), a_scale=float(d["input_scale"]),
                      w_scale=torch.from_numpy(d["weight_scale"]).cuda(), bias=torch.from_numpy(d["bias"]).cuda(),
                      out_dtype=torch.float32)
    assert rel_l2(y.cpu().numpy(), d["out"]) < 1e-6


def test_zipvoice_fp8linear_golden(G):
    d = np.load(GOLDEN / "fp8_linear_zipvoice.npz")
    n, k = d["weight_fp8"].shape
    lin = torch.nn.Linear(k, n).cuda()
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(e4m3_decode(d["weight_fp8"]) * d["weight_scale"]))
        lin.bias.copy_(torch.from_numpy(d["bias"]))
    mod = G.FP8Linear(lin, float(d["input_scale"]), float(d["weight_scale"]))
    assert torch.equal(mod.weight_fp8.view(torch.uint8).cpu(), torch.from_numpy(d["weight_fp8"]))
    assert rel_l2(mod(torch.from_numpy(d["a"]).cuda()).cpu().numpy(), d["out"]) < 1e-6


@pytest.mark.parametrize("m", [1, 300, 3040])
def test_dynamic_row_linear_matches_triton_contract(G, m):
    g = torch.Generator().manual_seed(m)
    w = (torch.randn(1536, 512, generator=g) * 0.02).bfloat16().float()
    packed, scales = G.pack_weight(w)
    x = (torch.randn(m, 512, generator=g) * 3).bfloat16()
    bias = torch.randn(1536, generator=g) * 0.1
    y = G.linear(x.cuda(), packed.cuda(), scales.cuda(), bias.cuda())
    assert y.dtype == torch.bfloat16 and y.shape == (m, 1536)
    ref = og.fp8_linear(x.float().numpy(), packed.view(torch.uint8).numpy(), scales.numpy(), bias.numpy(),
                        out_bf16=True)
    got = y.float().cpu().numpy()
    assert rel_l2(got, ref) < 1e-4                      # BF16 rounding flips from FP32 accumulation order only
    assert np.mean(got != ref) < 2e-2


@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (333, 1536, 512), (19840 // 20, 1536, 512), (64, 2048, 512)])
def test_gated_up_paired_and_interleaved(G, m, n, k):
    a, w1, sa, s1w, _ = fp8_operands(m, n, k, 3)
    _, w3, _, s3w, _ = fp8_operands(m, n, k, 4)
    s1 = (s1w * sa).astype(np.float32)
    s3 = (s3w * sa).astype(np.float32)
    _, _ = None, None
    gate = og.fp8_accumulate(a, w1) * s1[None, :]
    up = og.fp8_accumulate(a, w3) * s3[None, :]
    hv = gate / (1 + np.exp(-gate)) * up
    out_scale = float(np.abs(hv).max() / 448)
    ref_deq, ref_q = og.gated_up(a, w1, w3, s1, s3, out_scale)
    y = G.gated_up(dev_codes(a), dev_codes(w1), dev_codes(w3), torch.from_numpy(s1).cuda(),
                   torch.from_numpy(s3).cuda(), out_scale, dequant=True)
    assert rel_l2(y.cpu().numpy(), ref_deq) < 1e-2
    q = G.gated_up(dev_codes(a), dev_codes(w1), dev_codes(w3), torch.from_numpy(s1).cuda(),
                   torch.from_numpy(s3).cuda(), out_scale, dequant=False)
    got = q.view(torch.uint8).cpu().numpy()
    assert np.mean(got != ref_q) < 2e-2
    # interleaved layout: row 2n = gate n, row 2n+1 = up n
    wi = np.empty((2 * n, k), np.uint8)
    wi[0::2], wi[1::2] = w1, w3
    si = np.empty(2 * n, np.float32)
    si[0::2], si[1::2] = s1, s3
    qi = G.fp8_gated_up_interleaved_plugin(dev_codes(a), dev_codes(wi), torch.from_numpy(si).cuda(), float(sa),
                                           out_scale)
    np.testing.assert_array_equal(qi.view(torch.uint8).cpu().numpy(), got)
    np.testing.assert_array_equal(og.gated_up_interleaved(a, wi, si, out_scale), ref_q)


def test_gated_up_module_golden(G):
    d = np.load(GOLDEN / "gated_up.npz")
    mod = G.GatedUp(dict(w1=d["w1"], w3=d["w3"], w1_scale=d["w1_scale"], w3_scale=d["w3_scale"],
                         input_scale=float(d["input_scale"]), output_scale=float(d["output_scale"])), None)
    y = mod(torch.from_numpy(d["x"]).cuda().contiguous()).cpu().numpy()
    assert rel_l2(y, d["out"]) < 1e-2
    assert np.mean(y != d["out"]) < 3e-2


def test_full_size_zipformer_projection_property(G):
    """cfg-2 projection at full M (48640): linearity in the activation scale.
    Doubling a_scale doubles every FP32 output exactly (power-of-two scaling)."""
    m, n, k = 48640, 1536, 512
    g = torch.Generator(device="cuda").manual_seed(0)
    a = (torch.randn(m, k, device="cuda", generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = (torch.randn(n, k, device="cuda", generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn)
    sw = torch.rand(n, device="cuda", generator=g) * 1e-4
    y1 = G.scaled_gemm(a, w, a_scale=0.01, w_scale=sw, out_dtype=torch.float32)
    y2 = G.scaled_gemm(a, w, a_scale=0.02, w_scale=sw, out_dtype=torch.float32)
    assert torch.equal(y2, y1 * 2)
    # spot-check 64 rows against the oracle
    rows = torch.randint(0, m, (64,), generator=torch.Generator().manual_seed(1))
    ref = og.fp8_gemm(a[rows.cuda()].view(torch.uint8).cpu().numpy(), w.view(torch.uint8).cpu().numpy(), 0.01,
                      sw.cpu().numpy())
    assert rel_l2(y1[rows.cuda()].cpu().numpy(), ref) < 1e-6


def test_shape_and_dtype_errors(G):
    a = torch.zeros(4, 24, device="cuda").to(torch.float8_e4m3fn)
    w = torch.zeros(16, 24, device="cuda").to(torch.float8_e4m3fn)
    with pytest.raises(ValueError):
        G.scaled_gemm(a, w)                                           # K % 16
    with pytest.raises(ValueError):
        G.scaled_gemm(torch.zeros(4, 32, device="cuda").to(torch.float8_e4m3fn),
                      torch.zeros(16, 32, device="cuda", dtype=torch.int8))  # mixed operand types


@pytest.mark.parametrize("m", [1, 64, 128])
@pytest.mark.parametrize("n,k", [(1280, 1280), (3840, 1280), (1280, 5120), (5120, 1280), (208, 2048), (128, 128)])
def test_int8_decode_split_k_bit_exact(G, m, n, k):
    """M <= 128 runs the cluster split-K kernel: int32 partials add exactly."""
    g = np.random.default_rng(3 * m + n + k)
    qa = g.integers(-128, 128, (m, k), dtype=np.int64).astype(np.int8)
    qw = g.integers(-127, 128, (n, k), dtype=np.int64).astype(np.int8)
    sa = np.float32(1 / 127)
    sw = (g.random(n).astype(np.float32) * 1e-3 + 1e-4).astype(np.float32)
    bias = (g.standard_normal(n) * 0.1).astype(np.float32)
    r = g.standard_normal((m, n)).astype(np.float32)
    y = G.i8_residual(torch.from_numpy(qa).cuda(), torch.from_numpy(qw).cuda(), float(sa), torch.from_numpy(sw).cuda(),
                      torch.from_numpy(bias).cuda(), torch.from_numpy(r).cuda())
    np.testing.assert_array_equal(y.cpu().numpy(), og.int8_gemm(qa, qw, sa, sw, bias, r))


@pytest.mark.parametrize("m,n,k", [(64, 3840, 1280), (17, 1280, 5120), (128, 512, 1536)])
def test_fp8_decode_row_scales_residual(G, m, n, k):
    a, w, sa, sw, bias = fp8_operands(m, n, k, 29)
    rows = (np.random.default_rng(4).random(m).astype(np.float32) + 0.5) * sa
    res = torch.from_numpy(np.random.default_rng(5).standard_normal((m, n)).astype(np.float32)).bfloat16()
    y = G.scaled_gemm(dev_codes(a), dev_codes(w), a_scale_rows=torch.from_numpy(rows).cuda(),
                      w_scale=torch.from_numpy(sw).cuda(), bias=torch.from_numpy(bias).cuda(),
                      residual=res.cuda(), out_dtype=torch.float16)
    ref = og.fp8_gemm(a, w, rows, sw, bias, residual=res.float().numpy(), out="f32")
    assert rel_l2(y.float().cpu().numpy(), ref) < 1e-3      # F16 output rounding


# Streaming launches (K > 512) with more tiles than SMs run their last partial wave as
# half-N tiles: 9600 rows x N=512 is 150 tiles (2 split into 4 halves), the cfg-2
# ff_out shape 760 tiles (20 split into 40).
@pytest.mark.parametrize("m,n,k", [(9600, 512, 1536), (48640, 512, 1536), (9600, 1024, 1040)])
def test_fp8_streaming_tail_split(G, m, n, k):
    a, w, sa, sw, bias = fp8_operands(m, n, k, 31)
    y = G.scaled_gemm(dev_codes(a), dev_codes(w), a_scale=float(sa), w_scale=torch.from_numpy(sw).cuda(),
                      bias=torch.from_numpy(bias).cuda(), out_dtype=torch.float32)
    ref = og.fp8_gemm(a, w, sa, sw, bias, out="f32")
    got = y.cpu().numpy()
    assert rel_l2(got, ref) < 1e-6
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5 * np.abs(ref).max())


def test_int8_streaming_tail_split_bit_exact(G):
    m, n, k = 9600, 1024, 1280                         # 300 tiles: 4 split into 8 halves
    g = np.random.default_rng(41)
    qa = g.integers(-128, 128, (m, k), dtype=np.int64).astype(np.int8)
    qw = g.integers(-127, 128, (n, k), dtype=np.int64).astype(np.int8)
    sa = np.float32(1 / 127)
    sw = (g.random(n).astype(np.float32) * 1e-3 + 1e-4).astype(np.float32)
    bias = (g.standard_normal(n) * 0.1).astype(np.float32)
    r = g.standard_normal((m, n)).astype(np.float32)
    y = G.i8_residual(torch.from_numpy(qa).cuda(), torch.from_numpy(qw).cuda(), float(sa), torch.from_numpy(sw).cuda(),
                      torch.from_numpy(bias).cuda(), torch.from_numpy(r).cuda())
    ref = og.int8_gemm(qa, qw, sa, sw, bias, r)
    np.testing.assert_array_equal(y.cpu().numpy(), ref)


def test_residual_dual_output_tail_split(G):
    m, n, k = 9600, 512, 1024                          # 150 tiles: residual + dual E4M3 on half tiles
    a, w, sa, sw, bias = fp8_operands(m, n, k, 7)
    alpha = np.float32(sa * sw.mean())
    r = np.random.default_rng(3).standard_normal((m, n)).astype(np.float32)
    inv = np.float32(30.0)
    y, q = G.fused_projection_residual(dev_codes(a), dev_codes(w), torch.from_numpy(bias).cuda(),
                                       torch.from_numpy(r).cuda(), float(alpha), float(inv))
    zref, qref = og.residual_dual(a, w, alpha, bias, r, inv)
    assert rel_l2(y.cpu().numpy(), zref) < 1e-6
    assert np.mean(q.view(torch.uint8).cpu().numpy() != qref) < 1e-3


# ---------------------------------------------------------------------------
# INT8 nonlinear value (three stacked projections, tanh(z0) * z1 and z2)
# ---------------------------------------------------------------------------
def _nlv_operands(steps, groups, n, k, seed):
    g = np.random.default_rng(seed)
    q = g.integers(-128, 128, (steps, groups, k), dtype=np.int8)
    w = g.integers(-127, 128, (3 * n, k), dtype=np.int8)
    ws = (g.random(3 * n) * 2e-3 + 1e-4).astype(np.float32)
    bias = (g.standard_normal(3 * n) * 0.1).astype(np.float32)
    return q, w, np.float32(0.011), ws, bias


def _nlv_check(value, gate, ref_value, ref_gate):
    # z = acc * (AS * WS) + bias from an exact int32 accumulator: bit-exact; CUDA's
    # tanhf and numpy's tanh are each within 2 ulps of tanh, so value within 4 ulps
    np.testing.assert_array_equal(gate, ref_gate)
    np.testing.assert_array_max_ulp(value, ref_value, maxulp=4)


@pytest.mark.parametrize("case,groups", [("b1", 1), ("b16", 16)])
def test_int8_nonlinear_value_golden(G, case, groups):
    d = np.load(GOLDEN / "int8_nonlinear_value.npz")
    q = torch.from_numpy(d[f"{case}_q"]).cuda()
    value, gate = G.int8_nonlinear_value(q, torch.from_numpy(d["w"]).cuda(), float(d[f"{case}_as"][0]),
                                         torch.from_numpy(d[f"{case}_ws"]).cuda(),
                                         torch.from_numpy(d[f"{case}_bias"]).cuda())
    assert tuple(value.shape) == d[f"{case}_value"].shape and tuple(gate.shape) == d[f"{case}_gate"].shape
    _nlv_check(value.cpu().numpy(), gate.cpu().numpy(), d[f"{case}_value"], d[f"{case}_gate"])


@pytest.mark.parametrize("steps,groups,n,k", [(300, 1, 384, 512), (37, 8, 80, 512), (200, 1, 128, 1024),
                                              (5, 3, 16, 48), (760, 64, 384, 512)])
def test_int8_nonlinear_value_vs_oracle(G, steps, groups, n, k):
    """Ragged N tiles (80 = 64 + 16), the streaming schedule (K = 1024), tiny
    shapes, and the config-2 batch (B64 x 760 frames, M = 48640), every row."""
    q, w, a_s, ws, bias = _nlv_operands(steps, groups, n, k, steps + n + k)
    value, gate = G.int8_nonlinear_value(torch.from_numpy(q).cuda(), torch.from_numpy(w).cuda(), float(a_s),
                                         torch.from_numpy(ws).cuda(), torch.from_numpy(bias).cuda())
    rv, rg = og.int8_nonlinear_value(q.reshape(-1, k), w, a_s, ws, bias, groups)
    _nlv_check(value[0].cpu().numpy(), gate.reshape(-1, n).cpu().numpy(), rv, rg)
