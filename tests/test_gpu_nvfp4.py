"""GPU parity: NVFP4 block-scaled GEMM (tcgen05 kind::mxf4nvf4), the NVFP4
gated-up with NVFP4 requant of h, the tensor-core scale layout, and the
config-3 chain, against the oracle restatement."""
import numpy as np
import pytest
import torch

from oracle import normquant as onq
from oracle import nvfp4 as ofp4

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def F():
    from inspark_proper_format_b200 import _lib, nvfp4
    yield nvfp4
    assert _lib.read_device_error(clear=True) == 0, "a bounded device wait expired"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def operands(m, n, k, seed):
    """Oracle-quantized NVFP4 activations and weight (row-major scales)."""
    g = np.random.default_rng(seed)
    a = g.standard_normal((m, k)).astype(np.float32)
    a[:, g.choice(k, 4, replace=False)] *= 10
    w = (g.standard_normal((n, k)) * 0.02).astype(np.float32)
    g_a = ofp4.activation_global_scale(float(np.abs(a).max()))
    a_p, a_s = onq.quant_nvfp4(a, g_a)
    w_p, w_s, g_w = ofp4.quantize_weight(w)
    return a_p, a_s, g_a, w_p, w_s, g_w


def to_dev(F, packed, scodes, k):
    codes = torch.from_numpy(packed).cuda()
    sf = torch.from_numpy(ofp4.sf_to_mma_layout(scodes)).cuda()
    return codes, sf


@pytest.mark.parametrize("r,k", [(1, 64), (127, 512), (128, 128), (300, 2048), (1000, 1280)])
def test_scales_to_mma_matches_oracle_layout(F, r, k):
    src = np.random.default_rng(r + k).integers(0, 256, (r, k // 16), dtype=np.uint8)
    got = F.scales_to_mma(torch.from_numpy(src).cuda(), k).cpu().numpy()
    np.testing.assert_array_equal(got, ofp4.sf_to_mma_layout(src))


@pytest.mark.parametrize("m,k", [(1, 64), (100, 512), (128, 512), (333, 2048), (64, 1280)])
def test_norm_quant_mma_layout_bit_exact(m, k):
    from inspark_proper_format_b200.norm_quant import norm_quant
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).bfloat16()
    gamma = torch.rand(k, generator=g) * 0.2 + 0.9
    gs = float(ofp4.activation_global_scale(float(x.float().abs().max()) * 0.5))
    x[0, :16] = 0
    codes, sf = norm_quant(x.cuda(), kind="rms_gptfast", fmt="nvfp4_mma", gamma=gamma.cuda(), global_scale=gs)
    ref_p, ref_s = onq.norm_quant(x.float().numpy(), onq.NORM_RMS_GPTFAST, onq.Q_NVFP4, gamma=gamma.numpy(),
                                  input_is_bf16=True, global_scale=gs)
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_p)
    got_s = ofp4.sf_from_mma_layout(sf.cpu().numpy(), m, k // 16)
    np.testing.assert_array_equal(got_s, ref_s)


@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (100, 256, 512), (128, 128, 320), (300, 200, 2048),
                                   (257, 512, 512), (64, 1536, 1280)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_nvfp4_gemm_matches_oracle(F, m, n, k, out_dtype):
    a_p, a_s, g_a, w_p, w_s, g_w = operands(m, n, k, m * 31 + n + k)
    bias = np.random.default_rng(1).standard_normal(n).astype(np.float32) * 0.1
    a_c, a_sf = to_dev(F, a_p, a_s, k)
    wq = F.NVFP4Weight.from_export(torch.from_numpy(w_p).cuda(), torch.from_numpy(w_s).cuda(), g_w)
    y = F.nvfp4_gemm(a_c, a_sf, float(g_a), wq, bias=torch.from_numpy(bias).cuda(), out_dtype=out_dtype)
    ref = ofp4.nvfp4_gemm(a_p, a_s, g_a, w_p, w_s, g_w, bias)
    tol = 1e-5 if out_dtype == torch.float32 else 5e-3
    assert rel_l2(y.float().cpu().numpy(), ref) < tol


def test_nvfp4_gemm_residual_and_zero_blocks(F):
    m, n, k = 200, 256, 512
    a_p, a_s, g_a, w_p, w_s, g_w = operands(m, n, k, 7)
    a_p[5] = 0                       # an all-zero row (codes 0, scale 1)
    a_s[5] = onq.nvfp4_block_scales(np.zeros((1, k), np.float32), g_a)[0]
    res = np.random.default_rng(3).standard_normal((m, n)).astype(np.float32)
    a_c, a_sf = to_dev(F, a_p, a_s, k)
    wq = F.NVFP4Weight.from_export(torch.from_numpy(w_p).cuda(), torch.from_numpy(w_s).cuda(), g_w)
    y = F.nvfp4_gemm(a_c, a_sf, float(g_a), wq, residual=torch.from_numpy(res).cuda(), out_dtype=torch.float32)
    ref = ofp4.nvfp4_gemm(a_p, a_s, g_a, w_p, w_s, g_w) + res
    assert rel_l2(y.cpu().numpy(), ref) < 1e-5
    np.testing.assert_allclose(y.cpu().numpy()[5], res[5], rtol=0, atol=0)


def test_weight_from_float_matches_oracle_quantizer(F):
    w = (torch.randn(384, 512, generator=torch.Generator().manual_seed(4)) * 0.02)
    wq = F.NVFP4Weight.from_float(w.cuda())
    wf16 = w.half().float().numpy()
    ref_p, ref_s, ref_g = ofp4.quantize_weight(wf16)
    assert np.float32(wq.global_scale) == ref_g
    np.testing.assert_array_equal(wq.codes.cpu().numpy(), ref_p)
    np.testing.assert_array_equal(ofp4.sf_from_mma_layout(wq.scales.cpu().numpy(), 384, 32), ref_s)


def dequant_rows(codes, scodes, g):
    return ofp4.dequantize(codes, scodes, g)


@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (100, 128, 512), (300, 256, 512), (129, 192, 1280)])
def test_nvfp4_gated_up_matches_oracle(F, m, n, k):
    g = np.random.default_rng(m + n + k)
    a = g.standard_normal((m, k)).astype(np.float32)
    w1 = (g.standard_normal((n, k)) * 0.02).astype(np.float32)
    w3 = (g.standard_normal((n, k)) * 0.02).astype(np.float32)
    g_a = ofp4.activation_global_scale(float(np.abs(a).max()))
    a_p, a_s = onq.quant_nvfp4(a, g_a)
    q1 = ofp4.quantize_weight(w1)
    q3 = ofp4.quantize_weight(w3)
    # calibrate h's global scale on the oracle's own h
    gate = ofp4.nvfp4_gemm(a_p, a_s, g_a, *q1)
    up = ofp4.nvfp4_gemm(a_p, a_s, g_a, *q3)
    h_amax = float(np.abs(gate / (1 + np.exp(-gate)) * up).max())
    g_h = ofp4.activation_global_scale(h_amax)
    ref_c, ref_s, ref_h = ofp4.gated_up_nvfp4(a_p, a_s, g_a, q1, q3, g_h)

    a_c, a_sf = to_dev(F, a_p, a_s, k)
    codes13 = F.stack_gate_up(torch.from_numpy(q1[0]), torch.from_numpy(q3[0])).cuda()
    sf13 = F.stack_gate_up(torch.from_numpy(q1[1]), torch.from_numpy(q3[1])).cuda()
    w13 = F.NVFP4Weight(codes13, F.scales_to_mma(sf13, k), 1.0, 2 * n, k)
    hc, hs = F.nvfp4_gated_up(a_c, a_sf, float(g_a), w13, float(q1[2]), float(q3[2]), float(g_h))
    got_c = hc.cpu().numpy()
    got_s = ofp4.sf_from_mma_layout(hs.cpu().numpy(), m, n // 16)
    # h differs from the oracle by the fast exp in SiLU and the FP32 accumulation order:
    # scales and codes agree except at rare decision boundaries.
    assert np.mean(got_s != ref_s) < 2e-3
    assert np.mean(got_c != ref_c) < 5e-3
    dq = dequant_rows(got_c, got_s, g_h)
    ref_dq = dequant_rows(ref_c, ref_s, g_h)
    assert rel_l2(dq, ref_dq) < 2e-2
    assert rel_l2(dq, ref_h) < 0.2     # NVFP4 quantization noise of h itself


def test_config3_chain_small(F):
    """x -> NVFP4 quant -> gated-up (NVFP4 h) -> down GEMM, module surface."""
    m, d, n = 384, 512, 2048
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(m, d, generator=gen).bfloat16()
    w1 = torch.randn(n, d, generator=gen) * 0.02
    w3 = torch.randn(n, d, generator=gen) * 0.02
    w2 = torch.randn(d, n, generator=gen) * 0.02
    xf = x.float().numpy()
    g_x = ofp4.activation_global_scale(float(np.abs(xf).max()))
    a_p, a_s = onq.quant_nvfp4(xf, g_x)
    q1 = ofp4.quantize_weight(w1.half().float().numpy())
    q3 = ofp4.quantize_weight(w3.half().float().numpy())
    q2 = ofp4.quantize_weight(w2.half().float().numpy())
    gate = ofp4.nvfp4_gemm(a_p, a_s, g_x, *q1)
    up = ofp4.nvfp4_gemm(a_p, a_s, g_x, *q3)
    h_amax = float(np.abs(gate / (1 + np.exp(-gate)) * up).max())
    g_h = ofp4.activation_global_scale(h_amax)
    h_p, h_s, _ = ofp4.gated_up_nvfp4(a_p, a_s, g_x, q1, q3, g_h)
    ref = ofp4.nvfp4_gemm(h_p, h_s, g_h, *q2)

    mod = F.NVFP4GatedUp(w1.cuda(), w3.cuda(), w2.cuda(), float(np.abs(xf).max()), h_amax)
    y = mod(x.cuda(), out_dtype=torch.float32)
    assert rel_l2(y.cpu().numpy(), ref) < 2e-2


def test_nvfp4_linear_module(F):
    """MatrixWeightOp(linear).apply_nvfp4 surface: K = 400 is padded to 448."""
    torch.manual_seed(0)
    lin = torch.nn.Linear(400, 320)
    x = torch.randn(50, 400)
    amax = float(x.abs().max())
    mod = F.NVFP4Linear(lin.cuda(), amax)
    y = mod(x.cuda()).cpu().numpy()
    w = np.pad(lin.weight.detach().cpu().float().numpy(), ((0, 0), (0, 48)))
    wq = ofp4.quantize_weight(w.astype(np.float16).astype(np.float32))
    g_x = ofp4.activation_global_scale(amax)
    a_p, a_s = onq.quant_nvfp4(np.pad(x.numpy(), ((0, 0), (0, 48))), g_x)
    ref = ofp4.nvfp4_gemm(a_p, a_s, g_x, *wq, lin.bias.detach().cpu().numpy())
    assert rel_l2(y, ref) < 1e-5
    assert rel_l2(y, lin(x.cuda()).detach().cpu().numpy()) < 0.25   # W4A4 error vs the float layer


def test_nvfp4_errors_before_launch(F):
    from inspark_proper_format_b200 import _lib
    lib = _lib.load()
    a = torch.zeros(128, 32, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(128 * 4, dtype=torch.uint8, device="cuda")
    out = torch.empty(128, 128, dtype=torch.bfloat16, device="cuda")
    s = _lib.stream_handle()
    # K % 64 != 0
    assert lib.isp_nvfp4_gemm(a.data_ptr(), sf.data_ptr(), a.data_ptr(), sf.data_ptr(), 128, 128, 48, 1.0,
                              None, None, _lib.F32, out.data_ptr(), _lib.BF16, s) == _lib.ISP_ERR_SHAPE
    # h_scale out of range
    assert lib.isp_nvfp4_gated_up(a.data_ptr(), sf.data_ptr(), a.data_ptr(), sf.data_ptr(), 128, 64, 64, 1.0, 1.0,
                                  0.0, out.data_ptr(), sf.data_ptr(), s) == _lib.ISP_ERR_ARG
    # N % 64 != 0 for the gated-up
    assert lib.isp_nvfp4_gated_up(a.data_ptr(), sf.data_ptr(), a.data_ptr(), sf.data_ptr(), 128, 96, 64, 1.0, 1.0,
                                  1.0, out.data_ptr(), sf.data_ptr(), s) == _lib.ISP_ERR_SHAPE
