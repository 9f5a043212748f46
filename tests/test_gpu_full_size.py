"""GPU parity at the full sizes of every BASELINE configuration the bench times.

The tile schedules only show their whole behaviour at size (B-stationary CTAs
walking many M tiles, persistent grids, the split last wave of streaming GEMMs,
thousands of FIR tiles per launch), so each configuration is checked here on
every row against the oracle (streamed in row blocks), or, for the FIR, against
the reference's Activation1d restated in float64 torch on the device
(``fir_torch_f64``, pinned to the reference fixture by a CPU test):

  * config 2: norm-quant [48640, 512] (bit-exact codes); attn_in 512->1536 with
    FP32 and BF16 outputs; ff_in 512->1536 with the E4M3 requant; ff_out
    1536->512 (streaming schedule with the half-N last wave);
  * config 3: NVFP4 activation quant, gated-up 2x2048 (NVFP4 h) and down
    2048->512 at M = 51200;
  * config 4: INT8 prefill, the four projections at M = 16384 (bit-exact);
  * config 5: one whole B64 x C512 x T16384 micro-batch and a B8 slice of
    C256 x T65536.
"""
import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import normquant as onq
from oracle import nvfp4 as ofp4
from oracle.formats import bf16_round, e4m3_decode

from fir_torch_f64 import activation1d_f64

pytestmark = pytest.mark.gpu
ROWS = 8192        # oracle row block


@pytest.fixture(scope="module")
def lib():
    from inspark_proper_format_b200 import _lib
    yield _lib
    assert _lib.read_device_error(clear=True) == 0, "a bounded device wait expired"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def fp8_weights(n, k, seed):
    g = np.random.default_rng(seed)
    w = (g.standard_normal((n, k)) * 0.02).astype(np.float32)
    ws = np.maximum((np.abs(w).max(1) / np.float32(448)).astype(np.float32), np.float32(1e-12))
    from oracle.formats import e4m3_encode
    codes = e4m3_encode(np.clip((w / ws[:, None]).astype(np.float32), -448, 448))
    bias = (g.standard_normal(n) * 0.01).astype(np.float32)
    return codes, ws, bias


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


# ---------------------------------------------------------------------------
# config 2: B64 x 760 frames, hidden 512, W8A8 static E4M3
# ---------------------------------------------------------------------------
M2 = 64 * 760


@pytest.fixture(scope="module")
def cfg2_codes(lib):
    """The norm-quant of a full config-2 batch (BF16 N(0,1), 1% outlier channels x10),
    checked bit-exact on every row; its codes feed the GEMM tests."""
    from inspark_proper_format_b200.norm_quant import norm_quant
    g = torch.Generator().manual_seed(2)
    x = torch.randn(M2, 512, generator=g)
    x[:, torch.randperm(512, generator=g)[:5]] *= 10
    x = x.bfloat16()
    gamma = torch.rand(512, generator=g) * 0.2 + 0.9
    scale = 0.035
    codes, _ = norm_quant(x.cuda(), kind="rms_gptfast", fmt="e4m3", gamma=gamma.cuda(), scale=scale)
    got = codes.view(torch.uint8).cpu().numpy()
    xf = x.float().numpy()
    for r in range(0, M2, ROWS):
        ref, _ = onq.norm_quant(xf[r:r + ROWS], onq.NORM_RMS_GPTFAST, onq.Q_E4M3_STATIC, gamma=gamma.numpy(),
                                scale=scale)
        np.testing.assert_array_equal(got[r:r + ROWS], ref, err_msg=f"rows {r}..")
    return got, np.float32(scale)


def test_cfg2_norm_quant_full_batch(cfg2_codes):
    assert cfg2_codes[0].shape == (M2, 512)


@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_cfg2_attn_in_every_row(lib, cfg2_codes, out):
    from inspark_proper_format_b200.gemm import scaled_gemm
    a, sa = cfg2_codes
    w, ws, bias = fp8_weights(1536, 512, 21)
    dtype = torch.float32 if out == "f32" else torch.bfloat16
    y = scaled_gemm(dev(a, torch.float8_e4m3fn), dev(w, torch.float8_e4m3fn), a_scale=float(sa), w_scale=dev(ws),
                    bias=dev(bias), out_dtype=dtype).float().cpu().numpy()
    worst = 0.0
    for r in range(0, M2, ROWS):
        ref = og.fp8_gemm(a[r:r + ROWS], w, sa, ws, bias, out="f32")
        got = y[r:r + ROWS]
        if out == "f32":
            worst = max(worst, rel_l2(got, ref))
        else:
            # exact products, FP32 sums in another order, then one BF16 rounding
            assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-5 * np.abs(ref).max()), r
            worst = max(worst, rel_l2(got, bf16_round(ref)))
    assert worst < (1e-6 if out == "f32" else 5e-4)


def test_cfg2_ff_in_e4m3_requant_every_row(lib, cfg2_codes):
    from inspark_proper_format_b200.gemm import scaled_gemm
    a, sa = cfg2_codes
    w, ws, bias = fp8_weights(1536, 512, 22)
    inv = np.float32(448.0 / 3.0)
    q = scaled_gemm(dev(a, torch.float8_e4m3fn), dev(w, torch.float8_e4m3fn), a_scale=float(sa), w_scale=dev(ws),
                    bias=dev(bias), out_dtype=torch.float8_e4m3fn, out_inv_scale=float(inv))
    got = q.view(torch.uint8).cpu().numpy()
    diff = 0
    for r in range(0, M2, ROWS):
        ref = og.fp8_gemm(a[r:r + ROWS], w, sa, ws, bias, out="f32")
        ref_q = og._emit((ref * inv).astype(np.float32), "e4m3", 1.0)
        bad = got[r:r + ROWS] != ref_q
        diff += int(bad.sum())
        # a differing code is one E4M3 step away (an accumulation-order tie)
        assert np.all(np.abs(e4m3_decode(got[r:r + ROWS][bad]) - e4m3_decode(ref_q[bad]))
                      <= np.abs(e4m3_decode(ref_q[bad])) * 0.125 + 2.0 ** -9), r
    assert diff / got.size < 1e-3


def test_cfg2_ff_out_streaming_every_row(lib, cfg2_codes):
    """K = 1536: the streaming schedule; 760 tiles on 148 SMs leave a last wave of 20
    that runs as 40 half-N tiles."""
    from inspark_proper_format_b200.gemm import scaled_gemm
    a512, sa = cfg2_codes
    h = np.concatenate([a512, a512[::-1], np.roll(a512, 7, axis=0)], axis=1)     # [M, 1536] codes
    w, ws, bias = fp8_weights(512, 1536, 23)
    y = scaled_gemm(dev(h, torch.float8_e4m3fn), dev(w, torch.float8_e4m3fn), a_scale=float(sa), w_scale=dev(ws),
                    bias=dev(bias), out_dtype=torch.float32).cpu().numpy()
    worst = 0.0
    for r in range(0, M2, ROWS):
        worst = max(worst, rel_l2(y[r:r + ROWS], og.fp8_gemm(h[r:r + ROWS], w, sa, ws, bias, out="f32")))
    assert worst < 1e-6


# ---------------------------------------------------------------------------
# config 3: NVFP4 CFM gated-up + down at B64 x 800 mel frames
# ---------------------------------------------------------------------------
M3 = 64 * 800


def test_cfg3_nvfp4_chain_every_row(lib):
    from inspark_proper_format_b200 import nvfp4 as F
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(M3, 512, generator=gen).bfloat16()
    w1, w3 = torch.randn(2048, 512, generator=gen) * 0.02, torch.randn(2048, 512, generator=gen) * 0.02
    w2 = torch.randn(512, 2048, generator=gen) * 0.02
    xf = x.float().numpy()
    g_x = ofp4.activation_global_scale(float(np.abs(xf).max()))
    q1, q3, q2 = (ofp4.quantize_weight(w.half().float().numpy()) for w in (w1, w3, w2))
    # h's global scale from a calibration slice of the oracle chain
    a_p, a_s = onq.quant_nvfp4(xf[:2048], g_x)
    gate, up = ofp4.nvfp4_gemm(a_p, a_s, g_x, *q1), ofp4.nvfp4_gemm(a_p, a_s, g_x, *q3)
    g_h = ofp4.activation_global_scale(float(np.abs(gate / (1 + np.exp(-gate)) * up).max()))

    xc, xs = F.quantize_activation(x.cuda(), float(g_x))
    codes13 = F.stack_gate_up(torch.from_numpy(q1[0]), torch.from_numpy(q3[0])).cuda()
    sf13 = F.stack_gate_up(torch.from_numpy(q1[1]), torch.from_numpy(q3[1])).cuda()
    w13 = F.NVFP4Weight(codes13, F.scales_to_mma(sf13, 512), 1.0, 4096, 512)
    hc, hs = F.nvfp4_gated_up(xc, xs, float(g_x), w13, float(q1[2]), float(q3[2]), float(g_h))
    w2q = F.NVFP4Weight(torch.from_numpy(q2[0]).cuda(), F.scales_to_mma(torch.from_numpy(q2[1]).cuda(), 2048),
                        float(q2[2]), 512, 2048)
    y = F.nvfp4_gemm(hc, hs, float(g_h), w2q, out_dtype=torch.float32).cpu().numpy()
    xc, hc = xc.cpu().numpy(), hc.cpu().numpy()
    xs, hs = xs.cpu().numpy().reshape(-1), hs.cpu().numpy().reshape(-1)     # tensor-core layout bytes

    bad_s = bad_c = 0
    worst_down = 0.0
    for r in range(0, M3, ROWS):
        nr = min(ROWS, M3 - r)                  # row blocks start on 128-row scale chunks
        rows = slice(r, r + nr)
        a_p, a_s = onq.quant_nvfp4(xf[rows], g_x)
        np.testing.assert_array_equal(xc[rows], a_p, err_msg=f"activation codes, rows {r}..")
        np.testing.assert_array_equal(ofp4.sf_from_mma_layout(xs[r * 32:(r + nr) * 32], nr, 32), a_s)
        ref_c, ref_s, _ = ofp4.gated_up_nvfp4(a_p, a_s, g_x, q1, q3, g_h)
        got_s = ofp4.sf_from_mma_layout(hs[r * 128:(r + nr) * 128], nr, 128)
        bad_s += int((got_s != ref_s).sum())
        bad_c += int((hc[rows] != ref_c).sum())
        # the down GEMM on the kernel's own h: exact block sums, FP32 accumulation order
        worst_down = max(worst_down, rel_l2(y[rows], ofp4.nvfp4_gemm(hc[rows], got_s, g_h, *q2)))
    # SiLU through tanh.approx and FP32 accumulation order move h across an NVFP4
    # decision point only rarely (the small-shape test's bounds)
    assert bad_s / (M3 * 128) < 2e-3
    assert bad_c / (M3 * 1024) < 5e-3
    assert worst_down < 1e-5


# ---------------------------------------------------------------------------
# config 4: INT8 SmoothQuant AR prefill, M = 64 x 256
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n,k", [(3840, 1280), (1280, 1280), (5120, 1280), (1280, 5120)])
def test_cfg4_int8_prefill_every_row_bit_exact(lib, n, k):
    from inspark_proper_format_b200.gemm import scaled_gemm
    m = 64 * 256
    g = np.random.default_rng(n + k)
    a = np.clip(np.rint(g.standard_normal((m, k)) * 40), -128, 127).astype(np.int8)
    w = g.integers(-127, 128, (n, k), dtype=np.int8)
    ws = (g.random(n) * 1e-3 + 1e-5).astype(np.float32)
    bias = (g.standard_normal(n) * 0.1).astype(np.float32)
    y = scaled_gemm(dev(a), dev(w), a_scale=1.0 / 127, w_scale=dev(ws), bias=dev(bias),
                    out_dtype=torch.bfloat16).float().cpu().numpy()
    for r in range(0, m, ROWS):
        ref = og.int8_gemm(a[r:r + ROWS], w, np.float32(1.0 / 127), ws, bias, out="bf16")
        np.testing.assert_array_equal(y[r:r + ROWS], ref, err_msg=f"rows {r}..")


# ---------------------------------------------------------------------------
# config 5: BigVGAN anti-aliased Snake FIR
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("b,c,t", [(64, 512, 16384), (8, 256, 65536)])
def test_cfg5_fir_whole_micro_batch(b, c, t):
    from inspark_proper_format_b200.alias_free import fir_snake, kaiser_sinc_filter, snake_inverse_beta
    gen = torch.Generator(device="cuda").manual_seed(c)
    x = torch.randn(b, c, t, device="cuda", generator=gen) * 0.5
    alpha = torch.rand(c, device="cuda", generator=gen) * 1.5 + 0.5
    ib = snake_inverse_beta(alpha).contiguous()
    filt = kaiser_sinc_filter().cuda()
    y = fir_snake(x, filt, filt, alpha, ib)
    num = den = 0.0
    worst = 0.0
    for u in range(0, b, 4):
        ref = activation1d_f64(x[u:u + 4], filt, alpha, ib)
        d = (y[u:u + 4].double() - ref)
        num += float((d * d).sum())
        den += float((ref * ref).sum())
        worst = max(worst, float(d.abs().max()))
    assert (num / den) ** 0.5 < 2e-6          # FP32 kernel vs float64 reference
    assert worst < 2e-5
