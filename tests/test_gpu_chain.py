"""GPU: one config-2 layer fragment launched back to back, as the stack runs it --
norm-quant -> FP8 GEMM with E4M3 requant -> FP8 GEMM with BF16 output -> the next
norm-quant -- with no synchronization between the launches (the kernels overlap
their prologues with the previous kernel's tail), each stage checked against the
oracle applied to the GPU's own previous stage."""
import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import normquant as onq
from oracle.formats import bf16_round, e4m3_decode

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _weight(n, k, g):
    w = torch.randn(n, k, generator=g) * 0.02
    ws = (w.abs().amax(1) / 448).clamp_min(1e-12)
    return (w / ws[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn), ws


def test_back_to_back_layer_fragment_matches_oracle_stage_by_stage():
    from inspark_proper_format_b200.gemm import scaled_gemm
    from inspark_proper_format_b200.norm_quant import norm_quant
    g = torch.Generator().manual_seed(17)
    m, d, f = 3040, 512, 1536
    x = torch.randn(m, d, generator=g)
    x[:, torch.randperm(d, generator=g)[:5]] *= 10
    x = x.bfloat16()
    gamma = torch.rand(d, generator=g) * 0.2 + 0.9
    gamma2 = torch.rand(d, generator=g) * 0.2 + 0.9
    w_in, s_in = _weight(f, d, g)
    w_out, s_out = _weight(d, f, g)
    b_in = torch.randn(f, generator=g) * 0.01
    b_out = torch.randn(d, generator=g) * 0.01
    s_a, s_h, s_a2 = 0.011, 0.037, 0.013
    dev = torch.device("cuda")
    xd, gd, g2d = x.to(dev), gamma.to(dev), gamma2.to(dev)
    wid, wod, sid, sod, bid, bod = (t.to(dev) for t in (w_in, w_out, s_in, s_out, b_in, b_out))
    torch.cuda.synchronize()
    # four launches, no host synchronization in between
    a, _ = norm_quant(xd, kind="rms_gptfast", fmt="e4m3", gamma=gd, scale=s_a)
    h = scaled_gemm(a, wid, a_scale=s_a, w_scale=sid, bias=bid, out_dtype=torch.float8_e4m3fn, out_inv_scale=1 / s_h)
    y = scaled_gemm(h, wod, a_scale=s_h, w_scale=sod, bias=bod, out_dtype=torch.bfloat16)
    a2, _ = norm_quant(y, kind="rms_gptfast", fmt="e4m3", gamma=g2d, scale=s_a2)
    torch.cuda.synchronize()
    a_c = a.view(torch.uint8).cpu().numpy()
    h_c = h.view(torch.uint8).cpu().numpy()
    y_v = y.float().cpu().numpy()
    a2_c = a2.view(torch.uint8).cpu().numpy()

    ref_a, _ = onq.norm_quant(bf16_round(x.float().numpy()), onq.NORM_RMS_GPTFAST, onq.Q_E4M3_STATIC,
                              gamma=gamma.numpy(), scale=s_a)
    np.testing.assert_array_equal(a_c, ref_a)
    ref_h = og.fp8_gemm(a_c, w_in.view(torch.uint8).numpy(), np.float32(s_a), s_in.numpy(), b_in.numpy(),
                        out="e4m3", out_scale=np.float32(s_h))
    assert np.mean(h_c != ref_h) < 5e-3                          # accumulation-order ties only
    assert rel_l2(e4m3_decode(h_c), e4m3_decode(ref_h)) < 1e-2
    ref_y = og.fp8_gemm(h_c, w_out.view(torch.uint8).numpy(), np.float32(s_h), s_out.numpy(), b_out.numpy(),
                        out="bf16")
    assert rel_l2(y_v, ref_y) < 4e-3                             # BF16 rounding of accumulation-order ulps
    ref_a2, _ = onq.norm_quant(y_v, onq.NORM_RMS_GPTFAST, onq.Q_E4M3_STATIC, gamma=gamma2.numpy(), scale=s_a2)
    np.testing.assert_array_equal(a2_c, ref_a2)


def test_bench_stack_shards_are_slices_of_the_full_batch():
    """The multi-GPU split of ``bench.py``: a rank running utterances [u0, u1) of the
    B64 x 760 batch with the whole-batch calibration computes exactly rows
    [760 u0, 760 u1) of the single-GPU output (two layers, bit-exact)."""
    import bench
    dev = torch.device("cuda", 0)
    full = bench.Stack(dev, layers=2)
    full.run()
    torch.cuda.synchronize()
    ref = full.output.clone()
    scales = full.calibrated_scales()
    del full
    for u0, u1 in ((0, 24), (24, 64)):
        lo, hi = u0 * bench.FRAMES, u1 * bench.FRAMES
        part = bench.Stack(dev, rows=(lo, hi), layers=2, scales=scales)
        part.run()
        torch.cuda.synchronize()
        assert torch.equal(part.output, ref[lo:hi]), (u0, u1)
