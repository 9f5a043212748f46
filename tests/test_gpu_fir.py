"""GPU parity: fused BigVGAN FIR/Snake/FIR kernel vs the oracle and the reference fixtures."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fir as ofir

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def ops():
    from inspark_proper_format_b200 import alias_free
    return alias_free


def _params(c, seed):
    g = torch.Generator().manual_seed(seed)
    alpha = torch.rand(c, generator=g) * 1.5 + 0.5
    return alpha, torch.from_numpy(ofir.snake_inverse_beta(alpha.numpy()))


@pytest.mark.parametrize("b,c,t", [(1, 1, 1), (1, 3, 2), (2, 4, 5), (1, 2, 1023), (1, 2, 1025), (2, 3, 1028),
                                   (1, 2, 2047), (1, 2, 2048), (1, 2, 2049),
                                   (2, 8, 4095), (1, 4, 6145), (3, 5, 301),
                                   # T % 4 == 0: streamed by bulk copies, incl. tiles that end past T
                                   (1, 1, 4), (2, 3, 8), (1, 2, 12), (1, 3, 2052), (2, 2, 4100), (1, 3, 6144),
                                   (3, 7, 16384)])
def test_fir_matches_oracle(ops, b, c, t):
    f_up, f_down = ofir.bigvgan_filters()
    g = torch.Generator().manual_seed(t)
    x = torch.randn(b, c, t, generator=g) * 0.5
    alpha, ib = _params(c, t)
    y = ops.fir_snake(x.cuda(), torch.from_numpy(f_up).cuda(), torch.from_numpy(f_down).cuda(),
                      alpha.cuda(), ib.cuda()).cpu().numpy()
    ref = ofir.alias_free_snake(x.numpy(), f_up, f_down, alpha.numpy(), ib.numpy())
    assert rel_l2(y, ref) < 2e-6
    np.testing.assert_allclose(y, ref, atol=3e-6, rtol=0)


@pytest.mark.parametrize("t", [1, 2, 5, 12, 301, 1000])
def test_fir_golden_activation1d(ops, t):
    d = np.load(GOLDEN / "fir.npz")
    alpha = torch.from_numpy(d["alpha"])
    ib = torch.from_numpy(ofir.snake_inverse_beta(d["alpha"]))
    y = ops.fir_snake(torch.from_numpy(d[f"x_{t}"]).cuda(), torch.from_numpy(d["up"]).cuda(),
                      torch.from_numpy(d["down"]).cuda(), alpha.cuda(), ib.cuda()).cpu().numpy()
    assert rel_l2(y, d[f"y_{t}"]) < 2e-6


def test_tiled_fir_logscale_snakebeta(ops):
    d = np.load(GOLDEN / "fir.npz")
    tiled = ops.TiledFIR(torch.from_numpy(d["up"]).cuda(), torch.from_numpy(d["down"]).cuda(),
                         torch.from_numpy(d["log_alpha"]).cuda(), torch.from_numpy(d["log_beta"]).cuda())
    y = tiled(torch.from_numpy(d["x_301"]).cuda()).cpu().numpy()
    assert rel_l2(y, d["y_beta_301"]) < 2e-6
    small = ops.SmallFIR(torch.from_numpy(d["up"]).cuda(), torch.from_numpy(d["down"]).cuda(),
                         torch.from_numpy(d["log_alpha"]).cuda(), torch.from_numpy(d["log_beta"]).cuda())
    assert rel_l2(small(torch.from_numpy(d["x_301"]).cuda()).cpu().numpy(), d["y_beta_301"]) < 2e-6


def test_fir_quant_int8(ops):
    f_up, f_down = ofir.bigvgan_filters()
    c, t = 6, 3000
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, c, t, generator=g) * 0.5
    log_a = torch.randn(c, generator=g) * 0.3
    log_b = torch.randn(c, generator=g) * 0.3
    smooth = torch.rand(c, generator=g) + 0.5
    scale = 0.01
    q = ops.fir_quant(x.cuda(), torch.from_numpy(f_up).cuda(), torch.from_numpy(f_down).cuda(), log_a.cuda(),
                      log_b.cuda(), smooth.cuda(), scale).cpu().numpy()
    a = np.exp(log_a.numpy()).astype(np.float32)
    ib = (np.float32(1) / (np.exp(log_b.numpy()).astype(np.float32) + np.float32(1e-9))).astype(np.float32)
    ref = ofir.alias_free_snake_int8(x.numpy(), f_up, f_down, a, ib, smooth.numpy(), scale)
    # FP32 FIR values sitting on an INT8 rounding tie may land on either side.
    assert np.mean(q != ref) < 1e-4
    assert np.abs(q.astype(int) - ref.astype(int)).max() <= 1


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_fir_quant_int8_golden(ops, case):
    """Against ``deployment/multibatch/fir_quant_kernel.py`` itself (Triton CPU
    interpreter fixture): log-scale alpha/beta, the INT8 rule, ragged F."""
    d = np.load(GOLDEN / "fir_quant.npz")
    q = ops.fir_quant(torch.from_numpy(d[f"{case}_x"]).cuda(), torch.from_numpy(d["up"]).cuda(),
                      torch.from_numpy(d["down"]).cuda(), torch.from_numpy(d[f"{case}_log_alpha"]).cuda(),
                      torch.from_numpy(d[f"{case}_log_beta"]).cuda(), torch.from_numpy(d[f"{case}_smooth"]).cuda(),
                      float(d[f"{case}_scale"][0])).cpu().numpy()
    ref = d[f"{case}_q"]
    # the reference divides sin^2 by (beta + 1e-9), the kernel multiplies by the
    # reciprocal, and the sines differ by ulps: values on an INT8 tie may flip by one
    assert np.count_nonzero(q != ref) <= max(1, q.size // 10000)
    assert np.abs(q.astype(int) - ref.astype(int)).max() <= 1


def test_fused_alias_free_install_swaps_activation1d(ops):
    class Activation1d(torch.nn.Module):   # same attribute surface as the reference module
        def __init__(self, c):
            super().__init__()
            f_up, f_down = ofir.bigvgan_filters()
            self.up_ratio = self.down_ratio = 2
            self.act = torch.nn.Module()
            self.act.alpha = torch.nn.Parameter(torch.rand(c) + 0.5)
            self.act.alpha_logscale = False
            self.upsample = torch.nn.Module()
            self.upsample.kernel_size = 12
            self.upsample.register_buffer("filter", torch.from_numpy(f_up).view(1, 1, 12))
            self.downsample = torch.nn.Module()
            self.downsample.lowpass = torch.nn.Module()
            self.downsample.lowpass.kernel_size = 12
            self.downsample.lowpass.register_buffer("filter", torch.from_numpy(f_down).view(1, 1, 12))

    voc = torch.nn.Sequential(torch.nn.Sequential(Activation1d(4)), Activation1d(4)).cuda()
    changed = ops.install(voc)
    assert changed == ["vocoder.0.0", "vocoder.1"]
    x = torch.randn(2, 4, 100, device="cuda") * 0.5
    y = voc[1](x)
    a = voc[1].alpha.cpu().numpy()
    ref = ofir.alias_free_snake(x.cpu().numpy(), *ofir.bigvgan_filters(), a, ofir.snake_inverse_beta(a))
    assert rel_l2(y.cpu().numpy(), ref) < 2e-6


def test_full_size_row_properties(ops):
    """A full cfg-5 row length (T = 65536) on a few channels: parity and constant-signal fixed point."""
    f_up, f_down = ofir.bigvgan_filters()
    c, t = 3, 65536
    x = torch.randn(1, c, t, generator=torch.Generator().manual_seed(5)) * 0.5
    alpha, ib = _params(c, 6)
    y = ops.fir_snake(x.cuda(), torch.from_numpy(f_up).cuda(), torch.from_numpy(f_down).cuda(), alpha.cuda(), ib.cuda())
    ref = ofir.alias_free_snake(x.numpy(), f_up, f_down, alpha.numpy(), ib.numpy())
    assert rel_l2(y.cpu().numpy(), ref) < 2e-6
    # A constant input is a fixed point of both unit-gain filters: y == Snake(x).
    const = torch.full((1, c, 4096), 0.3).cuda()
    yc = ops.fir_snake(const, torch.from_numpy(f_up).cuda(), torch.from_numpy(f_down).cuda(), alpha.cuda(), ib.cuda())
    expect = 0.3 + ib.numpy()[:, None] * np.sin(0.3 * alpha.numpy()[:, None]) ** 2
    np.testing.assert_allclose(yc[0].cpu().numpy(), np.broadcast_to(expect, (c, 4096)), rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("alpha_scale,x_scale", [(60.0, 0.5), (1.0, 3e5), (1.0, 1e-30)])
def test_fir_wide_snake_arguments(ops, alpha_scale, x_scale):
    """Snake arguments from tiny to beyond the polynomial's reduction range
    (|alpha v| > 1e6 takes CUDA's sinf): still within the FIR tolerance."""
    f_up, f_down = ofir.bigvgan_filters()
    c, t = 4, 3001
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, c, t, generator=g) * x_scale
    alpha = (torch.rand(c, generator=g) * 1.5 + 0.5) * alpha_scale
    ib = torch.from_numpy(ofir.snake_inverse_beta(alpha.numpy()))
    y = ops.fir_snake(x.cuda(), torch.from_numpy(f_up).cuda(), torch.from_numpy(f_down).cuda(), alpha.cuda(),
                      ib.cuda()).cpu().numpy()
    ref = ofir.alias_free_snake(x.numpy(), f_up, f_down, alpha.numpy(), ib.numpy())
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) < 2e-6
