"""Generate golden vectors by running the reference's own PyTorch modules.

Run from the repository root, in a container where the reference checkout is
available (it is NOT needed to run the tests):

    PYTHONPATH=<reference>/src:<reference> python tests/golden/make_golden.py <reference>

Every fixture is a small ``.npz`` produced by calling reference code
(xiro2416/inspark_proper_format) on seeded inputs; ``MANIFEST.sha256`` pins
the bytes.  The reference publishes no known-answer vectors for this path, so
these are the parity anchors for the oracle.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _save(name, **arrays):
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **arrays)
    return path


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _fp8_codes(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy()


def activations(rows, k, outliers, factor, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    idx = torch.randperm(k, generator=g)[:outliers]
    x[:, idx] *= factor
    return x


def main(reference_root: str):
    sys.path[:0] = [str(Path(reference_root) / "src"), str(Path(reference_root))]
    from inspark_infer.build.unified_acoustic_export import ExportWeightOp, StaticAliasFree, _QDQ
    from inspark_infer.models.indextts2.dspark.draft import RMSNorm as QwenRMSNorm
    from inspark_infer.models.indextts2.upstream.s2mel.modules.bigvgan.activations import Snake, SnakeBeta
    from inspark_infer.models.indextts2.upstream.s2mel.modules.bigvgan.alias_free_activation.torch.act import Activation1d
    from inspark_infer.models.indextts2.upstream.s2mel.modules.bigvgan.alias_free_activation.torch.filter import kaiser_sinc_filter1d
    from inspark_infer.models.indextts2.upstream.s2mel.modules.gpt_fast.model import RMSNorm
    from inspark_infer.models.zipvoice.reference.models.modules.scaling import BiasNorm
    from inspark_infer.quantization.unified import smoothing_scale
    from inspark_infer.quantization.weights import pack_weight
    from inspark_infer.runtime.zipvoice_fp8.quantization import FP8Linear, export_qdq

    torch.set_num_threads(8)
    written = []
    e4m3_zero = torch.zeros((), dtype=torch.float8_e4m3fn)

    # --- norm -> static E4M3 (config 1 front end): gpt_fast RMSNorm + _QDQ -------------
    x = activations(256, 512, 4, 20.0, 0).bfloat16()
    g = torch.Generator().manual_seed(1)
    norm = RMSNorm(512, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(512, generator=g) * 0.2 + 0.9)
        y = norm(x)                                   # FP32 (BF16 * FP32 gamma)
        scale = torch.tensor(float(y.abs().amax()) / 448.0)
        qdq = _QDQ.apply(y, scale, e4m3_zero, 0)
        codes = (y.float() / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    written.append(_save("normquant_gptfast_e4m3", x_bf16=_bf16_bits(x), gamma=norm.weight.detach().numpy(),
                         eps=np.float32(1e-6), scale=np.float32(scale), y=y.numpy(), qdq=qdq.numpy(),
                         codes=_fp8_codes(codes)))

    # --- Qwen-style RMSNorm (gamma in FP32, one rounding) + _QDQ ---------------------
    qn = QwenRMSNorm(512, eps=1e-6)
    with torch.no_grad():
        qn.weight.copy_(norm.weight)
        y = qn(x)                                     # BF16
        scale = torch.tensor(float(y.float().abs().amax()) / 448.0)
        qdq = _QDQ.apply(y.float(), scale, e4m3_zero, 0)
        codes = (y.float() / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    written.append(_save("normquant_qwen_e4m3", x_bf16=_bf16_bits(x), gamma=qn.weight.detach().numpy(),
                         eps=np.float32(1e-6), scale=np.float32(scale), y_bf16=_bf16_bits(y), qdq=qdq.numpy(),
                         codes=_fp8_codes(codes)))

    # --- gpt_fast AdaptiveLayerNorm (RMSNorm + per-utterance FP32 affine) + _QDQ -------
    from inspark_infer.models.indextts2.upstream.s2mel.modules.gpt_fast.model import AdaptiveLayerNorm
    ada = AdaptiveLayerNorm(512, RMSNorm(512, eps=1e-6))
    with torch.no_grad():
        ada.norm.weight.copy_(norm.weight)
        ga = torch.Generator().manual_seed(7)
        ada.project_layer.weight.copy_(torch.randn(1024, 512, generator=ga) * 0.02)
        ada.project_layer.bias.copy_(torch.randn(1024, generator=ga) * 0.1
                                     + torch.cat([torch.ones(512), torch.zeros(512)]))
        emb = torch.randn(4, 1, 512, generator=ga)             # 4 utterances x 64 frames
        y = ada(x.view(4, 64, 512), emb).reshape(256, 512)     # FP32
        w, b = torch.split(ada.project_layer(emb), 512, dim=-1)
        scale = torch.tensor(float(y.abs().amax()) / 448.0)
        codes = (y / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    written.append(_save("normquant_adaln_e4m3", x_bf16=_bf16_bits(x), gamma=ada.norm.weight.detach().numpy(),
                         eps=np.float32(1e-6), ada_w=w.reshape(4, 512).numpy(), ada_b=b.reshape(4, 512).numpy(),
                         rows_per_group=np.int64(64), scale=np.float32(scale), y=y.numpy(), codes=_fp8_codes(codes)))

    # --- learned Conv1d / ConvTranspose1d through ExportWeightOp (FP8 Q/DQ, FP32 conv) --
    gc = torch.Generator().manual_seed(11)
    conv = torch.nn.Conv1d(64, 48, 7, padding=9, dilation=3)
    deconv = torch.nn.ConvTranspose1d(32, 24, 8, stride=4, padding=2)
    with torch.no_grad():
        for mod in (conv, deconv):
            mod.weight.copy_(torch.randn(mod.weight.shape, generator=gc) * 0.05)
            mod.bias.copy_(torch.randn(mod.bias.shape, generator=gc) * 0.1)
        xc = torch.randn(2, 64, 40, generator=gc)
        xd = torch.randn(2, 32, 20, generator=gc)
        sc = conv.weight.abs().amax(dim=(1, 2)) / 448
        sd = deconv.weight.abs().amax(dim=(0, 2)) / 448
        op_c = ExportWeightOp(conv, {"precision": "fp8", "input_scale": float(xc.abs().max()) / 448,
                                     "weight_scale": sc.tolist(), "weight_axis": 0})
        op_d = ExportWeightOp(deconv, {"precision": "fp8", "input_scale": float(xd.abs().max()) / 448,
                                       "weight_scale": sd.tolist(), "weight_axis": 1,
                                       "conv_transpose_rewrite": "zero_insert_conv"})
        yc, yd = op_c(xc), op_d(xd)
    written.append(_save("conv_fp8_export", x=xc.numpy(), w=conv.weight.detach().numpy(),
                         bias=conv.bias.detach().numpy(),
                         in_scale=np.float32(op_c.input_scale), w_scale=op_c.weight_scale.numpy(),
                         dilation=np.int64(3), padding=np.int64(9), y=yc.numpy(),
                         xd=xd.numpy(), wd=deconv.weight.detach().numpy(), biasd=deconv.bias.detach().numpy(),
                         in_scale_d=np.float32(op_d.input_scale), w_scale_d=op_d.weight_scale.numpy(),
                         stride_d=np.int64(4), padding_d=np.int64(2), yd=yd.numpy()))

    # --- Zipformer BiasNorm (FP32) + ZipVoice export_qdq ------------------------------
    xf = activations(192, 512, 5, 10.0, 2)
    bn = BiasNorm(512)
    with torch.no_grad():
        gb = torch.Generator().manual_seed(3)
        bn.bias.copy_(torch.randn(512, generator=gb) * 0.1)
        bn.log_scale.fill_(0.3)
        bn.eval()
        y = bn(xf)
        scale = torch.tensor(float(y.abs().amax()) / 448.0)
        qdq = export_qdq(y, scale, e4m3_zero)
        codes = (y / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    written.append(_save("normquant_biasnorm_e4m3", x=xf.numpy(), bias=bn.bias.detach().numpy(),
                         log_scale_exp=np.float32(bn.log_scale.detach().exp()), scale=np.float32(scale),
                         y=y.numpy(), qdq=qdq.numpy(), codes=_fp8_codes(codes)))

    # --- per-output-channel E4M3 weight packing (also the dynamic per-row rule) -------
    gw = torch.Generator().manual_seed(4)
    w = (torch.randn(96, 512, generator=gw) * 0.02).bfloat16().float()
    packed, wscale = pack_weight(w)
    written.append(_save("pack_weight", w=w.numpy(), packed=_fp8_codes(packed), scale=wscale.numpy()))

    # --- FP8 W8A8 linear, ExportWeightOp (dequantized FP32 reference) ----------------
    gl = torch.Generator().manual_seed(5)
    lin = torch.nn.Linear(512, 256, bias=True)
    with torch.no_grad():
        lin.weight.copy_((torch.randn(256, 512, generator=gl) * 0.02).bfloat16().float())
        lin.bias.copy_(torch.randn(256, generator=gl) * 0.1)
    a = activations(160, 512, 4, 20.0, 6)
    in_scale = float(a.abs().amax()) / 448.0
    op = ExportWeightOp(lin, dict(precision="fp8", input_scale=in_scale)).prepare_reference_weights()
    with torch.no_grad():
        out = op(a)
        a_codes = (a / torch.tensor(in_scale)).clamp(-448, 448).to(torch.float8_e4m3fn)
        w_codes = (lin.weight / op.weight_scale[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    written.append(_save("fp8_linear_export", a=a.numpy(), w=lin.weight.detach().numpy(), bias=lin.bias.detach().numpy(),
                         input_scale=np.float32(in_scale), weight_scale=op.weight_scale.numpy(), out=out.numpy(),
                         a_codes=_fp8_codes(a_codes), w_codes=_fp8_codes(w_codes)))

    # --- ZipVoice FP8Linear (export_qdq + per-tensor weight DQ) -----------------------
    wt_scale = float(lin.weight.abs().amax()) / 448.0
    fl = FP8Linear(lin, in_scale, wt_scale)
    with torch.no_grad():
        out = fl(a)
    written.append(_save("fp8_linear_zipvoice", a=a.numpy(), weight_fp8=_fp8_codes(fl.weight_fp8),
                         bias=lin.bias.detach().numpy(), input_scale=np.float32(in_scale),
                         weight_scale=np.float32(wt_scale), out=out.numpy()))

    # --- INT8 SmoothQuant (alpha = 1): smoothing_scale + ExportWeightOp ---------------
    gi = torch.Generator().manual_seed(7)
    lin8 = torch.nn.Linear(1280, 384, bias=True)
    with torch.no_grad():
        lin8.weight.copy_((torch.randn(384, 1280, generator=gi) * 0.02).bfloat16().float())
        lin8.bias.copy_(torch.randn(384, generator=gi) * 0.1)
    calib = activations(256, 1280, 8, 30.0, 8)
    amax = calib.abs().amax(0)
    smooth = smoothing_scale(amax, lin8.weight.detach(), 1, alpha=1.0)
    smoothed_w = lin8.weight.detach() * smooth[None, :]
    spec = dict(precision="int8", smooth_scale=smooth.tolist(),
                input_scale=max(float((amax / smooth).max()) / 127.0, 1e-12),
                weight_scale=(smoothed_w.abs().amax(1) / 127.0).clamp_min(1e-12).tolist())
    op8 = ExportWeightOp(lin8, spec).prepare_reference_weights()
    a8 = activations(64, 1280, 8, 30.0, 8)        # same outlier channels as calibration
    with torch.no_grad():
        out8 = op8(a8)
        qa = (a8 / smooth).div(torch.tensor(spec["input_scale"])).round().clamp(-128, 127).to(torch.int8)
        qw = (smoothed_w / op8.weight_scale[:, None]).round().clamp(-128, 127).to(torch.int8)
    written.append(_save("int8_smoothquant", a=a8.numpy(), w=lin8.weight.detach().numpy(), bias=lin8.bias.detach().numpy(),
                         amax=amax.numpy(), smooth=smooth.numpy(), input_scale=np.float32(spec["input_scale"]),
                         weight_scale=op8.weight_scale.numpy(), out=out8.numpy(), a_q=qa.numpy(), w_q=qw.numpy()))

    # --- CFM gated-up SwiGLU with static requant (gpt_fast FeedForward + _QDQ) -------
    gg = torch.Generator().manual_seed(9)
    w1 = (torch.randn(256, 512, generator=gg) * 0.02).bfloat16().float()
    w3 = (torch.randn(256, 512, generator=gg) * 0.02).bfloat16().float()
    h_in = activations(128, 512, 4, 20.0, 10)
    in_s = torch.tensor(float(h_in.abs().amax()) / 448.0)
    s1 = (w1.abs().amax(1) / 448.0).clamp_min(1e-12)
    s3 = (w3.abs().amax(1) / 448.0).clamp_min(1e-12)
    with torch.no_grad():
        xa = _QDQ.apply(h_in, in_s, e4m3_zero, 0)
        w1q = _QDQ.apply(w1, s1, torch.zeros(256, dtype=torch.float8_e4m3fn), 0)
        w3q = _QDQ.apply(w3, s3, torch.zeros(256, dtype=torch.float8_e4m3fn), 0)
        hidden = torch.nn.functional.silu(torch.nn.functional.linear(xa, w1q)) * torch.nn.functional.linear(xa, w3q)
        out_s = torch.tensor(float(hidden.abs().amax()) / 448.0)
        hq = _QDQ.apply(hidden, out_s, e4m3_zero, 0)
    written.append(_save("gated_up", x=h_in.numpy(), w1=w1.numpy(), w3=w3.numpy(), input_scale=np.float32(in_s),
                         w1_scale=s1.numpy(), w3_scale=s3.numpy(), output_scale=np.float32(out_s),
                         hidden=hidden.numpy(), out=hq.numpy()))

    # --- BigVGAN alias-free activation: Snake, SnakeBeta(logscale), StaticAliasFree ---
    filt = kaiser_sinc_filter1d(0.25, 0.3, 12).flatten()
    ga = torch.Generator().manual_seed(11)
    c = 16
    snake_act = Activation1d(Snake(c))
    with torch.no_grad():
        snake_act.act.alpha.copy_(torch.rand(c, generator=ga) * 1.5 + 0.5)
    cases = {}
    for t in (1, 2, 5, 12, 301, 1000):
        xs = torch.randn(2, c, t, generator=ga) * 0.5
        with torch.no_grad():
            cases[f"x_{t}"] = xs.numpy()
            cases[f"y_{t}"] = snake_act(xs).numpy()
    static = StaticAliasFree(snake_act, fir_polyphase=True)
    with torch.no_grad():
        cases["y_static_1000"] = static(torch.from_numpy(cases["x_1000"])).numpy()
    beta_act = Activation1d(SnakeBeta(c, alpha_logscale=True))
    with torch.no_grad():
        beta_act.act.alpha.copy_(torch.randn(c, generator=ga) * 0.3)
        beta_act.act.beta.copy_(torch.randn(c, generator=ga) * 0.3)
        cases["y_beta_301"] = beta_act(torch.from_numpy(cases["x_301"])).numpy()
    written.append(_save("fir", filter=filt.numpy(), up=snake_act.upsample.filter.flatten().numpy(),
                         down=snake_act.downsample.lowpass.filter.flatten().numpy(),
                         alpha=snake_act.act.alpha.detach().numpy(),
                         log_alpha=beta_act.act.alpha.detach().numpy(), log_beta=beta_act.act.beta.detach().numpy(),
                         **cases))

    # the reference's FP8 Triton kernels, through Triton's CPU interpreter (own process:
    # the interpreter is switched on by an environment variable read at import)
    import os
    import subprocess
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(sys.path[:2] + [os.environ.get("PYTHONPATH", "")]))
    out = subprocess.run([sys.executable, str(HERE / "make_golden_triton.py"), reference_root], env=env, check=True,
                         capture_output=True, text=True).stdout
    written += [HERE / name for name in out.split()]

    lines = [f"{hashlib.sha256(p.read_bytes()).hexdigest()}  {p.name}" for p in sorted(written)]
    (HERE / "MANIFEST.sha256").write_text("\n".join(lines) + "\n")
    for line in lines:
        print(line)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
