"""Golden vectors from two more reference Triton kernels (run on the CPU through
Triton's interpreter) and from the reference's eager FP8 layer modules.

    PYTHONPATH=<reference>/src:<reference> python tests/golden/make_golden_kernels.py <reference>

Writes (and adds to ``MANIFEST.sha256``):
  * ``fir_quant.npz``: ``deployment/multibatch/fir_quant_kernel.py:10-40`` (FP32
    polyphase up-FIR, log-scale Snake, low-pass, then the signed INT8 rule
    ``rint(div_rn(div_rn(y, smooth[c]), scale))``), grid and constexprs as its
    plugin launches it (``fir_quant_plugin.py:26-30``: BLOCK 256, HIGH 512, grid
    (B*C, cdiv(F, 248)));
  * ``int8_nonlinear_value.npz``: ``ops/tensorrt/zipvoice/a1007/b1/
    int8_nonlinear_value_runtime_kernel.py:6-34`` (one [T, 1, 512] batch) and its
    16-group variant ``.../b16_geo1/int8_nonlinear_value_runtime_kernel.py``
    ([T, 16, 512]), at the plugin's tile sizes (``int8_nonlinear_value_aot.py``);
  * ``fp8_layer_eager.npz``: one FM layer built from the reference's own
    modules — gpt_fast ``RMSNorm`` (``gpt_fast/model.py:246-258``), ``_QDQ``
    (``build/unified_acoustic_export.py:22-36``) and ten FP8 ``ExportWeightOp``
    linears with ``prepare_reference_weights`` (``:75-216``) — the arithmetic
    the CPU reference arm of ``bench.py`` times.

The interpreter has no ``triton.language.extra.cuda.libdevice``; the kernels'
``libdevice`` global is pointed at numpy equivalents (``exp``, ``sin``,
``tanh``, ``rint``, ``div_rn`` = IEEE division), so the fixtures pin the
kernels' indexing, rounding rules and epilogue order, with numpy's ``sin``,
``exp`` and ``tanh`` standing in for CUDA's (a few ulps apart).
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def _libdevice_shim():
    from types import SimpleNamespace

    import triton.language as tl
    from triton.runtime.interpreter import TensorHandle

    def wrap(fn):
        def f(*xs, _semantic=None):
            data = fn(*[x.handle.data for x in xs]).astype(xs[0].handle.data.dtype)
            return tl.core.tensor(TensorHandle(data, xs[0].handle.dtype.scalar), xs[0].type)
        return f
    return SimpleNamespace(tanh=wrap(np.tanh), exp=wrap(np.exp), sin=wrap(np.sin), rint=wrap(np.rint),
                           div_rn=wrap(np.divide))


def fir_quant_fixture(g):
    import triton

    import deployment.multibatch.fir_quant_kernel as mod
    from inspark_infer.models.indextts2.upstream.s2mel.modules.bigvgan.alias_free_activation.torch.filter import \
        kaiser_sinc_filter1d
    mod.fir_quant.fn.__globals__["libdevice"] = _libdevice_shim()
    filt = kaiser_sinc_filter1d(0.25, 0.3, 12).reshape(-1).float().contiguous()
    arrays = {"up": filt.numpy(), "down": filt.numpy()}
    for name, (b, c, f) in {"a": (2, 3, 600), "b": (1, 4, 249), "c": (2, 2, 37)}.items():
        x = torch.randn(b, c, f, generator=g) * 0.5
        x[0, 0, :7] *= 8                                         # large Snake arguments at the left edge
        log_a = torch.randn(c, generator=g) * 0.3
        log_b = torch.randn(c, generator=g) * 0.3
        smooth = torch.rand(c, generator=g) + 0.5
        scale = torch.tensor([0.006])
        out = torch.zeros(b, c, f, dtype=torch.int8)
        mod.fir_quant[(b * c, triton.cdiv(f, 248))](x, filt, filt, log_a, log_b, smooth, scale, out, c, f, 256, 512)
        arrays.update({f"{name}_x": x.numpy(), f"{name}_log_alpha": log_a.numpy(), f"{name}_log_beta": log_b.numpy(),
                       f"{name}_smooth": smooth.numpy(), f"{name}_scale": scale.numpy(), f"{name}_q": out.numpy()})
    return arrays


def nonlinear_value_fixture(g):
    import triton

    import inspark_infer.ops.tensorrt.zipvoice.a1007.b16_geo1.int8_nonlinear_value_runtime_kernel as k16
    import inspark_infer.ops.tensorrt.zipvoice.a1007.b1.int8_nonlinear_value_runtime_kernel as k1
    shim = _libdevice_shim()
    w = torch.randint(-127, 128, (1152, 512), generator=g, dtype=torch.int8)   # the exported [1152, 512]
    arrays = {"w": w.numpy()}
    for name, mod, groups, steps, (bm, bn, bk) in (("b1", k1, 1, 70, (128, 32, 64)),
                                                    ("b16", k16, 16, 9, (64, 64, 128))):
        mod.int8_nonlinear_value.fn.__globals__["libdevice"] = shim
        q = torch.randint(-128, 128, (steps, groups, 512), generator=g, dtype=torch.int8)
        as_ = torch.tensor([0.011])
        ws = torch.rand(1152, generator=g) * 2e-3 + 1e-4
        bias = torch.randn(1152, generator=g) * 0.1
        v = torch.zeros(1, groups, steps, 384)
        gate = torch.zeros(steps, groups, 384)
        grid = (triton.cdiv(steps * groups, bm), triton.cdiv(384, bn))
        mod.int8_nonlinear_value[grid](q, w, as_, ws, bias, v, gate, steps, bm, bn, bk)
        arrays.update({f"{name}_q": q.numpy(), f"{name}_as": as_.numpy(),
                       f"{name}_ws": ws.numpy(), f"{name}_bias": bias.numpy(), f"{name}_value": v.numpy(),
                       f"{name}_gate": gate.numpy()})
    return arrays


# (N, K) of the ten projections in the order oracle/torch_path.FP8Layer takes them:
# ff0 in/out, ff1 in/out, ff2 in/out, attn in, attn out, conv in, conv out (hidden 64)
LAYER = [(192, 64), (64, 192), (192, 64), (64, 192), (192, 64), (64, 192), (192, 64), (64, 64), (128, 64),
         (64, 128)]


def eager_layer_fixture(g):
    from torch import nn

    from inspark_infer.build.unified_acoustic_export import ExportWeightOp, _QDQ
    from inspark_infer.models.indextts2.upstream.s2mel.modules.gpt_fast.model import RMSNorm
    rows, hidden = 40, 64
    x = torch.randn(rows, hidden, generator=g)
    x[:, torch.randperm(hidden, generator=g)[:2]] *= 10
    x = x.bfloat16()
    norm = RMSNorm(hidden, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(hidden, generator=g) * 0.2 + 0.9)
    norm_scale = torch.tensor(0.02)
    act_scales = [torch.tensor(v) for v in (0.05, 0.04, 0.06, 0.03)]    # ff0/ff1/ff2 hidden, conv hidden
    ops, arrays = [], {}
    for i, (n, k) in enumerate(LAYER):
        lin = nn.Linear(k, n, bias=False)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, generator=g) * 0.02)
        ws = (lin.weight.detach().abs().amax(1) / 448).clamp_min(1e-12)
        in_scale = norm_scale if i in (0, 2, 4, 6, 7, 8) else act_scales[{1: 0, 3: 1, 5: 2, 9: 3}[i]]
        op = ExportWeightOp(lin, {"precision": "fp8", "input_scale": float(in_scale), "weight_scale": ws})
        op.prepare_reference_weights()
        ops.append(op)
        arrays[f"w{i}"] = lin.weight.detach().numpy()
        arrays[f"wq{i}"] = op.weight.numpy()                  # the folded (Q/DQ'd) weight the reference uses
    with torch.no_grad():
        normed = norm(x)                                       # bf16 normalized * gamma -> FP32
        a = _QDQ.apply(normed, norm_scale, torch.zeros((), dtype=torch.float8_e4m3fn), 0)
        outs = []
        for f in range(3):
            h = ops[2 * f](normed)
            outs.append(ops[2 * f + 1](h))
        outs.append(ops[6](normed))
        outs.append(ops[7](normed))
        c1 = ops[8](normed)
        outs.append(ops[9](c1))
    for i, o in enumerate(outs):
        arrays[f"y{i}"] = o.numpy()
    arrays.update(x_bits=x.view(torch.int16).numpy().view(np.uint16), gamma=norm.weight.detach().numpy(),
                  norm_scale=np.float32(norm_scale), act_scales=np.array([float(s) for s in act_scales], np.float32),
                  a=a.numpy())
    return arrays


def main(reference_root: str):
    sys.path[:0] = [str(Path(reference_root) / "src"), str(Path(reference_root))]
    torch.set_num_threads(8)
    g = torch.Generator().manual_seed(31)
    written = []
    for name, fn in (("fir_quant", fir_quant_fixture), ("int8_nonlinear_value", nonlinear_value_fixture),
                     ("fp8_layer_eager", eager_layer_fixture)):
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **fn(g))
        written.append(path)
    manifest = HERE / "MANIFEST.sha256"
    lines = {ln.split()[1]: ln for ln in manifest.read_text().splitlines() if ln.strip()}
    for p in written:
        lines[p.name] = f"{hashlib.sha256(p.read_bytes()).hexdigest()}  {p.name}"
        print(p.name)
    manifest.write_text("".join(lines[k] + "\n" for k in sorted(lines)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_kernels.py <reference checkout>")
    main(sys.argv[1])
