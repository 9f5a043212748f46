"""Golden vectors from the reference's own FP8 Triton kernels, run on the CPU
through Triton's interpreter (``TRITON_INTERPRET=1``, set before Triton is
imported; no GPU is involved).

    PYTHONPATH=<reference>/src:<reference> python tests/golden/make_golden_triton.py <reference>

Called by ``make_golden.py`` (which then pins every fixture's bytes in
``MANIFEST.sha256``).  Writes
  * ``conv_matrix_fp8.npz``: ``ops/triton/fp8_conv.conv1d`` (dynamic per-utterance
    scale, weights from ``quantization/weights.pack_weight``) on Conv1d (dilated,
    strided) and ConvTranspose1d (regular and ragged phases, output_padding)
    geometries, FP32 and BF16 inputs;
  * ``fp8_linear_triton.npz``: ``ops/triton/fp8.linear`` (dynamic per-row scale),
    single and split-K tiles.
The interpreter's float -> E4M3 cast mishandles values that round up into the
next binade (125.9 -> 64 instead of 128), a defect of the interpreter, not of
the kernels.  The inputs are therefore exact E4M3 values times a power of two
per utterance (per row for the linear), with one element at 448 times it, so
the dynamic scale is that power of two and every cast is exact: the fixtures
pin the kernels' indexing, scale flow and epilogue, while E4M3 rounding is
pinned by the norm-quant fixtures.  The interpreter also stores FP32 -> BF16 by
truncation (the GPU kernel rounds to nearest), so the BF16 case pins the FP32
value before the store through its truncation.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent

# name: (transpose, ci, co, kw, stride, padding, dilation, output_padding, batch, t, bias, bf16)
CONV_CASES = {
    "dilated": (False, 40, 48, 7, 1, 9, 3, 0, 2, 50, True, False),
    "strided": (False, 32, 24, 4, 2, 1, 1, 0, 2, 37, False, False),
    "deconv": (True, 32, 24, 8, 4, 2, 1, 0, 2, 20, True, False),
    "deconv_ragged": (True, 24, 16, 3, 2, 1, 2, 1, 3, 11, True, False),
    "bf16": (False, 136, 40, 3, 1, 1, 1, 0, 2, 33, True, True),
}


def exact_e4m3(shape, generator, exponents, lead_dim_rows=False):
    """Values e4m3(randn) * 2**exponents[b] (b = first index), the first
    element of every b slice set to 448 * 2**exponents[b]."""
    v = (torch.randn(shape, generator=generator) * 40).to(torch.float8_e4m3fn).float()
    v.view(shape[0], -1)[:, 0] = 448.0
    return v * torch.tensor([2.0 ** e for e in exponents]).reshape((-1,) + (1,) * (len(shape) - 1))


def main(reference_root: str):
    sys.path[:0] = [str(Path(reference_root) / "src"), str(Path(reference_root))]
    from types import SimpleNamespace

    from inspark_infer.ops.planning.planner import Tile
    from inspark_infer.ops.triton import fp8 as tfp8
    from inspark_infer.ops.triton import fp8_conv
    from inspark_infer.quantization.weights import pack_weight

    written = []
    g = torch.Generator().manual_seed(21)
    arrays = {}
    tile = SimpleNamespace(bm=32, bn=32, bk=32, warps=4, stages=1)
    for name, (tr, ci, co, kw, s, pad, dil, op, b, t, has_bias, bf16) in CONV_CASES.items():
        mod = (torch.nn.ConvTranspose1d(ci, co, kw, stride=s, padding=pad, dilation=dil, output_padding=op)
               if tr else torch.nn.Conv1d(ci, co, kw, stride=s, padding=pad, dilation=dil))
        with torch.no_grad():
            mod.weight.copy_(torch.randn(mod.weight.shape, generator=g) * 0.05)
            mod.bias.copy_(torch.randn(mod.bias.shape, generator=g) * 0.1)
        weight = mod.weight.detach()
        dense = weight.permute(1, 0, 2) if tr else weight          # quantization/precision.py:34-36
        packed, scales = pack_weight(dense.reshape(co, ci * kw))
        x = exact_e4m3((b, ci, t), g, [-9 - i for i in range(b)])
        if bf16:
            x = x.bfloat16()
        bias = mod.bias.detach() if has_bias else None
        y = fp8_conv.conv1d(x, packed, scales, bias, ci, co, kw, s, pad, dil, tr, op, tile)
        arrays[f"{name}_x"] = x.float().numpy()
        arrays[f"{name}_w"] = weight.numpy()
        arrays[f"{name}_packed"] = packed.view(torch.uint8).numpy()
        arrays[f"{name}_scales"] = scales.numpy()
        if has_bias:
            arrays[f"{name}_bias"] = bias.numpy()
        arrays[f"{name}_y"] = y.float().numpy()
        arrays[f"{name}_geom"] = np.array([tr, ci, co, kw, s, pad, dil, op, int(bf16)], np.int64)
    path = HERE / "conv_matrix_fp8.npz"
    np.savez_compressed(path, **arrays)
    written.append(path)

    arrays = {}
    w = torch.randn(96, 320, generator=g) * 0.03
    packed, scales = pack_weight(w)
    x = exact_e4m3((37, 320), g, [-(i % 7) - 4 for i in range(37)])
    bias = torch.randn(96, generator=g) * 0.1
    for split in (1, 3):
        y = tfp8.linear(x, packed, scales, bias, Tile(32, 32, 32, 4, 1, split_k=split))
        arrays[f"y_split{split}"] = y.numpy()
    arrays.update(x=x.numpy(), w=w.numpy(), packed=packed.view(torch.uint8).numpy(), scales=scales.numpy(),
                  bias=bias.numpy())
    path = HERE / "fp8_linear_triton.npz"
    np.savez_compressed(path, **arrays)
    written.append(path)
    for p in written:
        print(p.name)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_triton.py <reference checkout>")
    main(sys.argv[1])
