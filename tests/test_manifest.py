"""Loader for the reference's exported checkpoints: a synthetic export written the
way ``scripts/export_weights.py:38-75`` and ``scripts/export_nvfp4_weights.py:25-46``
write theirs (CPU), and the mapped roles run on the GPU against the oracle."""
import json

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import normquant as onq
from oracle import nvfp4 as ofp4


def synthetic_export(seed=0):
    """One component with an FP8, an INT8, an NVFP4, a BF16 and a conv role, in the
    exporters' storage format (codes, scales, manifest)."""
    g = torch.Generator().manual_seed(seed)
    state, roles = {}, {}
    # fp8 / int8 (export_weights.py: w / scale, clamp, cast; INT8 smoothed first)
    for role, key, prec in (("cfm.blocks.0.w1", "transformer.layers.0.w1.weight", "fp8"),
                            ("target.blocks.0.qkv", "layers.0.qkv.weight", "int8")):
        w = torch.randn(192, 256, generator=g) * 0.02
        spec = {"precision": prec, "weight_axis": 0, "weight_input_axis": 1, "input_scale": 0.0123}
        if prec == "int8":
            smooth = torch.rand(256, generator=g) + 0.5
            w = w * smooth[None, :]
            spec["smooth_scale"] = smooth.tolist()
            state[key + ".smooth_scale"] = smooth
        scale = (w.abs().amax(1) / (127 if prec == "int8" else 448)).clamp_min(1e-12)
        q = (w / scale[:, None]).round().clamp(-128, 127).to(torch.int8) if prec == "int8" else \
            (w / scale[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
        spec["weight_scale"] = scale.tolist()
        state[key] = q
        state[key + ".weight_scale"] = scale
        state[key + ".input_scale"] = torch.tensor(spec["input_scale"])
        state[key[:-len(".weight")] + ".bias"] = torch.randn(192, generator=g) * 0.1
        roles[role] = dict(spec, state_key=key, stored_layout="canonical_weight")
    # nvfp4 (export_nvfp4_weights.py: FP16 matrix, two-level scales, low nibble = even K)
    w = (torch.randn(128, 256, generator=g) * 0.02).half().float()
    packed, scodes, gw = ofp4.quantize_weight(w.numpy())
    key = "transformer.layers.0.w2.weight"
    state[key] = torch.from_numpy(packed)
    state[key + ".block_scale"] = torch.from_numpy(scodes).view(torch.float8_e4m3fn)
    state[key + ".global_scale"] = torch.tensor(float(gw))
    state[key + ".activation_global_scale"] = torch.tensor(float(ofp4.activation_global_scale(4.0)))
    roles["cfm.blocks.0.w2"] = {"precision": "nvfp4", "state_key": key, "block_size": 16, "activation_amax": 4.0,
                                "packed_nibble_order": "low=evenK;high=oddK"}
    # bf16 protected role and a learned conv (3-D) role
    state["proj.weight"] = (torch.randn(64, 256, generator=g) * 0.02).bfloat16()
    roles["cfm.proj"] = {"precision": "bf16", "state_key": "proj.weight"}
    state["conv_pre.weight"] = torch.randn(64, 32, 7, generator=g).to(torch.float8_e4m3fn)
    roles["vocoder.conv_pre"] = {"precision": "fp8", "state_key": "conv_pre.weight", "input_scale": 0.1,
                                 "weight_scale": [0.01] * 64, "weight_axis": 0, "weight_input_axis": 1}
    state["conv_pre.weight.weight_scale"] = torch.full((64,), 0.01)
    state["conv_pre.weight.input_scale"] = torch.tensor(0.1)
    state["conv_pre.bias"] = torch.randn(64, generator=g) * 0.1
    # INT8 SmoothQuant ConvTranspose1d role ([CI, CO, KW]: scales on axis 1, smoothing on 0)
    w = torch.randn(32, 24, 8, generator=g) * 0.05
    smooth = torch.rand(32, generator=g) + 0.5
    w = w * smooth[:, None, None]
    scale = (w.abs().amax(dim=(0, 2)) / 127).clamp_min(1e-12)
    key = "ups.0.0.weight"
    state[key] = (w / scale[None, :, None]).round().clamp(-128, 127).to(torch.int8)
    state[key + ".weight_scale"] = scale
    state[key + ".input_scale"] = torch.tensor(0.02)
    state[key + ".smooth_scale"] = smooth
    state["ups.0.0.bias"] = torch.randn(24, generator=g) * 0.1
    roles["vocoder.stages.0.ups.0"] = {"precision": "int8", "state_key": key, "input_scale": 0.02,
                                       "weight_scale": scale.tolist(), "smooth_scale": smooth.tolist(),
                                       "weight_axis": 1, "weight_input_axis": 0}
    meta = {"component": "cfm", "scheme": "mixed", "roles": roles}
    return state, meta


CONV_GEOMETRY = {"vocoder.conv_pre": {"stride": 1, "padding": 3, "dilation": 1},
                 "vocoder.stages.0.ups.0": {"stride": 4, "padding": 2, "dilation": 1, "transposed": True}}


def test_artifact_validation_rules():
    from inspark_proper_format_b200.manifest import check_artifact
    ok = {"schema": 1, "scheme": "fp8", "role_specs": {"a": {"precision": "fp8", "input_scale": 0.1,
                                                               "weight_scale": [0.1, 0.2]}}}
    assert check_artifact(ok, "fp8") is ok
    with pytest.raises(ValueError):
        check_artifact(dict(ok, schema=2))
    with pytest.raises(ValueError):
        check_artifact(ok, "int8")
    bad = json.loads(json.dumps(ok)); bad["role_specs"]["a"]["weight_scale"] = [0.1, -1.0]
    with pytest.raises(ValueError):
        check_artifact(bad)
    bad = json.loads(json.dumps(ok)); bad["role_specs"]["a"].update(precision="int8", smooth_scale=[])
    with pytest.raises(ValueError):
        check_artifact(bad)
    bad = {"schema": 1, "scheme": "nvfp4", "role_specs": {"b": {"precision": "nvfp4", "activation_amax": 1.0,
                                                                "block_size": 32}}}
    with pytest.raises(ValueError):
        check_artifact(bad)


def test_safetensors_round_trip_and_role_mapping_cpu():
    from safetensors.torch import load, save
    state, meta = synthetic_export()
    restored = load(save(state))
    assert set(restored) == set(state)
    for k, v in state.items():
        assert torch.equal(restored[k].reshape(-1).view(torch.uint8), v.reshape(-1).view(torch.uint8)), k
    # role metadata the loader needs is all present
    for role, spec in meta["roles"].items():
        assert spec["state_key"] in restored


@pytest.mark.gpu
def test_exported_roles_run_on_the_kernels():
    from safetensors.torch import save
    from inspark_proper_format_b200.manifest import load_component_bytes
    state, meta = synthetic_export(1)
    roles, skipped = load_component_bytes(save(state), meta)
    assert set(skipped) == {"vocoder.conv_pre", "vocoder.stages.0.ups.0"}     # no geometry given
    x = torch.randn(96, 256, generator=torch.Generator().manual_seed(2))
    xf = x.numpy()
    # fp8: static E4M3 Q then acc * input_scale * weight_scale + bias
    k = "transformer.layers.0.w1.weight"
    y = roles["cfm.blocks.0.w1"](x.cuda(), out_dtype=torch.float32).cpu().numpy()
    a = onq.quant_e4m3_static(xf, np.float32(0.0123))
    ref = og.fp8_gemm(a, state[k].view(torch.uint8).numpy(), np.float32(0.0123), state[k + ".weight_scale"].numpy(),
                      state[k[:-7] + ".bias"].numpy(), out="f32")
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5
    # int8: SmoothQuant Q then the i8 epilogue
    k = "layers.0.qkv.weight"
    y = roles["target.blocks.0.qkv"](x.cuda(), out_dtype=torch.float32).cpu().numpy()
    qa = onq.quant_int8_static(xf, np.float32(0.0123), state[k + ".smooth_scale"].numpy())
    ref = og.int8_gemm(qa, state[k].numpy(), np.float32(0.0123), state[k + ".weight_scale"].numpy(),
                       state[k[:-7] + ".bias"].numpy())
    np.testing.assert_array_equal(y, ref)
    # nvfp4
    k = "transformer.layers.0.w2.weight"
    y = roles["cfm.blocks.0.w2"](x.cuda(), out_dtype=torch.float32).cpu().numpy()
    gx = float(state[k + ".activation_global_scale"])
    ap, asc = onq.quant_nvfp4(xf, gx)
    ref = ofp4.nvfp4_gemm(ap, asc, gx, state[k].numpy(), state[k + ".block_scale"].view(torch.uint8).numpy(),
                          float(state[k + ".global_scale"]))
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5
    # bf16 protected role
    y = roles["cfm.proj"](x.cuda(), out_dtype=torch.float32).cpu()
    ref = torch.nn.functional.linear(x.bfloat16(), state["proj.weight"]).float()
    assert torch.allclose(y, ref, rtol=1e-2, atol=1e-3)


@pytest.mark.gpu
def test_exported_conv_roles_run_on_the_conv_kernels():
    """fp8 Conv1d and INT8 SmoothQuant ConvTranspose1d roles with the caller's geometry:
    static input Q (INT8: divided by the smoothing factors), exact code sums, then
    ``acc * input_scale * weight_scale[co] + bias`` (``ExportWeightOp`` conv roles)."""
    from safetensors.torch import save
    from inspark_proper_format_b200.manifest import load_component_bytes
    from oracle import conv as oconv
    state, meta = synthetic_export(3)
    roles, skipped = load_component_bytes(save(state), meta, conv_geometry=CONV_GEOMETRY)
    assert not skipped
    g = torch.Generator().manual_seed(4)
    for role, key, ci, fmt in (("vocoder.conv_pre", "conv_pre.weight", 32, "e4m3"),
                               ("vocoder.stages.0.ups.0", "ups.0.0.weight", 32, "int8")):
        geo = CONV_GEOMETRY[role]
        tr = geo.get("transposed", False)
        x = torch.randn(2, ci, 48, generator=g) * 2
        y = roles[role](x.cuda(), out_dtype=torch.float32).cpu().numpy()
        s_in = np.float32(state[key + ".input_scale"])
        smooth = state.get(key + ".smooth_scale")
        xq = oconv.quantize_input(x.numpy(), s_in, fmt, None if smooth is None else smooth.numpy())
        codes = state[key]
        codes = codes.view(torch.uint8) if fmt == "e4m3" else codes
        wq = codes.permute(1, 0, 2).numpy() if tr else codes.numpy()              # [CO, CI, KW]
        kw = wq.shape[-1]
        t_out = oconv.conv_out_length(48, kw, geo["stride"], geo["padding"], geo["dilation"], tr)
        acc = oconv.gather_conv_codes(xq, wq, fmt, stride=geo["stride"], padding=geo["padding"],
                                      dilation=geo["dilation"], transpose=tr, t_out=t_out).astype(np.float32)
        ref = ((acc * s_in).astype(np.float32) * state[key + ".weight_scale"].numpy()[None, :, None]).astype(np.float32)
        ref = (ref + state[key[:-7] + ".bias"].numpy()[None, :, None]).astype(np.float32)
        assert y.shape == ref.shape
        assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5, role
