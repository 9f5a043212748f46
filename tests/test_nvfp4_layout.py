"""CPU checks of the NVFP4 tensor-core scale layout and the gate/up stacking
(host-side index arithmetic; no GPU)."""
import numpy as np
import torch

from oracle import nvfp4 as ofp4


def test_sf_layout_round_trip_and_padding():
    rng = np.random.default_rng(0)
    for r, kb in [(1, 4), (127, 32), (128, 8), (300, 128)]:
        sf = rng.integers(0, 256, (r, kb), dtype=np.uint8)
        tiled = ofp4.sf_to_mma_layout(sf)
        assert tiled.size == (r + 127) // 128 * 128 * kb
        np.testing.assert_array_equal(ofp4.sf_from_mma_layout(tiled, r, kb), sf)
        covered = np.zeros(tiled.size, bool)
        rows = np.arange(r)[:, None]
        ks = np.arange(kb)[None, :]
        covered[((rows // 128) * (kb // 4) + ks // 4) * 512 + (rows % 32) * 16 + ((rows % 128) // 32) * 4
                + ks % 4] = True
        assert covered.sum() == r * kb                   # a bijection onto the real rows
        assert not tiled[~covered].any()                 # padding rows are zero


def test_sf_layout_known_positions():
    sf = np.zeros((256, 8), np.uint8)
    sf[0, 0], sf[33, 1], sf[127, 5], sf[130, 7] = 1, 2, 3, 4
    t = ofp4.sf_to_mma_layout(sf)
    assert t[0] == 1                                     # row 0, block 0
    assert t[1 * 16 + 1 * 4 + 1] == 2                    # row 33: lane 1, quarter 1, block 1
    assert t[512 + 31 * 16 + 3 * 4 + 1] == 3             # row 127, block 5: second K chunk
    assert t[(1 * 2 + 1) * 512 + 2 * 16 + 0 * 4 + 3] == 4  # row 130 (second row block), block 7


def test_stack_gate_up_rows():
    from inspark_proper_format_b200.nvfp4 import stack_gate_up
    w1 = torch.arange(128 * 3).reshape(128, 3)
    w3 = -torch.arange(128 * 3).reshape(128, 3) - 1
    s = stack_gate_up(w1, w3)
    assert s.shape == (256, 3)
    assert torch.equal(s[0:64], w1[0:64]) and torch.equal(s[64:128], w3[0:64])
    assert torch.equal(s[128:192], w1[64:128]) and torch.equal(s[192:256], w3[64:128])
