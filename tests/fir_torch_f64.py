"""BigVGAN ``Activation1d(Snake)`` restated in float64 torch for the full-size FIR
parity test, which runs it on the device (the oracle's numpy loops are too slow
for a whole B64 x C512 x T16384 micro-batch) — test infrastructure only.

Same operators as the reference module
(``models/indextts2/upstream/s2mel/modules/bigvgan/alias_free_activation/torch/``):
``UpSample1d(2, 12)`` = replicate-pad 5, ``2 * conv_transpose1d(stride 2, groups C)``,
crop 15/15 (``resample.py:9-27``); Snake ``x + inv_beta * sin(alpha x)^2``
(``bigvgan/activations.py:48-54``); ``DownSample1d(2, 12)`` = replicate-pad (5, 6),
``conv1d(stride 2, groups C)`` (``filter.py:44-70``, ``resample.py:30-39``).
Pinned against the reference's own outputs (``golden/fir.npz``) by
``test_oracle_golden.test_fir_torch_f64_matches_activation1d``.
"""
import torch
import torch.nn.functional as F


def activation1d_f64(x, filt, alpha, inv_beta):
    """x [B, C, T]; filt [12] (both filters of BigVGAN are the same Kaiser sinc);
    alpha, inv_beta [C] (linear).  Returns float64 [B, C, T] on x's device."""
    x = x.double()
    c = x.shape[1]
    f = filt.double().reshape(1, 1, -1).expand(c, 1, -1)
    u = F.pad(x, (5, 5), mode="replicate")
    u = 2.0 * F.conv_transpose1d(u, f, stride=2, groups=c)[..., 15:-15]
    a = alpha.double().reshape(1, -1, 1)
    u = u + inv_beta.double().reshape(1, -1, 1) * torch.sin(u * a) ** 2
    u = F.pad(u, (5, 6), mode="replicate")
    return F.conv1d(u, f, stride=2, groups=c)
