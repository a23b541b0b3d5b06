"""The UNet callers of configs 4 and 5 (unet_callers.py): layout checks on CPU.

The eligible-conv counts are the ones the configs name (49 for SD 1.5, 38 for
SDXL), and the parameter counts are those of the published UNets (0.86 B and
2.57 B).  Built on the meta device, so no weights are allocated.
"""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "nova-wino-amd_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import unet_callers as U  # noqa: E402
from nova_winograd.surgery import is_eligible  # noqa: E402


@pytest.mark.parametrize("spec,n_eligible,params_b", [(U.SD15, 49, 0.860), (U.SDXL, 38, 2.567)])
def test_layout_counts(spec, n_eligible, params_b):
    with torch.device("meta"):
        m = U.UNet(spec)
    assert sum(1 for mod in m.modules() if is_eligible(mod)) == n_eligible
    n = sum(p.numel() for p in m.parameters())
    assert abs(n / 1e9 - params_b) < 0.002


def test_eligible_conv_channels():
    # The replaced convs carry the 320 / 640 / 1280 channel counts (plus the
    # 4-channel conv_in / conv_out, which take the SIMT GEMM path).
    with torch.device("meta"):
        m = U.UNet(U.SD15)
    chans = {(mod.in_channels, mod.out_channels) for mod in m.modules() if is_eligible(mod)}
    assert (4, 320) in chans and (320, 4) in chans
    assert {(320, 320), (640, 640), (1280, 1280)} <= chans


@pytest.mark.parametrize("xl", [False, True])
def test_tiny_forward_shapes(xl):
    if xl:
        spec = U.UNetSpec(channels=(32, 64, 64), attn_depth=(0, 1, 2), mid_depth=2,
                          context_dim=24, head_dim=16, linear_proj=True, add_embed=True,
                          groups=8, pooled_dim=20, add_time_dim=8)
    else:
        spec = U.UNetSpec(channels=(32, 64), attn_depth=(1, 1), mid_depth=1, context_dim=16,
                          heads=4, groups=8)
    torch.manual_seed(0)
    m = U.UNet(spec).eval()
    x, t, ctx, extra = U.make_inputs(spec, 2, 16, "cpu", torch.float32, seed=3)
    with torch.no_grad():
        y = m(x, t, ctx, **extra)
    assert y.shape == x.shape and torch.isfinite(y).all()


def test_sinusoid_layout():
    e = U.sinusoid(torch.tensor([0.0, 1.0]), 8)
    assert e.shape == (2, 8)
    assert torch.allclose(e[0], torch.tensor([1.0] * 4 + [0.0] * 4))
    assert torch.isclose(e[1, 0], torch.cos(torch.tensor(1.0)))
