"""Parity at the configurations the benchmark times.

The synthetic layers are built by the same code and seeds as ``bench.py``, so
these are the timed inputs themselves.  Full batches run on the GPU; sampled
images (the first two and the last two) are checked against the CPU oracle,
by the bars of ``tests/test_gpu_parity.py``: rel L2 <= 1e-2 against the
oracle's reference-precision math, error against an FP64 direct convolution
<= 1.1x the oracle's, no NaN/Inf.

* config 2: every ResNet-50 3x3 layer at batch 1, 8, 32 and 128 (the
  reference's grid, ``benchmarks/bench_layers.py:38-49``), plus batch 256 for
  conv2_x and conv5_x (the north star's GEMM-stage batch);
* config 3: ResNet-50 with its 13 eligible convs replaced; every replaced
  conv's output for one image, from the activations the model feeds it;
* configs 4/5: one UNet ResBlock with a concatenated skip (C != K) and one
  with C == K at UNet channel counts, replaced, per conv.
"""

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402
import nova_oracle as o  # noqa: E402
from nova_winograd import NovaWinogradConv2d, replace_conv2d_with_nova  # noqa: E402

pytestmark = pytest.mark.gpu

GRID = [(name, B) for name, _, _ in bench.LAYERS for B in (1, 8, 32, 128)]
GRID += [("conv2_x", 256), ("conv5_x", 256)]


@pytest.mark.parametrize("layer,B", GRID, ids=[f"{n}_B{b}" for n, b in GRID])
def test_timed_layer_parity(layer, B):
    shape = [l for l in bench.LAYERS if l[0] == layer]
    (name, C, H, conv, x), = bench.build_layers(B, torch.device("cuda"), shape)
    with torch.no_grad():
        y = conv(x)
    torch.cuda.synchronize()
    r = bench.sample_parity(name, x, conv.weight, y)
    assert r["ok"], r


def module_parity(mod, xin, yout):
    """One replaced conv: output (bias included, added in FP16 as the module
    does) against the oracle plus the same bias, for the images given."""
    x = xin.cpu().numpy()
    w = mod.weight.detach().float().cpu().numpy()
    y = yout.float().cpu().numpy()
    y_o = o.nova_forward(x, w, mod.padding, "ref")
    d = o.direct_conv_fp64(x, w, mod.padding)
    if mod.bias is not None:
        b16 = mod.bias.detach().half().cpu().view(1, -1, 1, 1)
        y_o = (torch.from_numpy(y_o) + b16).numpy()
        d = d + b16.double().numpy()
    assert np.isfinite(y).all()
    par, err, err_o = o.rel_l2(y, y_o), o.rel_l2(y, d), o.rel_l2(y_o, d)
    assert par <= bench.PARITY_TOL, (mod, par)
    assert err <= bench.ACCURACY_FACTOR * err_o, (mod, err, err_o)
    return par


def capture(model, run):
    """(module, input, output) of every NovaWinogradConv2d during run()."""
    seen = []
    hooks = [m.register_forward_hook(lambda m, i, out: seen.append((m, i[0][:1].clone(),
                                                                    out[:1].clone())))
             for m in model.modules() if isinstance(m, NovaWinogradConv2d)]
    try:
        with torch.no_grad():
            run()
    finally:
        for h in hooks:
            h.remove()
    return seen


def test_resnet50_replaced_convs_parity():
    torchvision = pytest.importorskip("torchvision")
    torch.manual_seed(1234)
    model = torchvision.models.resnet50().cuda().half().eval()
    ref = torchvision.models.resnet50().cuda().half().eval()
    ref.load_state_dict(model.state_dict())
    assert replace_conv2d_with_nova(model, verbose=False) == 13
    x = torch.randn(2, 3, 224, 224, device="cuda", dtype=torch.float16)
    seen = capture(model, lambda: model(x))
    assert len(seen) == 13
    worst = max(module_parity(m, xi, yi) for m, xi, yi in seen)
    assert worst <= bench.PARITY_TOL
    with torch.no_grad():
        out, out_ref = model(x), ref(x)
    assert torch.isfinite(out).all()
    rel = ((out.float() - out_ref.float()).norm() / out_ref.float().norm()).item()
    assert rel < 0.1, rel  # the whole network against cuDNN (FP16 drift over 13 convs)


@pytest.mark.parametrize("cin,cout,hw", [(960, 320, 32), (640, 640, 16), (2560, 1280, 8)])
def test_unet_resblock_replaced_convs_parity(cin, cout, hw):
    import unet_callers as U
    torch.manual_seed(cin + cout)
    blk = U.ResBlock(cin, cout, 1280, 32).cuda().half().eval()
    assert replace_conv2d_with_nova(blk, verbose=False) == 2
    x = torch.randn(2, cin, hw, hw, device="cuda", dtype=torch.float16)
    temb = torch.randn(2, 1280, device="cuda", dtype=torch.float16)
    seen = capture(blk, lambda: blk(x, temb))
    assert len(seen) == 2
    for m, xi, yi in seen:
        module_parity(m, xi, yi)
