"""CPU tests of the Python surface that need no kernel: public names, module
construction, from_conv2d, surgery eligibility, and loud failure without a GPU."""

import pytest
import torch
import torch.nn as nn

import nova_winograd
from nova_winograd import (NovaWinogradConv2d, NovaWinogradConv2dCompilable,
                           NovaWinogradConv2dTrainable, replace_conv2d_with_nova)


def test_public_names_match_reference():
    # nova_winograd/__init__.py:29-36 of the reference.
    assert set(nova_winograd.__all__) == {
        "NovaWinogradConv2d", "NovaWinogradConv2dTrainable", "NovaWinogradConv2dCompilable",
        "nova_forward", "compute_tiling", "replace_conv2d_with_nova"}


def test_module_state_dict_interchangeable_with_conv2d():
    conv = nn.Conv2d(16, 32, 3, padding=1, bias=True)
    nova = NovaWinogradConv2d.from_conv2d(conv)
    assert set(nova.state_dict()) == set(conv.state_dict()) == {"weight", "bias"}
    assert torch.equal(nova.weight, conv.weight) and torch.equal(nova.bias, conv.bias)
    assert nova.weight.dtype == torch.float32
    assert "F(6,3)" in repr(nova)


def test_from_conv2d_rejects_ineligible():
    with pytest.raises(ValueError):
        NovaWinogradConv2d.from_conv2d(nn.Conv2d(4, 4, 3, stride=2))
    with pytest.raises(ValueError):
        NovaWinogradConv2d.from_conv2d(nn.Conv2d(4, 4, 5))
    with pytest.raises(ValueError):
        NovaWinogradConv2d(4, 4, kernel_size=5)


def test_replace_conv2d_counts_like_reference():
    # tests/test_correctness.py:168-184 of the reference: 2 of 4 replaced.
    model = nn.Sequential(
        nn.Conv2d(3, 64, 3, padding=1, bias=False), nn.ReLU(),
        nn.Conv2d(64, 128, 3, stride=2, padding=1), nn.ReLU(),
        nn.Conv2d(128, 128, 3, padding=1, bias=True), nn.ReLU(),
        nn.Conv2d(128, 256, 1))
    assert replace_conv2d_with_nova(model, verbose=False) == 2
    assert isinstance(model[0], NovaWinogradConv2d)
    assert not isinstance(model[2], NovaWinogradConv2d)
    assert isinstance(model[4], NovaWinogradConv2d)
    assert replace_conv2d_with_nova(model, verbose=False) == 0  # idempotent


def test_replace_trainable_and_skip_dilated_grouped():
    model = nn.Sequential(nn.Conv2d(8, 8, 3, padding=1), nn.Conv2d(8, 8, 3, padding=2, dilation=2),
                          nn.Conv2d(8, 8, 3, padding=1, groups=2))
    assert replace_conv2d_with_nova(model, trainable=True, verbose=False) == 1
    assert isinstance(model[0], NovaWinogradConv2dTrainable)


def test_resnet50_has_13_eligible_convs():
    torchvision = pytest.importorskip("torchvision")
    model = torchvision.models.resnet50()
    assert replace_conv2d_with_nova(model, verbose=False) == 13  # docs/report/main.tex:185


def test_compilable_fake_kernel_shapes():
    conv = NovaWinogradConv2dCompilable(8, 16, padding=1)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(2, 8, 10, 12, dtype=torch.float16)
        y = torch.ops.nova.winograd_conv2d(x, torch.empty(16, 8, 3, 3), 1)
        assert tuple(y.shape) == (2, 16, 10, 12) and y.dtype == torch.float16


def test_forward_without_gpu_fails_loudly():
    if torch.cuda.is_available():
        pytest.skip("GPU visible")
    conv = NovaWinogradConv2d(8, 8)
    with pytest.raises(RuntimeError, match="CUDA device"):
        conv(torch.zeros(1, 8, 8, 8, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="CUDA device"):
        nova_winograd.compute_tiling(56, 56, 1)


def test_nhwc_eligibility_rule():
    """Channels-last inputs take the NHWC kernels only when C % 8 == 0, K is
    even and the base is 16-byte aligned; plain-contiguous tensors (including
    those that are both, C == 1 or H == W == 1) keep the NCHW path."""
    import torch
    from nova_winograd.ops import nhwc_eligible
    cl = torch.channels_last
    x = torch.zeros(2, 16, 9, 9, dtype=torch.float16).contiguous(memory_format=cl)
    assert nhwc_eligible(x, 16)
    assert not nhwc_eligible(x, 15)                       # odd K
    assert not nhwc_eligible(torch.zeros(2, 12, 9, 9, dtype=torch.float16)
                             .contiguous(memory_format=cl), 16)  # C % 8 != 0
    assert not nhwc_eligible(torch.zeros(2, 16, 9, 9, dtype=torch.float16), 16)  # NCHW
    both = torch.zeros(2, 16, 1, 1, dtype=torch.float16)  # contiguous in both formats
    assert not nhwc_eligible(both, 16)
    base = torch.zeros(2 * 16 * 9 * 9 + 1, dtype=torch.float16)
    off = base[1:].view(2, 9, 9, 16).permute(0, 3, 1, 2)  # channels-last view, 2-byte offset
    assert off.is_contiguous(memory_format=cl) and not nhwc_eligible(off, 16)
