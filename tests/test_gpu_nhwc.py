"""Channels-last (NHWC) path against the NCHW path and the oracle, stage by stage.

The NHWC input transform lands each block's tile windows with one TMA box load
of the [B][H][W][C] tensor and writes V in the NCHW path's layout; the NHWC
output transform reads M in that layout and writes [B][H_out][W_out][K].  The
NCHW path has several kernels per stage whose FP32 sums run in different orders,
so stage outputs are compared by the bar the library-against-reference pins
use (``tests/test_gpu_ref_pin.py``): |a - b| <= 1 FP16 ulp + 2 * terms * 2^-24 *
(sum of the terms' magnitudes), with at least 99.9 % of the values equal.  Whole
forwards: rel L2 against the NCHW forward <= 1e-3, and the parity bars against
the CPU oracle (rel L2 <= 1e-2, error against FP64 <= 1.1x the oracle's).
"""

import ctypes
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import nova_oracle as o  # noqa: E402
from nova_winograd import NovaWinogradConv2d, NovaWinogradConv2dTrainable, ops  # noqa: E402

pytestmark = pytest.mark.gpu

# (B, C, K, H, W, pad): the ResNet-50 3x3 layers, ragged and odd sizes, pad 0,
# C not a multiple of 64, C != K, a UNet width.
SHAPES = [
    (2, 64, 64, 56, 56, 1),
    (2, 128, 128, 28, 28, 1),
    (2, 256, 256, 14, 14, 1),
    (3, 512, 512, 7, 7, 1),
    (1, 64, 64, 13, 13, 1),
    (2, 32, 48, 20, 17, 1),
    (2, 8, 16, 9, 11, 0),
    (1, 24, 40, 5, 5, 1),
    (1, 320, 320, 16, 16, 1),
    (4, 16, 16, 3, 3, 1),
]


def _ids(shapes):
    return ["B{}_C{}_K{}_{}x{}_p{}".format(*s) for s in shapes]


def _tiles(H, W, pad):
    nh, nw, _, _ = ops.compute_tiling(H, W, pad)
    return nh, nw


def _assert_close_stage(got, want, scale, what):
    a = got.cpu().numpy()
    b = want.cpu().numpy()
    ok = o.within_fp32_reordering(a, b, scale, 16)
    assert ok.all(), f"{what}: {(~ok).sum()} of {ok.size} outside FP32 reordering"
    same = (a.astype(np.float32) == b.astype(np.float32)).mean()
    assert same >= 0.999, f"{what}: only {same:.5f} of the values equal"


def _assert_close_forward(y, y_ref):
    a, b = y.float(), y_ref.float()
    assert torch.isfinite(a).all()
    rel = ((a - b).norm() / b.norm()).item()
    assert rel <= 1e-3, rel


def _stage_v(x_nchw, C, H, W, pad, nhwc):
    lib = ops.get_lib()
    B = x_nchw.shape[0]
    nh, nw, _, _ = ops.compute_tiling(H, W, pad)
    BP = B * nh * nw
    V = torch.full((64, BP, C), float("nan"), dtype=torch.float16, device="cuda")
    s = ops.stream_ptr()
    if nhwc:
        x = x_nchw.contiguous(memory_format=torch.channels_last)
        ops.check(lib.nova_input_transform_nhwc_v2(ops.ptr(x), ops.ptr(V), B, C, H, W, pad, nh,
                                                   nw, BP, s), "input_transform_nhwc")
    else:
        ops.check(lib.nova_input_transform_v2(ops.ptr(x_nchw), ops.ptr(V), B, C, H, W, pad, nh,
                                              nw, BP, s), "input_transform")
    torch.cuda.synchronize()
    return V


@pytest.mark.parametrize("B,C,K,H,W,pad", SHAPES, ids=_ids(SHAPES))
def test_nhwc_input_transform_equals_nchw(B, C, K, H, W, pad):
    torch.manual_seed(B * 1000 + C + H)
    x = torch.randn(B, C, H, W, device="cuda", dtype=torch.float16)
    v_ref = _stage_v(x, C, H, W, pad, nhwc=False)
    v = _stage_v(x, C, H, W, pad, nhwc=True)
    assert torch.isfinite(v).all()
    _assert_close_stage(v, v_ref, o.input_transform_scale(x.cpu().numpy(), *_tiles(H, W, pad), pad),
                        "V")


@pytest.mark.parametrize("B,C,K,H,W,pad", SHAPES, ids=_ids(SHAPES))
def test_nhwc_forward_equals_nchw(B, C, K, H, W, pad):
    torch.manual_seed(7 * B + C + K)
    conv = NovaWinogradConv2d(C, K, padding=pad, bias=True).cuda()
    with torch.no_grad():
        conv.bias.normal_()
    x = torch.randn(B, C, H, W, device="cuda", dtype=torch.float16)
    xl = x.contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        y_ref = conv(x)
        y = conv(xl)
        y2 = conv(xl)  # the cached fast path
    assert y.is_contiguous(memory_format=torch.channels_last)
    _assert_close_forward(y, y_ref)
    assert torch.equal(y2, y)  # the same kernels again: identical
    # Alternating layouts on one module keeps each call's own layout.
    with torch.no_grad():
        y3 = conv(x)
    assert y3.is_contiguous() and torch.equal(y3, y_ref)


def test_nhwc_stage_output_transform_equals_nchw():
    """M from one NCHW forward's GEMM, transformed by both output kernels."""
    torch.manual_seed(11)
    B, C, K, H, W, pad = 2, 64, 96, 20, 23, 1
    conv = NovaWinogradConv2d(C, K, padding=pad).cuda()
    x = torch.randn(B, C, H, W, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        conv(x)
    lib = ops.get_lib()
    nh, nw, Ho, Wo = ops.compute_tiling(H, W, pad)
    BP = B * nh * nw
    V = _stage_v(x, C, H, W, pad, nhwc=False)
    M = torch.empty(64, BP, K, dtype=torch.float16, device="cuda")
    s = ops.stream_ptr()
    ops.check(lib.nova_batched_gemm_v2(conv._handle, ops.ptr(V), ops.ptr(M), BP, s), "gemm")
    y_ref = torch.empty(B, K, Ho, Wo, dtype=torch.float16, device="cuda")
    y = torch.empty(B, K, Ho, Wo, dtype=torch.float16, device="cuda",
                    memory_format=torch.channels_last)
    ops.check(lib.nova_output_transform_v2(ops.ptr(M), ops.ptr(y_ref), B, K, Ho, Wo, nh, nw, BP,
                                           s), "output_transform")
    ops.check(lib.nova_output_transform_nhwc_v2(ops.ptr(M), ops.ptr(y), B, K, Ho, Wo, nh, nw, BP,
                                                s), "output_transform_nhwc")
    torch.cuda.synchronize()
    scale = o.output_transform_scale(M.cpu().numpy(), B, nh, nw, Ho, Wo)
    _assert_close_stage(y.contiguous(), y_ref, scale, "y")


def test_nhwc_forward_matches_oracle():
    B, C, K, H, W, pad = 2, 64, 64, 14, 14, 1
    x, w = o.synthetic_case(B, C, K, H, W, seed=21)
    xt = torch.from_numpy(x).cuda().contiguous(memory_format=torch.channels_last)
    wt = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    y = ops.nova_forward(xt, wt, pad)
    assert y.is_contiguous(memory_format=torch.channels_last)
    y = y.float().cpu().numpy()
    y_o = o.nova_forward(x, w, pad, "ref")
    d = o.direct_conv_fp64(x, w, pad)
    assert np.isfinite(y).all()
    assert o.rel_l2(y, y_o) <= 1e-2
    assert o.rel_l2(y, d) <= 1.1 * o.rel_l2(y_o, d)


def test_nhwc_ineligible_shapes_fall_back_to_nchw():
    """C % 8 != 0 (no TMA box) or odd K: channels-last in, channels-last out,
    through an on-device copy to NCHW."""
    torch.manual_seed(3)
    for C, K in ((6, 8), (8, 7)):
        conv = NovaWinogradConv2d(C, K).cuda()
        x = torch.randn(2, C, 12, 12, device="cuda", dtype=torch.float16)
        with torch.no_grad():
            y_ref = conv(x)
            y = conv(x.contiguous(memory_format=torch.channels_last))
        assert y.is_contiguous(memory_format=torch.channels_last)
        assert torch.equal(y.contiguous(), y_ref)  # the NCHW kernels on a copy


def test_nhwc_entry_points_refuse_bad_arguments():
    lib = ops.get_lib()
    x = torch.zeros(1, 12, 8, 8, device="cuda", dtype=torch.float16).contiguous(
        memory_format=torch.channels_last)
    V = torch.empty(64, 4, 12, device="cuda", dtype=torch.float16)
    s = ops.stream_ptr()
    # C % 8 != 0
    assert lib.nova_input_transform_nhwc_v2(ops.ptr(x), ops.ptr(V), 1, 12, 8, 8, 1, 2, 2, 4, s) != 0
    # odd K
    y = torch.empty(1, 8, 8, 7, device="cuda", dtype=torch.float16)
    assert lib.nova_output_transform_nhwc_v2(ops.ptr(V), ops.ptr(y), 1, 7, 8, 8, 2, 2, 4, s) != 0
    # the forward on a handle with odd K
    h = ops.create_handle(torch.device("cuda"))
    try:
        w = torch.randn(7, 8, 3, 3, device="cuda")
        ops.check(lib.nova_set_weights_v2(h, ops.ptr(w), 7, 8, s), "set_weights")
        x8 = torch.zeros(1, 8, 8, 8, device="cuda", dtype=torch.float16).contiguous(
            memory_format=torch.channels_last)
        assert lib.nova_forward_nhwc_v2(h, ops.ptr(x8), ops.ptr(y), 1, 8, 8, 1, s) != 0
    finally:
        lib.nova_destroy(h)
    torch.cuda.synchronize()


def test_nhwc_trainable_backward():
    torch.manual_seed(5)
    conv = NovaWinogradConv2dTrainable(32, 32).cuda()
    x = torch.randn(2, 32, 12, 12, device="cuda", dtype=torch.float16)
    xl = x.contiguous(memory_format=torch.channels_last).requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    y = conv(xl)
    y_ref = conv(xr)
    assert y.is_contiguous(memory_format=torch.channels_last)
    _assert_close_forward(y, y_ref)
    g = torch.randn_like(y_ref)
    y.backward(g)
    gw = conv.weight.grad.clone()
    conv.weight.grad = None
    y_ref.backward(g)
    assert torch.allclose(xl.grad.float(), xr.grad.float(), rtol=1e-3, atol=1e-3)
    assert torch.allclose(gw, conv.weight.grad, rtol=1e-3, atol=1e-3)
