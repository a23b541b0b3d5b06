"""GPU parity tests: the CUDA path (through the C ABI) against the CPU oracle.

Bars (floating point, FP16 storage as in the reference):
  * rel L2 (CUDA vs oracle "ref" mode) <= PARITY_TOL = 1e-2 -- same algorithm,
    same FP16 roundings; only the FP32 summation order differs (tensor-core
    accumulation vs BLAS), which moves a small fraction of the FP16 roundings of
    V, M and y by one ulp.  Measured: ~2e-3 at config 1.  The bar sits 5x below
    the algorithm's own FP16 error (~5 %) and 3x below the cost of a single
    FP16 rounding stage (~3 %), so a real defect (a wrong constant, a dropped
    tile, a layout slip) cannot hide under it.
  * rel L2 (CUDA vs FP64 direct conv) <= 1.1 x rel L2 (oracle "ref" vs FP64) --
    the accuracy bar of the north star.
  * stage kernels (input / output / filter transforms) within 1 FP16 ulp of
    the oracle on >= 99.9 % of elements.
"""

import ctypes

import numpy as np
import pytest
import torch

import nova_oracle as o
from nova_winograd import ops

pytestmark = pytest.mark.gpu

PARITY_TOL = 1e-2
ACCURACY_FACTOR = 1.1


def lib():
    return ops.get_lib()


def to_dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def run_forward(x, w, pad, path=0, workspace="caller"):
    """Forward through the C ABI on explicit tensors; returns (y numpy fp16, path ran)."""
    L = lib()
    B, C, H, W = x.shape
    K = w.shape[0]
    xd, wd = to_dev(x, torch.float16), to_dev(w, torch.float32)
    nh, nw, Ho, Wo = ops.compute_tiling(H, W, pad)
    y = torch.full((B, K, Ho, Wo), float("nan"), dtype=torch.float16, device="cuda")
    h = ops.create_handle()
    try:
        s = ops.stream_ptr()
        ops.check(L.nova_set_weights_v2(h, ops.ptr(wd), K, C, s), "set_weights")
        ops.check(L.nova_set_path(h, path), "set_path")
        if workspace == "caller":
            V = torch.empty(64 * C * B * nh * nw, dtype=torch.float16, device="cuda")
            M = torch.empty(64 * K * B * nh * nw, dtype=torch.float16, device="cuda")
            ops.check(L.nova_forward_workspace_v2(h, ops.ptr(xd), ops.ptr(y), ops.ptr(V),
                                                  ops.ptr(M), B, H, W, pad, nh, nw, s), "forward_ws")
        else:
            ops.check(L.nova_forward_v2(h, ops.ptr(xd), ops.ptr(y), B, H, W, pad, s), "forward")
        ops.check(L.nova_device_status(h), "device_status")
        ran = L.nova_get_path(h)
    finally:
        L.nova_destroy(h)
    return y.cpu().numpy(), ran


def check_parity(x, w, pad, y):
    y_ref = o.nova_forward(x, w, pad, "ref")
    assert y.shape == y_ref.shape
    assert np.isfinite(y.astype(np.float32)).all(), "NaN/Inf in output"
    d = o.direct_conv_fp64(x, w, pad)
    par = o.rel_l2(y, y_ref)
    err, err_ref = o.rel_l2(y, d), o.rel_l2(y_ref, d)
    assert par <= PARITY_TOL, f"parity rel L2 {par:.3e}"
    assert err <= ACCURACY_FACTOR * err_ref, f"accuracy {err:.4f} vs oracle {err_ref:.4f}"
    return par, err, err_ref


# BASELINE config 1 and the config-2 shapes at batch 1, plus shapes the
# reference suite uses (tests/test_correctness.py:38-106).
PARITY_CASES = [
    (1, 64, 64, 56, 56, 1),
    (1, 128, 128, 28, 28, 1),
    (1, 256, 256, 14, 14, 1),
    (1, 512, 512, 7, 7, 1),
    (2, 64, 64, 32, 32, 1),
    (2, 128, 256, 28, 28, 1),
    (1, 64, 128, 20, 17, 1),     # ragged tiles, C != K
    (3, 72, 48, 13, 11, 1),      # C not a multiple of 64, K = 48 (MMA N = 48)
    (1, 64, 320, 9, 9, 1),       # K = 320 -> two N = 160 tiles
    (1, 40, 32, 15, 15, 0),      # pad 0
    (1, 32, 32, 10, 10, 2),      # pad 2
    (1, 3, 64, 50, 50, 1),       # C = 3: SIMT GEMM path
    (2, 16, 4, 12, 12, 1),       # K = 4: SIMT GEMM path
    (1, 8, 16, 1, 1, 1),         # single pixel
    (3, 96, 80, 40, 40, 1),      # TMA paths with a partial last 64-channel group (x, V, y clipped)
    # SD 1.5 / SDXL UNet channel counts (configs 4 and 5) at small spatial sizes:
    (1, 320, 320, 32, 32, 1),    # GEMM N = 160 (non-TMA epilogue)
    (1, 640, 640, 16, 16, 1),    # N = 160, 4 column tiles
    (1, 1280, 1280, 8, 8, 1),    # N = 256, 5 column tiles
]


@pytest.mark.parametrize("B,C,K,H,W,pad", PARITY_CASES)
def test_forward_parity_auto(B, C, K, H, W, pad):
    x, w = o.synthetic_case(B, C, K, H, W, seed=1234 + B * 7 + C + K + H)
    y, ran = run_forward(x, w, pad)
    assert ran in expected_paths(C, K)
    check_parity(x, w, pad, y)


def fused_eligible(C, K):
    return 16 <= C <= 64 and C % 16 == 0 and 1 <= K <= 64


def expected_paths(C, K):
    """Paths the automatic dispatch may pick (the fused one only up to a tile count)."""
    tc = 1 if (C % 8 == 0 and K % 16 == 0) else 2
    return {tc, 3} if fused_eligible(C, K) else {tc}


# Fused single kernel (reference csrc/nova_winograd_fused.hip:283-440, K, C <= 64).
FUSED_CASES = [
    (1, 64, 64, 56, 56, 1),
    (3, 64, 64, 20, 17, 1),      # ragged tiles, last CTA partly past BP
    (2, 32, 16, 13, 11, 0),      # pad 0, odd W_out
    (1, 48, 40, 15, 15, 2),      # C = 48 (three MMA k-steps), K % 16 != 0, pad 2
    (1, 16, 64, 9, 9, 1),
    (4, 64, 8, 7, 7, 1),
    (1, 16, 1, 1, 1, 1),         # single pixel, single output channel
    (8, 64, 64, 56, 56, 1),      # 100 groups of 8 tiles: 2-CTA clusters
    (12, 32, 16, 64, 64, 1),     # 182 groups: one CTA per group
]


@pytest.mark.parametrize("B,C,K,H,W,pad", FUSED_CASES)
def test_fused_parity(B, C, K, H, W, pad):
    x, w = o.synthetic_case(B, C, K, H, W, seed=4321 + B + C + K + H + W)
    y, ran = run_forward(x, w, pad, path=3)
    assert ran == 3
    check_parity(x, w, pad, y)


def test_fused_matches_three_pass():
    # Same roundings (V, M to FP16) and the same MMA k-order: only the FP32
    # order inside the output transform differs.
    x, w = o.synthetic_case(2, 64, 64, 30, 30, seed=11)
    y3, r3 = run_forward(x, w, 1, path=3)
    y1, r1 = run_forward(x, w, 1, path=1)
    assert (r3, r1) == (3, 1)
    assert o.rel_l2(y3, y1) < 1e-3


def test_fused_refused_outside_its_shapes():
    L = lib()
    h = ops.create_handle()
    try:
        w = torch.randn(64, 128, 3, 3, device="cuda")
        ops.check(L.nova_set_weights_v2(h, ops.ptr(w), 64, 128, None), "set_weights")
        assert L.nova_set_path(h, 3) == 1
    finally:
        L.nova_destroy(h)


@pytest.mark.parametrize("B,C,K,H,pad", [(1, 64, 64, 28, 1), (2, 128, 64, 14, 1), (1, 64, 96, 9, 0)])
def test_tcgen05_and_simt_paths_agree(B, C, K, H, pad):
    x, w = o.synthetic_case(B, C, K, H, H, seed=99 + C)
    y_tc, r1 = run_forward(x, w, pad, path=1)
    y_simt, r2 = run_forward(x, w, pad, path=2)
    assert (r1, r2) == (1, 2)
    check_parity(x, w, pad, y_tc)
    check_parity(x, w, pad, y_simt)
    assert o.rel_l2(y_tc, y_simt) < PARITY_TOL


def test_internal_workspace_path_matches_caller_workspace():
    x, w = o.synthetic_case(2, 64, 64, 30, 30, seed=5)
    y1, _ = run_forward(x, w, 1, workspace="caller")
    y2, _ = run_forward(x, w, 1, workspace="internal")
    np.testing.assert_array_equal(y1, y2)


def test_batch_consistency_bit_exact():
    # Images are independent: a batch equals its images run one at a time.
    x, w = o.synthetic_case(5, 64, 128, 23, 23, seed=77)
    yb, _ = run_forward(x, w, 1)
    for b in range(5):
        yi, _ = run_forward(x[b:b + 1], w, 1)
        np.testing.assert_array_equal(yb[b:b + 1], yi)


def test_plane_launch_shapes_agree():
    # 14x14 images are 3x3 tiles.  At batch 40 with 256 channels, 160 blocks
    # of 64 channels take the throughput plane kernels (3-warp input
    # transform).  A single image takes the one-warp-per-tile kernels.  Same
    # arithmetic per tile, so the outputs are bit-identical.
    x, w = o.synthetic_case(40, 256, 256, 14, 14, seed=404)
    yb, _ = run_forward(x, w, 1, path=1)
    for b in (0, 17, 39):
        yi, _ = run_forward(x[b:b + 1], w, 1, path=1)
        np.testing.assert_array_equal(yb[b:b + 1], yi)
    check_parity(x[:2], w, 1, yb[:2])


def forward_in_child(x, w, pad, env_overrides):
    """The same C-ABI forward in a child process with extra environment switches."""
    import os
    import subprocess
    import sys
    import tempfile
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    with tempfile.TemporaryDirectory() as tmp:
        np.save(os.path.join(tmp, "x.npy"), x)
        np.save(os.path.join(tmp, "w.npy"), w)
        code = (
            "import sys, numpy as np\n"
            f"sys.path[:0] = [{os.path.join(root, 'nova-wino-amd_b200')!r}, {here!r}, "
            f"{os.path.join(root, 'oracle')!r}]\n"
            "from test_gpu_parity import run_forward\n"
            f"x = np.load({os.path.join(tmp, 'x.npy')!r}); w = np.load({os.path.join(tmp, 'w.npy')!r})\n"
            f"y, _ = run_forward(x, w, {pad})\n"
            f"np.save({os.path.join(tmp, 'y.npy')!r}, y)\n")
        env = dict(os.environ, **env_overrides)
        subprocess.run([sys.executable, "-c", code], check=True, env=env, timeout=600)
        return np.load(os.path.join(tmp, "y.npy"))


def test_programmatic_launch_off_matches_default():
    # The same forward in a child process with programmatic dependent launch
    # disabled (NOVA_PDL_MASK=0) writes the same bytes.
    x, w = o.synthetic_case(3, 64, 128, 30, 30, seed=505)
    y, _ = run_forward(x, w, 1)
    np.testing.assert_array_equal(y, forward_in_child(x, w, 1, {"NOVA_PDL_MASK": "0"}))


# Plane-mode shapes (images of at most 3x3 tiles) at batches that launch at
# least one block per SM, so the throughput plane kernels run: images of
# fewer than 9 tiles land by bulk copies of 64 channels; 3x3-tile images with
# even W load cell pairs with 4-byte loads, odd W keeps 2-byte loads.
PLANE_THROUGHPUT_CASES = [
    (80, 72, 64, 14, 14, 1),     # 3x3 tiles, last 64-channel group holds 8 channels
    (40, 264, 72, 7, 7, 1),      # 2x2 tiles, odd H*W, last C and K groups hold 8 channels
    (160, 64, 32, 12, 12, 0),    # pad 0: 10x10 output, 2x2 tiles
    (150, 16, 16, 4, 4, 1),      # 1x1 tile, 16 channels
    (160, 64, 32, 20, 20, 0),    # pad 0, 3x3 tiles over a full 20x20 input plane
    (150, 64, 64, 15, 15, 1),    # 3x3 tiles, odd W
]


@pytest.mark.parametrize("B,C,K,H,W,pad", PLANE_THROUGHPUT_CASES)
def test_plane_throughput_parity(B, C, K, H, W, pad):
    x, w = o.synthetic_case(B, C, K, H, W, seed=606 + B + C + H)
    y, _ = run_forward(x, w, pad)
    check_parity(x[:4], w, pad, y[:4])
    check_parity(x[-4:], w, pad, y[-4:])


def test_plane_input_loaders_agree():
    # The plane input loaders stage the same values: the outputs are
    # bit-identical.
    # Every loader (0: 2-byte lane loads, 2: cell pairs, 32/64: bulk copies)
    # against the default one for the shape.
    cases = PLANE_THROUGHPUT_CASES
    for (B, C, K, H, W, pad), env in ((cases[0], {"NOVA_PLANE_LAND": "0"}),
                                      (cases[0], {"NOVA_PLANE_LAND": "32"}),
                                      (cases[1], {"NOVA_PLANE_LAND": "0"}),
                                      (cases[2], {"NOVA_PLANE_LAND": "2"}),
                                      (cases[4], {"NOVA_PLANE_LAND": "0"})):
        x, w = o.synthetic_case(B, C, K, H, W, seed=707 + C)
        y, _ = run_forward(x, w, pad)
        np.testing.assert_array_equal(y, forward_in_child(x, w, pad, env))


def test_empty_batch_is_a_no_op():
    L = lib()
    w = torch.randn(16, 8, 3, 3, device="cuda")
    h = ops.create_handle()
    try:
        ops.check(L.nova_set_weights_v2(h, ops.ptr(w), 16, 8, None), "set_weights")
        assert L.nova_forward_workspace_v2(h, None, None, None, None, 0, 8, 8, 1, 2, 2, None) == 0
        assert L.nova_forward_v2(h, None, None, 0, 8, 8, 1, None) == 0
    finally:
        L.nova_destroy(h)


def test_guard_bands_untouched():
    x, w = o.synthetic_case(1, 64, 64, 17, 17, seed=3)
    L = lib()
    xd, wd = to_dev(x, torch.float16), to_dev(w, torch.float32)
    nh, nw, Ho, Wo = ops.compute_tiling(17, 17, 1)
    n_out = 64 * Ho * Wo
    guard = 4096
    buf = torch.full((n_out + 2 * guard,), 12345.0, dtype=torch.float16, device="cuda")
    V = torch.full((64 * 64 * nh * nw + 2 * guard,), 777.0, dtype=torch.float16, device="cuda")
    M = torch.full((64 * 64 * nh * nw + 2 * guard,), 777.0, dtype=torch.float16, device="cuda")
    h = ops.create_handle()
    try:
        ops.check(L.nova_set_weights_v2(h, ops.ptr(wd), 64, 64, None), "set_weights")
        yptr = ctypes.c_void_p(buf.data_ptr() + guard * 2)
        ops.check(L.nova_forward_workspace_v2(
            h, ops.ptr(xd), yptr, ctypes.c_void_p(V.data_ptr() + guard * 2),
            ctypes.c_void_p(M.data_ptr() + guard * 2), 1, 17, 17, 1, nh, nw, None), "fwd")
        ops.check(L.nova_device_status(h), "status")
    finally:
        L.nova_destroy(h)
    b = buf.cpu().numpy()
    assert (b[:guard] == 12345.0).all() and (b[guard + n_out:] == 12345.0).all()
    for ws in (V, M):
        a = ws.cpu().numpy()
        assert (a[:guard] == 777.0).all() and (a[-guard:] == 777.0).all()
    check_parity(x, w, 1, b[guard:guard + n_out].reshape(1, 64, Ho, Wo))


def test_errors_are_reported_not_fatal():
    L = lib()
    h = ops.create_handle()
    try:
        x = torch.zeros(1, 8, 8, 8, dtype=torch.float16, device="cuda")
        y = torch.zeros(1, 8, 8, 8, dtype=torch.float16, device="cuda")
        # forward before set_weights (reference exit(1)s, csrc/nova_winograd.hip:491-494)
        assert L.nova_forward_v2(h, ops.ptr(x), ops.ptr(y), 1, 8, 8, 1, None) == 2
        w = torch.randn(8, 8, 3, 3, device="cuda")
        ops.check(L.nova_set_weights_v2(h, ops.ptr(w), 8, 8, None), "set_weights")
        # workspace tiling too small
        assert L.nova_forward_workspace_v2(h, ops.ptr(x), ops.ptr(y), ops.ptr(y), ops.ptr(y),
                                           1, 8, 8, 1, 1, 1, None) == 3
        # tcgen05 path refused for K % 16 != 0
        assert L.nova_set_path(h, 1) == 1
        assert L.nova_get_K(h) == 8 and L.nova_get_C(h) == 8
        assert L.nova_device_status(h) == 0
    finally:
        L.nova_destroy(h)


# ---------------------------------------------------------------------------
# Stage entry points (reference layouts, reference tiling incl. dead tiles).
# ---------------------------------------------------------------------------

def stage_close(got, want, max_ulps=2, frac=0.999):
    """Elementwise FP16 comparison that tolerates cancellation near zero.

    Error is measured in units of one FP16 ulp of the larger magnitude, with
    magnitudes floored at 1e-4 of the tensor's largest value: an entry that
    cancels to ~0 carries the absolute FP32 rounding of its terms, which is
    no ulp-scale statement.  All entries within max_ulps, and a fraction
    `frac` within 1.
    """
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    scale = np.maximum(np.maximum(np.abs(g), np.abs(w)), 1e-4 * np.abs(w).max())
    ulp = 2.0 ** (np.floor(np.log2(scale)) - 10)
    u = np.abs(g - w) / ulp
    return u.max() <= max_ulps and (u <= 1).mean() >= frac, float(u.max()), float((u <= 1).mean())


@pytest.mark.parametrize("B,C,H,W,pad", [(1, 64, 56, 56, 1), (2, 24, 13, 9, 1), (1, 3, 30, 30, 0)])
def test_input_transform_stage(B, C, H, W, pad):
    x, _ = o.synthetic_case(B, C, 1, H, W, seed=21 + C)
    nh, nw, _, _ = o.compute_tiling(H, W, pad)
    BP = B * nh * nw
    V = torch.full((64, BP, C), 9.0, dtype=torch.float16, device="cuda")
    xd = to_dev(x, torch.float16)
    lib().nova_input_transform(ops.ptr(xd), ops.ptr(V), B, C, H, W, pad, nh, nw, BP)
    torch.cuda.synchronize()
    assert lib().nova_get_last_error(None) == 0
    got = V.cpu().numpy()
    want = o.input_transform(x, nh, nw, pad, "ref")
    ok, worst, within = stage_close(got, want)
    assert ok, (worst, within)


@pytest.mark.parametrize("B,K,H,W", [(1, 64, 56, 56), (2, 40, 13, 9)])
def test_output_transform_stage(B, K, H, W):
    rng = np.random.default_rng(K)
    nh, nw, Ho, Wo = o.compute_tiling(H, W, 1)
    BP = B * nh * nw
    M = rng.standard_normal((64, BP, K), dtype=np.float32).astype(np.float16)
    y = torch.full((B, K, Ho, Wo), 5.0, dtype=torch.float16, device="cuda")
    Md = to_dev(M, torch.float16)
    lib().nova_output_transform(ops.ptr(Md), ops.ptr(y), B, K, Ho, Wo, nh, nw, BP)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    want = o.output_transform(M, B, nh, nw, Ho, Wo, "ref")
    ok, worst, within = stage_close(got, want)
    assert ok, (worst, within)


@pytest.mark.parametrize("K,C", [(64, 64), (48, 24), (5, 3)])
def test_filter_transform_stage_and_get_U(K, C):
    _, w = o.synthetic_case(1, C, K, 1, 1, seed=K * C)
    wd = to_dev(w, torch.float32)
    U = torch.empty(64, C, K, dtype=torch.float16, device="cuda")
    lib().nova_filter_transform(ops.ptr(wd), ops.ptr(U), K, C)
    want = o.filter_transform(w, "ref")
    ok, worst, within = stage_close(U.cpu().numpy(), want)
    assert ok, (worst, within)
    h = ops.create_handle()
    try:
        ops.check(lib().nova_set_weights_v2(h, ops.ptr(wd), K, C, None), "set_weights")
        p = lib().nova_get_U_gemm(h)
        assert p
        Uh = torch.empty(64, C, K, dtype=torch.float16, device="cuda")
        Uh.copy_(_wrap_device_ptr(p, 64 * C * K).view(64, C, K))
        np.testing.assert_array_equal(Uh.cpu().numpy(), U.cpu().numpy())
    finally:
        lib().nova_destroy(h)


def _wrap_device_ptr(p, n):
    """A torch view of n FP16 elements at device pointer p (no copy)."""
    class _Holder:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f2", "data": (p, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(_Holder(), device="cuda")


@pytest.mark.parametrize("B,C,K,H", [(16, 64, 64, 56), (40, 256, 256, 14), (6, 128, 96, 28)])
def test_l2_windowed_three_pass_matches_single_window(B, C, K, H):
    # The batch cut into windows of whole tile rows whose V + M fit an 8 MB
    # budget (NOVA_L2_WINDOW_MB, reference tests/test_bp_tiled.hip:482-571):
    # every tile is computed by the same kernels, so the bytes are the same.
    x, w = o.synthetic_case(B, C, K, H, H, seed=808 + C + H)
    y, _ = run_forward(x, w, 1)
    yw = forward_in_child(x, w, 1, {"NOVA_L2_WINDOW_MB": "8"})
    np.testing.assert_array_equal(y, yw)
    check_parity(x[:2], w, 1, yw[:2])
    check_parity(x[-2:], w, 1, yw[-2:])
