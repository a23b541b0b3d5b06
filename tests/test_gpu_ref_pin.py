"""The reference's own kernels, run on the GPU, pin the CPU oracle and the library.

``oracle/_ref/libnova_ref.so`` is the reference's ``csrc/nova_winograd.hip``
compiled unchanged for sm_100a (``oracle/ref_build``; rocBLAS mapped onto
cuBLAS with FP32 compute).  On small seeded shapes these tests check:

* bit for bit: the reference's stage kernels (filter ``:214-255``, single-tile
  input ``:141-205`` and output ``:264-328`` transforms) against the oracle's
  exact-order restatements (``*_seq``: the kernels' FMA chains in their order);
* the same stages against the oracle's fast "ref" functions, and the
  library's stage kernels against the reference's, within FP32 reordering:
  |a - b| <= 1 FP16 ulp + 2 * terms * 2^-24 * (sum of the terms' magnitudes);
* the reference's whole forward (``forward_workspace``, ``:564-610``: the
  multi-tile kernels and the batched GEMM), stage by stage through the
  workspace it fills: its V bit for bit against the oracle, its M against the
  oracle's GEMM of its own U and V within FP32 reordering, its y bit for bit
  against the oracle's output transform of its own M;
* whole outputs: oracle, reference and library within the parity bar
  (rel L2 <= 1e-2), and the library's error against an FP64 direct
  convolution <= 1.1x the reference's.

When the reference library was not built (no reference checkout on the
building machine) the tests skip.
"""

import ctypes

import numpy as np
import pytest
import torch

import nova_oracle as o
import nova_ref_lib
from nova_winograd import ops

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not nova_ref_lib.available(),
                                 reason="oracle/_ref/libnova_ref.so not built")]

PARITY_TOL = 1e-2  # whole outputs, as in the oracle parity tests

CASES = [  # B, C, K, H, W, pad
    (1, 64, 64, 28, 28, 1),
    (2, 16, 32, 14, 14, 1),
    (2, 32, 48, 13, 17, 1),
    (1, 8, 24, 10, 9, 0),
    (3, 64, 128, 7, 7, 1),
    (1, 128, 64, 56, 56, 1),
]


def ids(c):
    return "B%d_C%d_K%d_%dx%d_p%d" % c


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def ordered(h):
    """FP16 bit patterns -> integers that are monotonic in the value."""
    i = np.asarray(h, dtype=np.float16).view(np.int16).astype(np.int32)
    return np.where(i < 0, -32768 - i, i)


def ulp_diff(a, b):
    return np.abs(ordered(a) - ordered(b))


def ref_tiling(H, W, pad):
    v = [ctypes.c_int() for _ in range(4)]
    nova_ref_lib.load().nova_compute_tiling(H, W, pad, *[ctypes.byref(t) for t in v])
    return tuple(t.value for t in v)


def input_scale(x, nh, nw, pad):
    return o.input_transform_scale(x, nh, nw, pad)


def filter_scale(w):
    return o.filter_transform_scale(w)


def output_scale(M, B, nh, nw, Ho, Wo):
    return o.output_transform_scale(M, B, nh, nw, Ho, Wo)


def assert_exact(got, want, what):
    bad = ulp_diff(got, want)
    assert bad.max() == 0, f"{what}: {(bad > 0).sum()} of {bad.size} differ (max {bad.max()} ulp)"


def assert_reordering(got, want, scale, terms, what):
    ok = o.within_fp32_reordering(got, want, scale, terms)
    assert ok.all(), f"{what}: {(~ok).sum()} of {ok.size} outside FP32 reordering"


@pytest.mark.parametrize("case", CASES, ids=ids)
def test_reference_stages_pin_oracle_stages(case):
    B, C, K, H, W, pad = case
    R = nova_ref_lib.load()
    x, w = o.synthetic_case(B, C, K, H, W, seed=500 + C + H)
    nh, nw, Ho, Wo = ref_tiling(H, W, pad)
    assert (nh, nw, Ho, Wo) == o.compute_tiling(H, W, pad)
    BP = B * nh * nw
    xd, wd = dev(x, torch.float16), dev(w, torch.float32)

    U = torch.empty(64, C, K, dtype=torch.float16, device="cuda")
    R.nova_filter_transform(ops.ptr(wd), ops.ptr(U), K, C)
    U = U.cpu().numpy()
    assert_exact(U, o.filter_transform_seq(w), "filter transform vs exact-order oracle")
    assert_reordering(U, o.filter_transform(w, "ref"), filter_scale(w), 9, "filter transform")

    V = torch.empty(64, BP, C, dtype=torch.float16, device="cuda")
    R.nova_input_transform(ops.ptr(xd), ops.ptr(V), B, C, H, W, pad, nh, nw, BP)
    torch.cuda.synchronize()
    V = V.cpu().numpy()
    assert_exact(V, o.input_transform_seq(x, nh, nw, pad), "input transform vs exact-order oracle")
    assert_reordering(V, o.input_transform(x, nh, nw, pad, "ref"), input_scale(x, nh, nw, pad),
                      16, "input transform")

    M_o = o.gemm(o.filter_transform(w, "ref"), o.input_transform(x, nh, nw, pad, "ref"), "ref")
    y = torch.full((B, K, Ho, Wo), float("nan"), dtype=torch.float16, device="cuda")
    R.nova_output_transform(ops.ptr(dev(M_o, torch.float16)), ops.ptr(y), B, K, Ho, Wo, nh, nw,
                            BP)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    assert_exact(y, o.output_transform_seq(M_o, B, nh, nw, Ho, Wo),
                 "output transform vs exact-order oracle")
    assert_reordering(y, o.output_transform(M_o, B, nh, nw, Ho, Wo, "ref"),
                      output_scale(M_o, B, nh, nw, Ho, Wo), 16, "output transform")


def reference_forward(x, w, pad, workspace=True):
    """The reference's NovaWinogradF63 (csrc/nova_winograd.hip:456-611).
    Returns (y, V, M): V [64][BP][C] and M [64][BP][K] from the caller
    workspace of forward_workspace, or None when ``workspace`` is False
    (forward allocates its own)."""
    R = nova_ref_lib.load()
    B, C, H, W = x.shape
    K = w.shape[0]
    nh, nw, Ho, Wo = ref_tiling(H, W, pad)
    BP = B * nh * nw
    xd, wd = dev(x, torch.float16), dev(w, torch.float32)
    y = torch.full((B, K, Ho, Wo), float("nan"), dtype=torch.float16, device="cuda")
    V = Mw = None
    torch.cuda.synchronize()
    h = R.nova_create()
    try:
        R.nova_set_weights(h, ops.ptr(wd), K, C)
        assert R.nova_get_K(h) == K and R.nova_get_C(h) == C and R.nova_get_U_gemm(h)
        if workspace:
            V = torch.full((64, BP, C), float("nan"), dtype=torch.float16, device="cuda")
            Mw = torch.full((64, BP, K), float("nan"), dtype=torch.float16, device="cuda")
            R.nova_forward_workspace(h, ops.ptr(xd), ops.ptr(y), ops.ptr(V), ops.ptr(Mw), B, H, W,
                                     pad, nh, nw)
        else:
            R.nova_forward(h, ops.ptr(xd), ops.ptr(y), B, H, W, pad)
        torch.cuda.synchronize()
    finally:
        R.nova_destroy(h)
    if workspace:
        return y.cpu().numpy(), V.cpu().numpy(), Mw.cpu().numpy()
    return y.cpu().numpy(), None, None


@pytest.mark.parametrize("case", CASES, ids=ids)
def test_reference_forward_pins_oracle_forward(case):
    B, C, K, H, W, pad = case
    x, w = o.synthetic_case(B, C, K, H, W, seed=600 + C + H)
    nh, nw, Ho, Wo = ref_tiling(H, W, pad)
    y_r, V_r, M_r = reference_forward(x, w, pad, workspace=True)
    assert np.isfinite(y_r.astype(np.float32)).all()
    # Stage by stage through the workspace the reference filled.
    assert_exact(V_r, o.input_transform_seq(x, nh, nw, pad), "forward V (multi-tile kernel)")
    U = o.filter_transform_seq(w)
    assert_reordering(M_r, o.gemm(U, V_r, "ref"), o.gemm_scale(U, V_r), C, "forward M (GEMM)")
    assert_exact(y_r, o.output_transform_seq(M_r, B, nh, nw, Ho, Wo),
                 "forward y (multi-tile kernel)")
    # Whole output: the oracle's forward and the reference's agree within the
    # parity bar, and so do their errors against FP64.
    y_o = o.nova_forward(x, w, pad, "ref")
    assert o.rel_l2(y_o, y_r) <= PARITY_TOL
    d = o.direct_conv_fp64(x, w, pad)
    assert abs(o.rel_l2(y_r, d) - o.rel_l2(y_o, d)) <= 0.05 * o.rel_l2(y_o, d)
    # nova_forward (internal workspace) is the same computation.
    y_a, _, _ = reference_forward(x, w, pad, workspace=False)
    assert o.rel_l2(y_a, y_r) <= PARITY_TOL


@pytest.mark.parametrize("case", CASES, ids=ids)
def test_library_matches_reference(case):
    B, C, K, H, W, pad = case
    L = ops.get_lib()
    R = nova_ref_lib.load()
    x, w = o.synthetic_case(B, C, K, H, W, seed=700 + C + H)
    nh, nw, Ho, Wo = ref_tiling(H, W, pad)
    BP = B * nh * nw
    xd, wd = dev(x, torch.float16), dev(w, torch.float32)
    s = ops.stream_ptr()

    # Stage entries, called the way benchmarks/bench_profile_stages.py calls them.
    V_r = torch.empty(64, BP, C, dtype=torch.float16, device="cuda")
    V_l = torch.empty_like(V_r)
    R.nova_input_transform(ops.ptr(xd), ops.ptr(V_r), B, C, H, W, pad, nh, nw, BP)
    torch.cuda.synchronize()
    ops.check(L.nova_input_transform_v2(ops.ptr(xd), ops.ptr(V_l), B, C, H, W, pad, nh, nw, BP, s),
              "input_transform")
    torch.cuda.synchronize()
    assert_reordering(V_l.cpu().numpy(), V_r.cpu().numpy(), input_scale(x, nh, nw, pad), 16,
                      "library V vs reference V")

    U_r = torch.empty(64, C, K, dtype=torch.float16, device="cuda")
    U_l = torch.empty_like(U_r)
    R.nova_filter_transform(ops.ptr(wd), ops.ptr(U_r), K, C)
    L.nova_filter_transform(ops.ptr(wd), ops.ptr(U_l), K, C)
    torch.cuda.synchronize()
    assert_reordering(U_l.cpu().numpy(), U_r.cpu().numpy(), filter_scale(w), 9,
                      "library U vs reference U")

    y_r, _, M_r = reference_forward(x, w, pad, workspace=True)
    y_m = torch.full((B, K, Ho, Wo), float("nan"), dtype=torch.float16, device="cuda")
    ops.check(L.nova_output_transform_v2(ops.ptr(dev(M_r, torch.float16)), ops.ptr(y_m), B, K, Ho,
                                         Wo, nh, nw, BP, s), "output_transform")
    torch.cuda.synchronize()
    assert_reordering(y_m.cpu().numpy(), y_r, output_scale(M_r, B, nh, nw, Ho, Wo), 16,
                      "library output transform vs reference on the reference's M")

    y_l = ops.nova_forward(xd, wd, padding=pad).cpu().numpy()
    assert np.isfinite(y_l.astype(np.float32)).all()
    par = o.rel_l2(y_l, y_r)
    assert par <= PARITY_TOL, f"library vs reference: rel L2 {par:.3e}"
    d = o.direct_conv_fp64(x, w, pad)
    assert o.rel_l2(y_l, d) <= 1.1 * o.rel_l2(y_r, d)
