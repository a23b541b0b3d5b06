"""GPU test of nova_forward_noalloc, the entry point for callers that may not
allocate device memory when they run the convolution (for example a plugin
inside a runtime that owns all device memory).  It must give the same result
as the ordinary nova_forward entry point, call after call, while keeping its
intermediates in the library's fixed scratch array.

Kept in a file of its own that pytest collects last.
"""

import numpy as np
import pytest
import torch

import nova_oracle as o
from nova_winograd import ops

pytestmark = pytest.mark.gpu

PARITY_TOL = 1e-2  # same bar as the other parity tests (tests/test_gpu_parity.py)


def _reference_forward(lib, xd, wd, pad):
    B, C, H, W = xd.shape
    K = wd.shape[0]
    _, _, Ho, Wo = ops.compute_tiling(H, W, pad)
    y = torch.empty(B, K, Ho, Wo, dtype=torch.float16, device="cuda")
    h = ops.create_handle()
    try:
        ops.check(lib.nova_set_weights_v2(h, ops.ptr(wd), K, C, None), "set_weights")
        ops.check(lib.nova_forward_v2(h, ops.ptr(xd), ops.ptr(y), B, H, W, pad, None), "forward")
        torch.cuda.synchronize()
    finally:
        lib.nova_destroy(h)
    return y


def test_noalloc_matches_forward_twice_in_a_row():
    lib = ops.get_lib()
    B, C, K, H, W, pad = 2, 64, 96, 28, 28, 1
    # Everything the caller owns is set up front; the no-alloc call itself
    # allocates nothing.
    U = torch.empty(64, C, K, dtype=torch.float16, device="cuda")
    y = torch.empty(B, K, H, W, dtype=torch.float16, device="cuda")
    for call, seed in enumerate((11, 12)):  # second call reuses the dirty scratch
        x, w = o.synthetic_case(B, C, K, H, W, seed=seed)
        xd = torch.from_numpy(x).cuda()
        wd = torch.from_numpy(w).cuda()
        lib.nova_filter_transform(ops.ptr(wd), ops.ptr(U), K, C)
        y.fill_(float("nan"))
        ops.check(lib.nova_forward_noalloc(ops.ptr(xd), ops.ptr(U), ops.ptr(y), B, C, K, H, W, pad,
                                           None), "nova_forward_noalloc")
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        want = _reference_forward(lib, xd, wd, pad).cpu().numpy()
        assert np.isfinite(got.astype(np.float32)).all(), f"call {call}: NaN/Inf"
        assert o.rel_l2(got, want) <= PARITY_TOL, f"call {call}: rel L2 {o.rel_l2(got, want):.3e}"
        # And against the CPU oracle, by the bars of the other parity tests.
        y_o = o.nova_forward(x, w, pad, "ref")
        d = o.direct_conv_fp64(x, w, pad)
        assert o.rel_l2(got, y_o) <= PARITY_TOL, f"call {call}: vs oracle {o.rel_l2(got, y_o):.3e}"
        assert o.rel_l2(got, d) <= 1.1 * o.rel_l2(y_o, d), f"call {call}: accuracy"


def test_noalloc_refuses_shapes_beyond_its_scratch():
    lib = ops.get_lib()
    B, C, K, H = 64, 64, 64, 56  # V + M ~ 105 MB > 32 MiB
    fake = torch.empty(16, dtype=torch.float16, device="cuda")
    rc = lib.nova_forward_noalloc(ops.ptr(fake), ops.ptr(fake), ops.ptr(fake), B, C, K, H, H, 1,
                                  None)
    assert rc == 3  # NOVA_ERR_WORKSPACE
    assert b"scratch" in lib.nova_last_error_string()
