"""CPU tests of the C ABI: the library loads, exports exactly what the header
declares, and its host-only entry points and argument checks behave (no kernel
is launched here)."""

import ctypes
import os
import re

import pytest

import nova_oracle as o
from nova_winograd import ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nova_winograd.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nova_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return ops.load_library(ops._find_lib())


def test_library_built_in_tree():
    path = ops._find_lib()
    assert path.startswith(os.path.join(ROOT, "nova-wino-amd_b200"))


def test_exports_every_header_symbol(lib):
    syms = header_symbols()
    assert len(syms) >= 30
    for name in syms:
        assert hasattr(lib, name), name


def test_bridge_binds_every_header_symbol():
    assert sorted(ops.SIGNATURES) == header_symbols()


def test_reference_symbols_present(lib):
    # The 12 symbols the reference bridge binds (ops.py:66-114) + nova_fused_* (fused.hip:619-652).
    for name in ["nova_create", "nova_destroy", "nova_set_weights", "nova_forward",
                 "nova_forward_workspace", "nova_compute_tiling", "nova_filter_transform",
                 "nova_input_transform", "nova_output_transform", "nova_get_K", "nova_get_C",
                 "nova_get_U_gemm", "nova_fused_create", "nova_fused_destroy",
                 "nova_fused_set_weights", "nova_fused_forward", "nova_fused_compute_tiling"]:
        assert hasattr(lib, name)


def _tiling(fn, H, W, pad):
    a, b, c, d = (ctypes.c_int() for _ in range(4))
    fn(H, W, pad, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), ctypes.byref(d))
    return a.value, b.value, c.value, d.value


def test_compute_tiling_matches_reference(lib):
    import json
    rows = json.load(open(os.path.join(ROOT, "tests", "golden", "tiling.json")))["rows"]
    for H, W, pad, nh, nw, Ho, Wo in rows:
        assert _tiling(lib.nova_compute_tiling, H, W, pad) == (nh, nw, Ho, Wo)
        assert _tiling(lib.nova_fused_compute_tiling, H, W, pad) == (nh, nw, Ho, Wo)


def test_null_handle_and_argument_errors(lib):
    # Host-side validation returns a status instead of exiting the process.
    assert lib.nova_set_weights_v2(None, None, 64, 64, None) == 1
    assert lib.nova_forward_v2(None, None, None, 1, 8, 8, 1, None) == 1
    assert lib.nova_filter_transform_v2(None, None, 4, 4, None) == 1
    assert lib.nova_input_transform_v2(None, None, 1, 4, 8, 8, 1, 2, 2, 4, None) == 1
    assert lib.nova_output_transform_v2(None, None, 1, 4, 8, 8, 2, 2, 4, None) == 1
    assert lib.nova_get_last_error(None) == 1
    assert b"bad arguments" in lib.nova_last_error_string()
    assert lib.nova_set_path(None, 0) == 1
    assert lib.nova_get_K(None) == 0 and lib.nova_get_C(None) == 0
    assert lib.nova_workspace_bytes(None, 1, 8, 8, 1) == -1
    # Void reference entry points with a null handle record the error and return.
    lib.nova_set_weights(None, None, 4, 4)
    lib.nova_forward(None, None, None, 1, 8, 8, 1)
    assert lib.nova_get_last_error(None) == 1


def test_nhwc_entries_validate_before_any_launch(lib):
    fake = ctypes.c_void_p(0x1000)
    # Null tensors, C % 8 != 0, odd K, misaligned x, BP short of the tiling.
    assert lib.nova_forward_nhwc_v2(None, None, None, 1, 8, 8, 1, None) == 1
    assert lib.nova_input_transform_nhwc_v2(None, None, 1, 8, 8, 8, 1, 2, 2, 4, None) == 1
    assert lib.nova_input_transform_nhwc_v2(fake, fake, 1, 12, 8, 8, 1, 2, 2, 4, None) == 1
    assert lib.nova_input_transform_nhwc_v2(ctypes.c_void_p(0x1004), fake, 1, 8, 8, 8, 1, 2, 2,
                                            4, None) == 1
    assert lib.nova_input_transform_nhwc_v2(fake, fake, 2, 8, 8, 8, 1, 2, 2, 7, None) == 1
    assert lib.nova_output_transform_nhwc_v2(fake, fake, 1, 7, 8, 8, 2, 2, 4, None) == 1
    assert lib.nova_output_transform_nhwc_v2(None, fake, 1, 8, 8, 8, 2, 2, 4, None) == 1
    assert b"bad arguments" in lib.nova_last_error_string()


def test_stage_bp_smaller_than_tiling_rejected(lib):
    fake = ctypes.c_void_p(0x1000)
    # BP must cover batch*nh*nw.
    assert lib.nova_input_transform_v2(fake, fake, 2, 4, 8, 8, 1, 2, 2, 7, None) == 1


def test_create_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU visible")
    assert lib.nova_create() is None
    assert b"no CUDA device" in lib.nova_last_error_string()


def test_oracle_tiling_equals_library_tiling(lib):
    for H in (1, 7, 14, 28, 56, 64, 100, 224):
        for pad in (0, 1, 2):
            if H + 2 * pad - 2 <= 0:
                continue
            assert _tiling(lib.nova_compute_tiling, H, H + 3, pad) == o.compute_tiling(H, H + 3, pad)
