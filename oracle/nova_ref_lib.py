"""Loader for oracle/_ref/libnova_ref.so: the reference's own kernels on a GPU.

TEST INFRASTRUCTURE ONLY.  ``oracle/ref_build/Makefile`` compiles the
reference's ``csrc/nova_winograd.hip`` (Jayluci4/nova-wino-amd) unchanged with
nvcc for sm_100a, through a HIP -> CUDA and rocBLAS -> cuBLAS name shim
(``oracle/ref_build/shim/``).  The library exports the reference's C API
(``csrc/nova_winograd.hip:684-754``) with the reference's own code behind it:

* ``nova_filter_transform``  ``filter_transform_kernel``  (``:214-255``)
* ``nova_input_transform``   ``input_transform_kernel``   (``:141-205``, one tile per block)
* ``nova_output_transform``  ``output_transform_kernel``  (``:264-328``)
* ``nova_forward[_workspace]``  ``input_transform_kernel_mt`` (``:338-392``) ->
  ``gemm_strided_batched_ex`` (``:534-548``, here cuBLAS with FP32 compute) ->
  ``output_transform_kernel_mt`` (``:398-450``); the multi-tile kernels'
  64-lane ``__shfl`` runs through an exact shared-memory exchange.

Tests use it to pin the numpy oracle and the product library against the
reference's arithmetic.  All entry points work on the legacy default stream,
and errors ``exit(1)`` the process, as in the reference.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libnova_ref.so")

_vp, _i = ctypes.c_void_p, ctypes.c_int
_SIGS = {
    "nova_create": (_vp, []),
    "nova_destroy": (None, [_vp]),
    "nova_set_weights": (None, [_vp, _vp, _i, _i]),
    "nova_forward": (None, [_vp, _vp, _vp, _i, _i, _i, _i]),
    "nova_forward_workspace": (None, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "nova_compute_tiling": (None, [_i, _i, _i] + [ctypes.POINTER(_i)] * 4),
    "nova_filter_transform": (None, [_vp, _vp, _i, _i]),
    "nova_input_transform": (None, [_vp, _vp] + [_i] * 8),
    "nova_output_transform": (None, [_vp, _vp] + [_i] * 7),
    "nova_get_K": (_i, [_vp]),
    "nova_get_C": (_i, [_vp]),
    "nova_get_U_gemm": (_vp, [_vp]),
}

_lib = None


def available() -> bool:
    return os.path.exists(REF_LIB)


def load():
    """The reference library (RTLD_LOCAL, so its nova_* symbols never shadow
    the product library's)."""
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(REF_LIB, mode=ctypes.RTLD_LOCAL)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
