"""ctypes bridge to ``libnova_winograd.so`` (B200, sm_100a).

Mirrors the reference bridge (Jayluci4/nova-wino-amd ``nova_winograd/ops.py``):
the same public names (``get_lib``, ``ptr``, ``compute_tiling``,
``nova_forward``) and the same lazy loading after ``torch.cuda.init()``
(``ops.py:31-114``).  The HSA/HIP preload loop of the reference is gone: the
CUDA library links its runtime statically.

Every call into the library is checked: the reference's library exits the
process on error, this one returns a status that is raised here as
``RuntimeError`` with the library's message.  There is no CPU fallback: without
the built library or a CUDA device these functions raise.
"""

import ctypes
import os

import torch

_lib = None
_LIB_NAME = "libnova_winograd.so"

NOVA_OK = 0

c_int, c_void_p, c_char_p, c_longlong = ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_longlong
_PI = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes): every symbol declared in include/nova_winograd.h.
SIGNATURES = {
    "nova_create": (c_void_p, []),
    "nova_destroy": (None, [c_void_p]),
    "nova_set_weights": (None, [c_void_p, c_void_p, c_int, c_int]),
    "nova_forward": (None, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int]),
    "nova_forward_workspace": (None, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_int, c_int, c_int, c_int]),
    "nova_compute_tiling": (None, [c_int, c_int, c_int, _PI, _PI, _PI, _PI]),
    "nova_filter_transform": (None, [c_void_p, c_void_p, c_int, c_int]),
    "nova_input_transform": (None, [c_void_p, c_void_p] + [c_int] * 8),
    "nova_output_transform": (None, [c_void_p, c_void_p] + [c_int] * 7),
    "nova_get_K": (c_int, [c_void_p]),
    "nova_get_C": (c_int, [c_void_p]),
    "nova_get_U_gemm": (c_void_p, [c_void_p]),
    "nova_fused_create": (c_void_p, []),
    "nova_fused_destroy": (None, [c_void_p]),
    "nova_fused_set_weights": (None, [c_void_p, c_void_p, c_int, c_int]),
    "nova_fused_forward": (None, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int]),
    "nova_fused_compute_tiling": (None, [c_int, c_int, c_int, _PI, _PI, _PI, _PI]),
    "nova_get_last_error": (c_int, [c_void_p]),
    "nova_last_error_string": (c_char_p, []),
    "nova_set_weights_v2": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "nova_forward_v2": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "nova_forward_workspace_v2": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "nova_filter_transform_v2": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "nova_input_transform_v2": (c_int, [c_void_p, c_void_p] + [c_int] * 8 + [c_void_p]),
    "nova_output_transform_v2": (c_int, [c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]),
    "nova_batched_gemm_v2": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "nova_forward_nhwc_v2": (c_int, [c_void_p, c_void_p, c_void_p] + [c_int] * 4 + [c_void_p]),
    "nova_forward_workspace_nhwc_v2": (c_int, [c_void_p] * 5 + [c_int] * 6 + [c_void_p]),
    "nova_input_transform_nhwc_v2": (c_int, [c_void_p, c_void_p] + [c_int] * 8 + [c_void_p]),
    "nova_output_transform_nhwc_v2": (c_int, [c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]),
    "nova_workspace_bytes": (c_longlong, [c_void_p, c_int, c_int, c_int, c_int]),
    "nova_set_path": (c_int, [c_void_p, c_int]),
    "nova_get_path": (c_int, [c_void_p]),
    "nova_device_status": (c_int, [c_void_p]),
    "nova_forward_noalloc": (c_int, [c_void_p, c_void_p, c_void_p] + [c_int] * 6 + [c_void_p]),
    "nova_weight_grad_workspace_bytes": (c_longlong, [c_int] * 6),
    "nova_weight_grad_v2": (c_int, [c_void_p] * 4 + [c_longlong] + [c_int] * 6 + [c_void_p]),
    "nova_version": (c_char_p, []),
}

# Path ids of nova_set_path / nova_get_path.
PATH_AUTO, PATH_TCGEN05, PATH_SIMT, PATH_FUSED = 0, 1, 2, 3


def lib_path_candidates():
    return [
        os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", _LIB_NAME),
        os.path.join(os.getcwd(), _LIB_NAME),
    ]


def _find_lib():
    """Locate the shared library: package ``lib/`` first, then the cwd (ops.py:16-28)."""
    candidates = lib_path_candidates()
    for path in candidates:
        if os.path.exists(path):
            return path
    raise FileNotFoundError(
        f"Cannot find {_LIB_NAME}. Build it with: make -C nova-wino-amd_b200\n"
        f"Searched: {candidates}"
    )


def load_library(path=None):
    """dlopen the library and declare every exported signature (no CUDA calls)."""
    lib = ctypes.CDLL(path or _find_lib(), mode=ctypes.RTLD_GLOBAL)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def _ensure_lib():
    """Load the library lazily, after torch has initialised CUDA (ops.py:31-38)."""
    global _lib
    if _lib is not None:
        return
    if not torch.cuda.is_available():
        raise RuntimeError("nova_winograd needs a CUDA device (B200, sm_100a); none is visible")
    torch.cuda.init()
    _lib = load_library()


def get_lib():
    """The loaded ctypes library handle."""
    _ensure_lib()
    return _lib


def ptr(tensor):
    """Raw device pointer of a torch tensor."""
    return ctypes.c_void_p(tensor.data_ptr())


def stream_ptr(stream=None):
    """cudaStream_t of a torch stream (default: the current stream) as void*."""
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def last_error_message():
    msg = get_lib().nova_last_error_string()
    return msg.decode() if msg else ""


def check(status, what="nova call"):
    """Raise RuntimeError for a non-zero library status."""
    if status != NOVA_OK:
        raise RuntimeError(f"{what} failed (status {status}): {last_error_message()}")
    return status


_tiling_cache = {}


def compute_tiling(H, W, pad):
    """(nh, nw, H_out, W_out) -- the reference's tiling (csrc/nova_winograd.hip:617-631).

    Computed by the library, as in the reference (ops.py:128-144), once per
    (H, W, pad): the module classes ask on every forward.
    """
    key = (int(H), int(W), int(pad))
    hit = _tiling_cache.get(key)
    if hit is not None:
        return hit
    _ensure_lib()
    nh, nw, H_out, W_out = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.nova_compute_tiling(H, W, pad, ctypes.byref(nh), ctypes.byref(nw),
                             ctypes.byref(H_out), ctypes.byref(W_out))
    res = (nh.value, nw.value, H_out.value, W_out.value)
    _tiling_cache[key] = res
    return res


def create_handle(device=None):
    """nova_create on ``device`` (default: current device); raises on failure."""
    lib = get_lib()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        h = lib.nova_create()
    if not h:
        raise RuntimeError(f"nova_create failed: {last_error_message()}")
    return h


def nhwc_eligible(x, K):
    """True when x is a channels-last [B, C, H, W] tensor (and not also plain
    contiguous) that the NHWC kernels take: C % 8 == 0, K even, a 16-byte
    aligned base."""
    return (x.dim() == 4 and not x.is_contiguous()
            and x.is_contiguous(memory_format=torch.channels_last)
            and x.shape[1] % 8 == 0 and K % 2 == 0 and x.data_ptr() % 16 == 0)


def nova_forward(input_fp16, weight_fp32, padding=1):
    """Functional API: NOVA Winograd F(6,3) forward (reference ops.py:147-176).

    Args:
        input_fp16:  [B, C, H, W] float16 CUDA tensor, contiguous, or channels-last
                     with C % 8 == 0 and K even (then the output is channels-last).
        weight_fp32: [K, C, 3, 3] float32 CUDA tensor, contiguous.
        padding:     convolution padding (default 1).

    Returns:
        [B, K, H_out, W_out] float16 tensor.

    Like the reference, this creates a handle, transforms the weights, runs the
    forward and destroys the handle on every call (the module classes cache
    all of that); unlike the reference it runs on the current stream and
    raises instead of exiting on error.
    """
    _ensure_lib()
    if not (input_fp16.is_cuda and input_fp16.dtype == torch.float16):
        raise TypeError("input must be a float16 CUDA tensor")
    if not (weight_fp32.is_cuda and weight_fp32.dtype == torch.float32):
        raise TypeError("weight must be a float32 CUDA tensor")
    nhwc = nhwc_eligible(input_fp16, weight_fp32.shape[0])
    if not ((input_fp16.is_contiguous() or nhwc) and weight_fp32.is_contiguous()):
        raise ValueError("input and weight must be contiguous")
    if weight_fp32.dim() != 4 or tuple(weight_fp32.shape[2:]) != (3, 3):
        raise ValueError("weight must be [K, C, 3, 3]")
    B, C, H, W = input_fp16.shape
    K = weight_fp32.shape[0]
    if weight_fp32.shape[1] != C:
        raise ValueError(f"weight has {weight_fp32.shape[1]} input channels, input has {C}")
    nh, nw, H_out, W_out = compute_tiling(H, W, padding)
    device = input_fp16.device
    fmt = torch.channels_last if nhwc else torch.contiguous_format
    output = torch.empty(B, K, H_out, W_out, dtype=torch.float16, device=device,
                         memory_format=fmt)
    fwd = _lib.nova_forward_nhwc_v2 if nhwc else _lib.nova_forward_v2
    with torch.cuda.device(device):
        s = stream_ptr()
        handle = create_handle(device)
        try:
            check(_lib.nova_set_weights_v2(handle, ptr(weight_fp32), K, C, s), "nova_set_weights")
            check(fwd(handle, ptr(input_fp16), ptr(output), B, H, W, padding, s), "nova_forward")
            torch.cuda.current_stream().synchronize()
        finally:
            _lib.nova_destroy(handle)
    return output


def nova_weight_grad(input_fp16, grad_output_fp16, padding=1):
    """dL/dw of the 3x3 stride-1 convolution by the NOVA F(6,3) Winograd
    algorithm on the GPU (the reference's FP32 unfold loop, conv2d.py:131-141,
    replaced by native kernels): input [B, C, H, W] and grad_output
    [B, K, H_out, W_out], both float16 CUDA tensors; returns float32
    [K, C, 3, 3].  Requires C to be a multiple of 16; its error against the
    exact gradient is of the order of the forward's (a few percent)."""
    lib = get_lib()
    if input_fp16.dtype != torch.float16 or grad_output_fp16.dtype != torch.float16:
        raise TypeError("input and grad_output must be float16")
    x = input_fp16.contiguous()
    dy = grad_output_fp16.contiguous()
    B, C, H, W = x.shape
    K = dy.shape[1]
    if not (x.is_cuda and dy.is_cuda and x.device == dy.device):
        raise ValueError("input and grad_output must be CUDA tensors on one device")
    with torch.cuda.device(x.device):
        nbytes = lib.nova_weight_grad_workspace_bytes(B, C, K, H, W, padding)
        if nbytes < 0:
            raise ValueError("bad sizes for nova_weight_grad")
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        dw = torch.empty(K, C, 3, 3, dtype=torch.float32, device=x.device)
        check(lib.nova_weight_grad_v2(ptr(x), ptr(dy), ptr(dw), ptr(ws), nbytes, B, C, K, H, W,
                                      padding, stream_ptr()), "nova_weight_grad")
    return dw
