"""ctypes binding of libargus_b200.so (the C ABI in include/argus_b200.h).

The library is the only compute path: if it is missing, or CUDA is unavailable, calls raise
instead of falling back to torch or CPU code.  Tensors are passed as raw device pointers;
work is enqueued on torch's current CUDA stream.
"""
import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libargus_b200.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_MISALIGNED = 2
ERR_CUDA = 3
ERR_UNSUPPORTED = 4
ERR_TIMEOUT = 5
ERR_CAPACITY = 6

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> argtypes (all return int status)
SIGNATURES = {
    "argus_quant_int8": [_p, _i64, _i32, _p, _p, _p],
    "argus_dequant_int8": [_p, _p, _i64, _i32, _p, _p],
    "argus_quant_fp8sim": [_p, _i64, _i32, _p, _p, _p],
    "argus_dequant_fp8sim": [_p, _p, _i64, _i32, _p, _p],
    "argus_quant_e4m3": [_p, _i64, _i32, _p, _p, _p],
    "argus_dequant_e4m3": [_p, _p, _i64, _i32, _p, _p],
    "argus_quant_int4": [_p, _i64, _i32, _p, _p, _p, _p],
    "argus_dequant_int4": [_p, _p, _p, _i64, _i32, _p, _p],
    "argus_quant_int2": [_p, _i64, _i32, _p, _p, _p, _p],
    "argus_dequant_int2": [_p, _p, _p, _i64, _i32, _p, _p],
    "argus_quant_1bit": [_p, _i64, _i32, _p, _p, _p],
    "argus_dequant_1bit": [_p, _p, _i64, _i32, _p, _p],
    "argus_pack_int4_codes": [_p, _i64, _i32, _p, _p],
    "argus_pack_1bit_signs": [_p, _i64, _i32, _p, _p],
    "argus_isolate_outliers": [_p, _i64, _i32, _f32, _p, _p, _p, _p],
    "argus_jl_apply": [_p, _p, _i64, _i32, _i32, _i32, _p, _p],
    "argus_memcpy_async": [_p, _p, _i64, _p],
    "argus_memcpy2d_async": [_p, _i64, _p, _i64, _i64, _i64, _p],
    "argus_attention_accumulate": [_p, _p, _p, _p, _i64, _i32, _p],
    "argus_scatter_coo": [_p, _i64, _i64, _i32, _i32, _i32, _i32, _p, _p, _i64, _p],
    "argus_outliers_to_coo": [_p, _p, _i32, _i32, _i32, _i32, _p, _p, _i64, _p, _p],
    "argus_selftest_fp16_quotients": [_p, _p],
    "argus_selftest_wait_timeout": [_i64, _p, _p],
}


class ArgusError(RuntimeError):
    """A failed call into libargus_b200 (status code and detail text)."""

    def __init__(self, fn, status, detail):
        self.status = status
        super().__init__(f"{fn}: {status_string(status)} ({detail})")


_lib = None


def lib():
    """Loads the library once; raises if it is absent or has no usable GPU."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libargus_b200.so not found at {LIB_PATH}; build it with `python -m argus_b200.build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.argus_status_string.restype = ctypes.c_char_p
        L.argus_status_string.argtypes = [_i32]
        L.argus_last_error.restype = ctypes.c_char_p
        L.argus_version.restype = _i32
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _i32
        _lib = L
    return _lib


def status_string(status):
    return lib().argus_status_string(status).decode()


def call(name, *args):
    """Calls an entry point and raises on a non-zero status.  Divisibility failures raise
    AssertionError, as the reference's asserts do (core/quantization.py:41,79,183)."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        detail = lib().argus_last_error().decode()
        if rc == ERR_INVALID_ARGUMENT and "multiple" in detail:
            raise AssertionError(f"{name}: {detail}")
        raise ArgusError(name, rc, detail)


def stream_handle(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr_stream(stream):
    return ctypes.c_void_p(stream.cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def require_cuda(t, what="tensor"):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"argus_b200 runs on CUDA tensors only; {what} is on "
                         f"{getattr(t, 'device', type(t).__name__)} (there is no CPU fallback)")
