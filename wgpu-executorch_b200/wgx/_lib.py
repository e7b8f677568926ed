"""ctypes binding of the C ABI declared in include/wgx.h.

Maps the in-tree ``lib/libwgx.so`` on first use: importing the package
(e.g. for the pure-Python program transforms in ``wgx.programs``) maps
nothing, and the first call through ``lib`` loads the library. There is no
fallback: when the library is missing, that first call raises ImportError,
so nothing can silently run on a CPU path. ``load()`` maps it eagerly.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, Union, c_char_p, c_double, c_float, c_int, c_int32,
                    c_int64, c_uint32, c_uint64, c_void_p)

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# WGX_LIBRARY=bounds loads the bounds-checking debug build (lib/libwgx_bounds.so,
# `make -C wgpu-executorch_b200 bounds`) instead of the normal library;
# WGX_LIBRARY_PATH names any other build of the same C ABI.
LIB_PATH = os.environ.get("WGX_LIBRARY_PATH") or os.path.join(
    PKG_DIR, "lib", "libwgx_bounds.so" if os.environ.get("WGX_LIBRARY") == "bounds" else "libwgx.so")

WGX_OK = 0
WGX_ERR_INVALID = 1
WGX_ERR_CUDA = 2
WGX_ERR_DESTROYED = 3
WGX_ERR_NOMEM = 4
WGX_ERR_DEVICE = 5

DTYPES = ["float32", "float16", "int32", "int8", "uint8", "bool", "float64", "int64"]
DTYPE_CODE = {n: i for i, n in enumerate(DTYPES)}
DTYPE_BYTESIZE = {"float32": 4, "float16": 2, "float64": 8, "int32": 4, "int64": 8,
                  "int8": 1, "uint8": 1, "bool": 1}

ARG_NULL, ARG_TENSOR, ARG_NUMBER, ARG_BOOL, ARG_INT_LIST, ARG_TENSOR_LIST, ARG_STRING = range(7)

ACT_NONE, ACT_CLAMP, ACT_SILU = 0, 1, 2
INJECT_ALLOC_FAIL, INJECT_SKIP_LOADS = 1, 2
BUILD_BOUNDS = 1
CONV_UMMA, CONV_SIMT_GEMM, CONV_DEPTHWISE, CONV_DIRECT, CONV_POINTWISE1 = 1, 2, 3, 4, 5


class _ArgValue(Union):
    _fields_ = [("tensor", c_void_p), ("number", c_double), ("boolean", c_int32),
                ("ints", POINTER(c_int64)), ("tensors", POINTER(c_void_p)),
                ("string", c_char_p)]


class WgxArg(Structure):
    _fields_ = [("kind", c_int32), ("count", c_int32), ("v", _ArgValue)]


class ConvParams(Structure):
    _fields_ = [(n, c_int32) for n in
                ("B", "IC", "IH", "IW", "OC", "OH", "OW", "KH", "KW", "sH", "sW", "pH", "pW",
                 "dH", "dW", "groups", "has_bias", "dtype", "act")] + \
               [("out_min", c_float), ("out_max", c_float)]


class ConvPlan(Structure):
    _fields_ = [("variant", c_int32), ("n_launches", c_int32), ("scratch_bytes", c_uint64),
                ("grid_ctas", c_uint64)]


# (name, argtypes) of every exported function; tests check each is present
SIGNATURES = {
    "wgx_last_error": ([], c_char_p),
    "wgx_version": ([], c_int),
    "wgx_device_count": ([POINTER(c_int)], c_int),
    "wgx_context_create": ([c_int, POINTER(c_void_p)], c_int),
    "wgx_context_destroy": ([c_void_p], c_int),
    "wgx_context_release": ([c_void_p], c_int),
    "wgx_storage_buffer": ([c_void_p, c_uint64, POINTER(c_void_p)], c_int),
    "wgx_buffer_create": ([c_int, c_uint64, c_uint32, POINTER(c_void_p)], c_int),
    "wgx_buffer_destroy": ([c_void_p], c_int),
    "wgx_buffer_info": ([c_void_p, POINTER(c_uint64), POINTER(c_uint32), POINTER(c_void_p)], c_int),
    "wgx_tensor_create": ([c_void_p, c_int, POINTER(c_int64), c_int, c_void_p, POINTER(c_void_p)],
                          c_int),
    "wgx_tensor_release": ([c_void_p], c_int),
    "wgx_tensor_info": ([c_void_p, POINTER(c_int), POINTER(c_int), POINTER(c_int64),
                         POINTER(c_uint64), POINTER(c_void_p)], c_int),
    "wgx_tensor_set_data": ([c_void_p, c_void_p, c_uint64], c_int),
    "wgx_tensor_get_data": ([c_void_p, c_void_p, c_uint64], c_int),
    "wgx_copy": ([c_void_p, c_void_p, c_void_p], c_int),
    "wgx_record_op": ([c_void_p, c_char_p, POINTER(WgxArg), c_int], c_int),
    "wgx_record_program": ([c_void_p, c_char_p, c_uint64, c_void_p, c_uint64, POINTER(WgxArg),
                            c_int], c_int),
    "wgx_submit": ([c_void_p], c_int),
    "wgx_sync": ([c_void_p], c_int),
    "wgx_reset": ([c_void_p], c_int),
    "wgx_context_stats": ([c_void_p, POINTER(c_int64), POINTER(c_int64)], c_int),
    "wgx_context_stream": ([c_void_p, POINTER(c_void_p)], c_int),
    "wgx_context_profile": ([c_void_p, c_int, POINTER(c_double), c_int, POINTER(c_int)], c_int),
    "wgx_context_command_name": ([c_void_p, c_int], c_char_p),
    "wgx_pipeline_create": ([c_void_p, c_void_p, c_void_p, c_int, POINTER(c_void_p)], c_int),
    "wgx_pipeline_step": ([c_void_p, c_void_p, c_void_p], c_int),
    "wgx_pipeline_sync": ([c_void_p], c_int),
    "wgx_pipeline_destroy": ([c_void_p], c_int),
    "wgx_mm_scratch_bytes": ([c_int64, c_int64, c_int64, c_int, POINTER(c_uint64)], c_int),
    "wgx_mm": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p,
                c_uint64, c_void_p], c_int),
    "wgx_conv2d_plan_for": ([POINTER(ConvParams), POINTER(ConvPlan)], c_int),
    "wgx_conv2d_describe": ([POINTER(ConvParams), c_char_p, c_int32], c_int),
    "wgx_conv2d": ([POINTER(ConvParams), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                    c_uint64, c_void_p], c_int),
    "wgx_conv2d_noalloc": ([POINTER(ConvParams), c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p], c_int),
    "wgx_device_error": ([c_int, POINTER(c_uint32), c_int], c_int),
    "wgx_debug_inject": ([c_uint32], c_int),
    "wgx_build_flags": ([POINTER(c_uint32)], c_int),
    "wgx_kernel_timing": ([c_int], c_int),
    "wgx_kernel_timing_read": ([c_char_p, POINTER(c_double), POINTER(c_int64), c_int], c_int),
}


class WgxError(Exception):
    """Raised with the library's message when a C-ABI call fails."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built: run `make -C {PKG_DIR}` "
                          "(or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


class _Library:
    """The C ABI, mapped on first attribute access (see the module
    docstring)."""

    _cdll = None

    def __getattr__(self, name):
        if _Library._cdll is None:
            _Library._cdll = _load()
        return getattr(_Library._cdll, name)


lib = _Library()


def load() -> ctypes.CDLL:
    """Maps the library now (raises ImportError when it is not built)."""
    lib.wgx_last_error  # noqa: B018  (first access maps it)
    return _Library._cdll


def check(code: int) -> None:
    if code != WGX_OK:
        msg = lib.wgx_last_error()
        raise WgxError(code, msg.decode() if msg else f"wgx error {code}")


def device_count() -> int:
    n = c_int(0)
    check(lib.wgx_device_count(ctypes.byref(n)))
    return n.value


def build_flags() -> int:
    """WGX_BUILD_* bits of the loaded library (BUILD_BOUNDS: the
    bounds-checking debug build)."""
    f = c_uint32(0)
    check(lib.wgx_build_flags(ctypes.byref(f)))
    return f.value
