"""TEST INFRASTRUCTURE ONLY: Python front-end of the CPU oracle.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
import this module, and only as the checker / timed CPU baseline. The
product (the wgx library and its Python mirror) never does.

* ``mm`` / ``conv2d`` / ``conv_transpose2d`` call the C restatement of the
  reference WGSL kernels in ``liboracle.so`` (wgsl_oracle.c), mode
  ``"exact"`` (fp64 accumulation, one rounding) or ``"wgsl"`` (the
  reference kernel's own f16/f32 arithmetic and summation order).
* elementwise ops follow the reference WGSL expressions with numpy
  (float16 numpy arithmetic rounds every operation, like shader f16 math).
* ``make_inputs`` draws the seeded synthetic inputs (numpy PCG64).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_float, c_int, c_int32, c_long, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

EXACT, WGSL = 0, 1
ACT_NONE, ACT_CLAMP, ACT_SILU = 0, 1, 2


class ConvParams(Structure):
    _fields_ = [(n, c_int32) for n in
                ("B", "IC", "IH", "IW", "OC", "OH", "OW", "KH", "KW", "sH", "sW", "pH", "pW",
                 "dH", "dW", "groups", "has_bias", "dtype", "act")] + \
               [("out_min", c_float), ("out_max", c_float)]


def _load():
    if not os.path.exists(LIB):
        raise ImportError(f"{LIB} missing: run `make -C {HERE}`")
    lib = ctypes.CDLL(LIB)
    lib.oracle_mm.argtypes = [c_int, c_int, c_void_p, c_void_p, c_void_p, c_long, c_long, c_long]
    lib.oracle_conv2d.argtypes = [c_int, c_int, POINTER(ConvParams), c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_int]
    lib.oracle_conv_transpose2d.argtypes = [c_int, POINTER(ConvParams), c_void_p, c_void_p,
                                            c_void_p, c_void_p]
    lib.oracle_num_threads.restype = c_int
    return lib


_lib = _load()


def num_threads() -> int:
    return int(_lib.oracle_num_threads())


def _mode(m):
    return {"exact": EXACT, "wgsl": WGSL}[m] if isinstance(m, str) else int(m)


def _dt(arr):
    if arr.dtype == np.float16:
        return 1
    if arr.dtype == np.float32:
        return 0
    raise TypeError(arr.dtype)


def _ptr(a):
    return a.ctypes.data_as(c_void_p) if a is not None else None


def mm(a: np.ndarray, b: np.ndarray, mode="exact") -> np.ndarray:
    """out = a @ b in the storage dtype (src/shaders/mm)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b.astype(a.dtype))
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    out = np.empty((M, N), dtype=a.dtype)
    _lib.oracle_mm(_dt(a), _mode(mode), _ptr(a), _ptr(b), _ptr(out), M, N, K)
    return out


def conv_out_hw(ih, iw, kh, kw, stride, pad, dil):
    oh = (ih + 2 * pad[0] - dil[0] * (kh - 1) - 1) // stride[0] + 1
    ow = (iw + 2 * pad[1] - dil[1] * (kw - 1) - 1) // stride[1] + 1
    return oh, ow


def _hw(v):
    v = list(v) if isinstance(v, (list, tuple)) else [v]
    return (v[0], v[0]) if len(v) == 1 else (v[0], v[1])


def conv2d(x, w, bias=None, stride=1, padding=0, dilation=1, groups=1, act=ACT_NONE,
           out_min=-np.inf, out_max=np.inf, mode="exact", clamp_op=False, bug_tile32=False):
    """Forward convolution NCHW / OIHW (aten.convolution, et_vk.conv_with_clamp).

    clamp_op=True selects the et_vk.conv_with_clamp kernel family (its
    single-output-channel 1x1 kernel and the clamp epilogue)."""
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w.astype(x.dtype))
    s, p, d = _hw(stride), _hw(padding), _hw(dilation)
    B, IC, IH, IW = x.shape
    OC, icpg, KH, KW = w.shape
    OH, OW = conv_out_hw(IH, IW, KH, KW, s, p, d)
    prm = ConvParams(B, IC, IH, IW, OC, OH, OW, KH, KW, s[0], s[1], p[0], p[1], d[0], d[1],
                     groups, int(bias is not None), _dt(x), act, float(out_min), float(out_max))
    out = np.empty((B, OC, OH, OW), dtype=x.dtype)
    bb = np.ascontiguousarray(bias.astype(x.dtype)) if bias is not None else None
    _lib.oracle_conv2d(_mode(mode), int(clamp_op), ctypes.byref(prm), _ptr(x), _ptr(w), _ptr(bb),
                       _ptr(out), int(bug_tile32))
    return out


def conv_transpose2d(x, w, bias=None, stride=1, padding=0, dilation=1, output_padding=0,
                     groups=1, mode="exact"):
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w.astype(x.dtype))
    s, p, d, op = _hw(stride), _hw(padding), _hw(dilation), _hw(output_padding)
    B, IC, IH, IW = x.shape
    _, ocpg, KH, KW = w.shape
    OC = ocpg * groups
    OH = (IH - 1) * s[0] - 2 * p[0] + d[0] * (KH - 1) + op[0] + 1
    OW = (IW - 1) * s[1] - 2 * p[1] + d[1] * (KW - 1) + op[1] + 1
    prm = ConvParams(B, IC, IH, IW, OC, OH, OW, KH, KW, s[0], s[1], p[0], p[1], d[0], d[1],
                     groups, int(bias is not None), _dt(x), 0, -np.inf, np.inf)
    out = np.empty((B, OC, OH, OW), dtype=x.dtype)
    bb = np.ascontiguousarray(bias.astype(x.dtype)) if bias is not None else None
    _lib.oracle_conv_transpose2d(_mode(mode), ctypes.byref(prm), _ptr(x), _ptr(w), _ptr(bb),
                                 _ptr(out))
    return out


# ------------------------------------------------------------ elementwise
def add(a, b, alpha=1.0):
    """aten.add.Tensor: in1 + f16(alpha) * in2 (add-elementwise-f16.wgsl.ts:30)."""
    dt = a.dtype
    return (a + dt.type(alpha) * b).astype(dt)


def sub(a, b, alpha=1.0):
    dt = a.dtype
    return (a - dt.type(alpha) * b).astype(dt)


def mul(a, b):
    return (a * b).astype(a.dtype)


def sigmoid(x):
    """1 / (1 + exp(-x)) in the storage type (sigmoid-f16.wgsl.ts:28)."""
    dt = x.dtype
    e = np.exp(-x.astype(np.float32)).astype(dt)
    return (dt.type(1) / (dt.type(1) + e)).astype(dt)


def relu(x):
    return np.maximum(x, x.dtype.type(0))


def hardswish(x):
    dt = x.dtype.type
    return (np.clip(x + dt(3), dt(0), dt(6)) * x / dt(6)).astype(x.dtype)


def silu_exact(v):
    v = v.astype(np.float64)
    return v / (1.0 + np.exp(-v))


# ---------------------------------------------------------------- inputs
def make_inputs(shapes, seed=0, dist="normal", dtype=np.float16, scale=None):
    """Seeded synthetic tensors (numpy PCG64): one array per shape, rounded
    to ``dtype`` (round-to-nearest-even)."""
    rng = np.random.default_rng(seed)
    out = []
    for i, shp in enumerate(shapes):
        d = dist[i] if isinstance(dist, (list, tuple)) else dist
        sc = scale[i] if isinstance(scale, (list, tuple)) else (scale or 1.0)
        if d == "normal":
            v = rng.standard_normal(shp, dtype=np.float32) * sc
        elif d == "uniform":  # U(-1, 1)
            v = rng.uniform(-1.0, 1.0, size=shp).astype(np.float32) * sc
        elif d == "uniform01":
            v = rng.uniform(0.0, 1.0, size=shp).astype(np.float32) * sc
        else:
            raise ValueError(d)
        out.append(v.astype(dtype))
    return out


def rel_err(y, ref):
    """max|y - ref| / max|ref| (the tolerance metric of the parity tests)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref)) / (den if den > 0 else 1.0))
