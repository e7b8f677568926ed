"""The reference's known-answer tests for the hot path, as data.

Each case restates the inputs of one test of barhanc/wgpu-executorch
(tests/shaders/mm.test.ts, convolution.test.ts, conv-with-clamp.test.ts,
tests/api/program.test.ts; file:line given per case) and checks the result
the same way that test does. Literal expected arrays come from
tests/golden/reference_kats.json (extracted from those files by
tests/golden/make_golden.py); computed expectations (the JS CPU references
inside the tests) are restated here in float64.

A case runs either on the CPU oracle (``run_oracle``) or on the engine
through the wgx API (``run_engine(ctx)``), with the same ``check``.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))


def literal(file_key: str, title_prefix: str, which: int = 0):
    for title, c in KATS["files"][file_key]["cases"].items():
        if title.startswith(title_prefix):
            e = c["expectTensorClose"][which]
            return np.array(e["expected"], dtype=np.float64), e["tolerance"]
    raise KeyError(title_prefix)


@dataclass
class Case:
    name: str
    ref: str  # reference test file:line
    op: str  # 'mm' | 'conv' | 'clamp' | 'convT'
    inputs: Dict[str, Any]
    params: Dict[str, Any] = field(default_factory=dict)
    check: Callable[[np.ndarray], None] = None


def close(expected, tol):
    expected = np.asarray(expected, dtype=np.float64).reshape(-1)

    def chk(actual):
        a = np.asarray(actual, dtype=np.float64).reshape(-1)
        assert a.shape == expected.shape, (a.shape, expected.shape)
        assert np.all(np.isfinite(a)), "non-finite output"
        diff = np.abs(a - expected)
        i = int(np.argmax(diff))
        assert diff[i] <= tol, f"mismatch at {i}: got {a[i]}, expected {expected[i]} (tol {tol})"
    return chk


def elementwise_lt(expected, tol):
    expected = np.asarray(expected, dtype=np.float64).reshape(-1)

    def chk(actual):
        a = np.asarray(actual, dtype=np.float64).reshape(-1)
        assert np.all(np.abs(a - expected) < tol), float(np.max(np.abs(a - expected)))
    return chk


def close_digits(index, value, digits):
    # vitest toBeCloseTo(v, d): |a - v| < 10^-d / 2
    def chk(actual):
        a = float(np.asarray(actual, dtype=np.float64).reshape(-1)[index])
        assert abs(a - value) < 10.0 ** (-digits) / 2, (a, value)
    return chk


def bounds(lo, hi):
    def chk(actual):
        a = np.asarray(actual, dtype=np.float64)
        assert np.all(a >= lo) and np.all(a <= hi), (a.min(), a.max())
    return chk


def _mm_js(a, b):
    return a.astype(np.float64) @ b.astype(np.float64)


def cases() -> List[Case]:
    C: List[Case] = []
    f32, f16 = np.float32, np.float16

    # ---------------------------------------------------------------- mm
    a = np.array([1, 2, 3, 4], f32).reshape(2, 2)
    b = np.array([5, 6, 7, 8], f32).reshape(2, 2)
    exp, tol = literal("mm", "multiplies 2x2 matrices")
    C.append(Case("mm_2x2", "tests/shaders/mm.test.ts:6", "mm", {"a": a, "b": b},
                  check=close(exp, tol)))
    for n, tol in ((64, 1e-3), (128, 1e-2)):
        i = np.arange(n * n)
        a = ((i % 7) - 3).astype(f32).reshape(n, n)
        b = ((i % 5) - 2).astype(f32).reshape(n, n)
        C.append(Case(f"mm_{n}x{n}", "tests/shaders/mm.test.ts:24" if n == 64 else
                      "tests/shaders/mm.test.ts:64", "mm", {"a": a, "b": b},
                      check=elementwise_lt(_mm_js(a, b), tol)))
    a = np.array([1, 2, 3, 4], f16).reshape(2, 2)
    b = np.array([5, 6, 7, 8], f16).reshape(2, 2)
    C.append(Case("mm_f16_2x2", "tests/shaders/mm.test.ts:103", "mm", {"a": a, "b": b},
                  check=lambda y: [close_digits(k, v, 1)(y) for k, v in
                                   enumerate([19, 22, 43, 50])]))
    i = np.arange(64 * 64)
    a = ((i % 7) - 3).astype(f16).reshape(64, 64)
    b = ((i % 5) - 2).astype(f16).reshape(64, 64)
    # the JS reference stores its f64 sums into a Float16Array
    C.append(Case("mm_f16_64x64", "tests/shaders/mm.test.ts:124", "mm", {"a": a, "b": b},
                  check=elementwise_lt(_mm_js(a, b).astype(f16), 0.5)))
    a = ((np.arange(35) % 5) - 2).astype(f32).reshape(5, 7)
    b = ((np.arange(21) % 3) + 1).astype(f32).reshape(7, 3)
    C.append(Case("mm_5x7x3", "tests/shaders/mm.test.ts:164", "mm", {"a": a, "b": b},
                  check=close(_mm_js(a, b), 1e-4)))

    # ------------------------------------------------------- convolution
    def conv(name, ref, x, w, bias, stride, pad, dil, groups, chk, op="conv", **extra):
        p = dict(stride=stride, padding=pad, dilation=dil, groups=groups)
        p.update(extra)
        C.append(Case(name, ref, op, {"x": x, "w": w, "bias": bias}, p, chk))

    x = np.arange(1, 10, dtype=f32).reshape(1, 1, 3, 3)
    w = np.array([1, 0, 0, 1], f32).reshape(1, 1, 2, 2)
    exp, tol = literal("convolution", "computes 2D dense convolution with bias")
    conv("conv_dense_bias", "tests/shaders/convolution.test.ts:6", x, w,
         np.array([10], f32), [1, 1], [0, 0], [1, 1], 1, close(exp, tol))
    x = np.array([1, 2, 3, 4, 10, 20, 30, 40], f32).reshape(1, 2, 2, 2)
    w = np.array([1, 1, 1, 1, 1, 0, 0, 1], f32).reshape(2, 1, 2, 2)
    exp, tol = literal("convolution", "computes depthwise grouped 2D convolution")
    conv("conv_depthwise", "tests/shaders/convolution.test.ts:47", x, w, None, [1, 1], [0, 0],
         [1, 1], 2, close(exp, tol))
    x = np.array([1, 2, 3, 4], f32).reshape(1, 1, 2, 2)
    w = np.ones((1, 1, 2, 2), f32)
    exp, tol = literal("convolution", "computes transposed 2D convolution")
    conv("convT_box", "tests/shaders/convolution.test.ts:94", x, w, None, [2, 2], [0, 0],
         [1, 1], 1, close(exp, tol), op="convT", output_padding=[0, 0])
    x = np.arange(1, 51, dtype=f32).reshape(1, 2, 5, 5)
    w = (np.arange(54, dtype=f32) + 1) * f32(0.1)
    w = w.reshape(3, 2, 3, 3)
    exp, tol = literal("convolution", "computes non-trivial multi-channel conv2d")
    conv("conv_multi_s2p1", "tests/shaders/convolution.test.ts:132", x, w,
         np.array([2.5, -1.0, 0.5], f32), [2, 2], [1, 1], [1, 1], 1, close(exp, tol))
    x = np.arange(1, 19, dtype=f32).reshape(1, 2, 3, 3)
    w = ((np.arange(36, dtype=f32) + 1) * f32(0.05)).reshape(2, 2, 3, 3)
    exp, tol = literal("convolution", "computes non-trivial multi-channel conv_transpose2d")
    # the JS literals are rounded to a few decimals; 1e-5 absolute is the
    # reference's own tolerance
    conv("convT_multi_s2p1op1", "tests/shaders/convolution.test.ts:178", x, w,
         np.array([1.5, -2.0], f32), [2, 2], [1, 1], [1, 1], 1, close(exp, max(tol, 2e-5)),
         op="convT", output_padding=[1, 1])
    x = np.arange(1, 10, dtype=f16).reshape(1, 1, 3, 3)
    w = np.array([1, 0, 0, 1], f16).reshape(1, 1, 2, 2)
    exp, tol = literal("convolution", "computes float16 2D dense convolution with bias")
    conv("conv_f16_dense_bias", "tests/shaders/convolution.test.ts:227", x, w,
         np.array([10], f16), [1, 1], [0, 0], [1, 1], 1, close(exp, tol))
    i = np.arange(64 * 64)
    x = (((np.arange(64 * 8 * 8) % 5) - 2) * 0.5).astype(f16).reshape(1, 64, 8, 8)
    w = (((np.arange(64 * 64) % 7) - 3) * 0.25).astype(f16).reshape(64, 64, 1, 1)
    e00 = float(np.sum(x[0, :, 0, 0].astype(np.float64) * w[0, :, 0, 0].astype(np.float64)))
    conv("conv_f16_1x1_64x64", "tests/shaders/convolution.test.ts:258", x, w, None, [1, 1],
         [0, 0], [1, 1], 1, close_digits(0, e00, 1))
    x = np.array([1, 2, 3, 4, 10, 20, 30, 40], f16).reshape(1, 2, 2, 2)
    w = np.array([2, 0.5], f16).reshape(2, 1, 1, 1)
    exp, tol = literal("convolution", "computes float16 depthwise convolution")
    conv("conv_f16_depthwise", "tests/shaders/convolution.test.ts:308", x, w, None, [1, 1],
         [0, 0], [1, 1], 2, close(exp, tol))
    x = np.arange(1, 17, dtype=f32).reshape(1, 4, 2, 2)
    w = (np.eye(4, dtype=f32) * 2).reshape(4, 4, 1, 1)
    conv("conv_1x1_vec4", "tests/shaders/convolution.test.ts:338", x, w, None, [1, 1], [0, 0],
         [1, 1], 1, elementwise_lt(x.astype(np.float64) * 2, 5e-5))
    x = ((np.arange(16 * 64) % 13) * 0.1).astype(f32).reshape(1, 16, 8, 8)
    w = ((np.arange(64 * 16) % 7) * 0.1).astype(f32).reshape(64, 16, 1, 1)
    e0 = float(np.sum(x[0, :, 0, 0].astype(np.float64) * w[0, :, 0, 0].astype(np.float64)))
    conv("conv_1x1_64x64", "tests/shaders/convolution.test.ts:382", x, w, None, [1, 1], [0, 0],
         [1, 1], 1, close_digits(0, e0, 3))
    x = np.ones((1, 4, 2, 2), f32)
    w = np.full((4, 2, 1, 1), 2, f32)
    conv("conv_grouped_g2", "tests/shaders/convolution.test.ts:422", x, w, None, [1, 1], [0, 0],
         [1, 1], 2, close(np.full(16, 4.0), 1e-3))

    # --------------------------------------------------- conv_with_clamp
    for dt in (f32, f16):
        for has_bias in (False, True):
            spatial = 260
            vals = ((np.arange(2 * 3 * spatial) % 13) - 6).astype(dt)
            x = vals.reshape(2, 3, 1, spatial)
            w = np.array([1, -2, 0.5], dt).reshape(1, 3, 1, 1)
            v = vals.astype(np.float64).reshape(2, 3, spatial)
            e = v[:, 0] - 2 * v[:, 1] + 0.5 * v[:, 2] + (3 if has_bias else 0)
            e = np.minimum(10, np.maximum(-5, e)).reshape(-1)
            conv(f"clamp_single_{np.dtype(dt).name}_bias{int(has_bias)}",
                 "tests/shaders/conv-with-clamp.test.ts:8", x, w,
                 np.array([3], dt) if has_bias else None, [1, 1], [0, 0], [1, 1], 1,
                 close(e, 1e-5), op="clamp", out_min=-5, out_max=10)
    x = np.array([60000, 60000, -60000, -60000, -60000, -60000, 60000, 60000, 4, 60000, -4,
                  -60000], f16).reshape(1, 3, 1, 4)
    w = np.array([2, 2, 2], f16).reshape(1, 3, 1, 1)
    exp, tol = literal("conv_with_clamp", "widens FP16 pointwise products")
    conv("clamp_f16_widening", "tests/shaders/conv-with-clamp.test.ts:57", x, w, None, [1, 1],
         [0, 0], [1, 1], 1, close(exp, tol), op="clamp", out_min=-100, out_max=100)
    x = np.arange(1, 10, dtype=f32).reshape(1, 1, 3, 3)
    w = np.array([1, 0, 0, 1], f32).reshape(1, 1, 2, 2)
    exp, tol = literal("conv_with_clamp", "computes 2D dense convolution with clamp and bias")
    conv("clamp_dense_bias", "tests/shaders/conv-with-clamp.test.ts:92", x, w,
         np.array([10], f32), [1, 1], [0, 0], [1, 1], 1, close(exp, tol), op="clamp",
         out_min=17.0, out_max=23.0)
    x = np.array([-5, -2, 1, 2, 2, 4, 1, 3], f32).reshape(1, 2, 2, 2)
    w = np.ones((2, 1, 2, 2), f32)
    exp, tol = literal("conv_with_clamp", "computes depthwise grouped convolution with clamp")
    conv("clamp_depthwise_relu6", "tests/shaders/conv-with-clamp.test.ts:133", x, w, None,
         [1, 1], [0, 0], [1, 1], 2, close(exp, tol), op="clamp", out_min=0.0, out_max=6.0)
    x = np.arange(1, 10, dtype=f16).reshape(1, 1, 3, 3)
    w = np.array([1, 0, 0, 1], f16).reshape(1, 1, 2, 2)
    exp, tol = literal("conv_with_clamp", "computes float16 2D dense convolution with clamp")
    conv("clamp_f16_dense_bias", "tests/shaders/conv-with-clamp.test.ts:183", x, w,
         np.array([10], f16), [1, 1], [0, 0], [1, 1], 1, close(exp, tol), op="clamp",
         out_min=17.0, out_max=23.0)
    x = (((np.arange(64 * 64) % 5) - 2) * 0.5).astype(f16).reshape(1, 64, 8, 8)
    w = (((np.arange(64 * 64) % 7) - 3) * 0.25).astype(f16).reshape(64, 64, 1, 1)
    conv("clamp_f16_64x64_bounds", "tests/shaders/conv-with-clamp.test.ts:216", x, w, None,
         [1, 1], [0, 0], [1, 1], 1, bounds(-1.01, 1.01), op="clamp", out_min=-1.0, out_max=1.0)
    x = np.array([-5, -2, 1, 2, 2, 4, 1, 3], f16).reshape(1, 2, 2, 2)
    w = np.ones((2, 1, 2, 2), f16)
    exp, tol = literal("conv_with_clamp", "computes float16 depthwise grouped convolution")
    conv("clamp_f16_depthwise", "tests/shaders/conv-with-clamp.test.ts:263", x, w, None, [1, 1],
         [0, 0], [1, 1], 2, close(exp, tol), op="clamp", out_min=0.0, out_max=6.0)
    x = ((np.arange(16 * 64) % 13) * 0.5 - 2.0).astype(f32).reshape(1, 16, 8, 8)
    w = ((np.arange(64 * 16) % 7) * 0.1).astype(f32).reshape(64, 16, 1, 1)
    conv("clamp_1x1_64x64_bounds", "tests/shaders/conv-with-clamp.test.ts:297", x, w, None,
         [1, 1], [0, 0], [1, 1], 1, bounds(0.0, 5.0001), op="clamp", out_min=0.0, out_max=5.0)
    return C


# ------------------------------------------------------------- runners
def run_oracle(case: Case, mode: str = "wgsl") -> np.ndarray:
    import oracle
    if case.op == "mm":
        return oracle.mm(case.inputs["a"], case.inputs["b"], mode=mode)
    x, w, b = case.inputs["x"], case.inputs["w"], case.inputs["bias"]
    p = case.params
    if case.op == "convT":
        return oracle.conv_transpose2d(x, w, b, p["stride"], p["padding"], p["dilation"],
                                       p["output_padding"], p["groups"], mode=mode)
    if case.op == "clamp":
        return oracle.conv2d(x, w, b, p["stride"], p["padding"], p["dilation"], p["groups"],
                             act=oracle.ACT_CLAMP, out_min=p["out_min"], out_max=p["out_max"],
                             mode=mode, clamp_op=True)
    return oracle.conv2d(x, w, b, p["stride"], p["padding"], p["dilation"], p["groups"], mode=mode)


def _dtname(a):
    return {np.dtype(np.float32): "float32", np.dtype(np.float16): "float16"}[a.dtype]


def run_engine(ctx, case: Case) -> np.ndarray:
    """Drives the engine exactly like the reference test: tensors, setData,
    recordShader, submit, sync, getData."""
    import wgx
    from oracle_shapes import conv_out_shape, convT_out_shape
    if case.op == "mm":
        a, b = case.inputs["a"], case.inputs["b"]
        ta = ctx.tensor(_dtname(a), a.shape).setData(a)
        tb = ctx.tensor(_dtname(b), b.shape).setData(b)
        out = ctx.tensor(_dtname(a), [a.shape[0], b.shape[1]])
        ctx.recordShader(wgx.shaders.mm, [ta, tb, out])
        ctx.submit()
        ctx.sync()
        return out.numpy()
    x, w, b = case.inputs["x"], case.inputs["w"], case.inputs["bias"]
    p = case.params
    dt = _dtname(x)
    tx = ctx.tensor(dt, x.shape).setData(x)
    tw = ctx.tensor(dt, w.shape).setData(w)
    tb = ctx.tensor(dt, b.shape).setData(b) if b is not None else None
    if case.op == "convT":
        oshape = convT_out_shape(x.shape, w.shape, p)
        out = ctx.tensor(dt, oshape)
        ctx.recordShader(wgx.shaders.convolution,
                         [tx, tw, tb, p["stride"], p["padding"], p["dilation"], True,
                          p["output_padding"], p["groups"], out])
    else:
        oshape = conv_out_shape(x.shape, w.shape, p)
        out = ctx.tensor(dt, oshape)
        if case.op == "clamp":
            ctx.recordShader(wgx.shaders.convWithClamp,
                             [tx, tw, tb, p["stride"], p["padding"], p["dilation"], False,
                              [0, 0], p["groups"], p["out_min"], p["out_max"], out])
        else:
            ctx.recordShader(wgx.shaders.convolution,
                             [tx, tw, tb, p["stride"], p["padding"], p["dilation"], False,
                              [0, 0], p["groups"], out])
    ctx.submit()
    ctx.sync()
    return out.numpy()
