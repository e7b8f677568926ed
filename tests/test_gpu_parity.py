"""Parity of the B200 kernels with the CPU oracle on seeded inputs.

Tolerances (metric: max|y - ref| / max|ref|, ``oracle.rel_err``):
  * fp32 paths (FFMA, fp32 accumulation): <= 1e-4 against both the exact
    oracle and the reference's own fp32 arithmetic (north-star bound 1e-4).
  * fp16 paths (tcgen05 fp32 accumulation, one rounding to fp16):
    <= 2e-3 against the exact oracle (one fp16 rounding is 2^-11 of a value)
    and <= 2e-2 against the reference's f16-accumulating arithmetic
    (north-star bound 2e-2).
"""
import ctypes

import numpy as np
import pytest

import oracle
import wgx
from wgx import _lib

pytestmark = pytest.mark.gpu

F16_EXACT, F16_WGSL, F32_TOL = 2e-3, 2e-2, 1e-4


def dtname(a):
    return "float16" if a.dtype == np.float16 else "float32"


def engine_conv(ctx, x, w, b, stride, pad, dil, groups, clamp=None):
    dt = dtname(x)
    tx = ctx.tensor(dt, x.shape).setData(x)
    tw = ctx.tensor(dt, w.shape).setData(w)
    tb = ctx.tensor(dt, b.shape).setData(b) if b is not None else None
    B, IC, H, W = x.shape
    OC, _, KH, KW = w.shape
    OH, OW = oracle.conv_out_hw(H, W, KH, KW, (stride,) * 2 if np.isscalar(stride) else stride,
                                (pad,) * 2 if np.isscalar(pad) else pad,
                                (dil,) * 2 if np.isscalar(dil) else dil)
    out = ctx.tensor(dt, [B, OC, OH, OW])
    hw = lambda v: [v, v] if np.isscalar(v) else list(v)
    if clamp is None:
        ctx.recordShader(wgx.shaders.convolution,
                         [tx, tw, tb, hw(stride), hw(pad), hw(dil), False, [0, 0], groups, out])
    else:
        ctx.recordShader(wgx.shaders.convWithClamp,
                         [tx, tw, tb, hw(stride), hw(pad), hw(dil), False, [0, 0], groups,
                          clamp[0], clamp[1], out])
    ctx.submit()
    ctx.sync()
    res = out.numpy()
    ctx.reset()
    return res


def check_f16(y, x, w, b, stride, pad, dil, groups, act=oracle.ACT_NONE, lo=-np.inf, hi=np.inf,
              clamp_op=False):
    ex = oracle.conv2d(x, w, b, stride, pad, dil, groups, act=act, out_min=lo, out_max=hi,
                       mode="exact", clamp_op=clamp_op)
    e1 = oracle.rel_err(y, ex)
    assert np.all(np.isfinite(y.astype(np.float32)))
    tol = F16_EXACT
    if groups > 1 and groups == x.shape[1] == w.shape[0]:
        # fp16 depthwise accumulates its KH*KW products in f16, as the
        # reference's conv2d-depthwise-f16 kernel does: the running sum's
        # rounding error grows with the number of taps
        tol = F16_EXACT * max(1.0, w.shape[2] * w.shape[3] / 25.0)
    assert e1 <= tol, f"vs exact oracle: {e1}"
    if act != oracle.ACT_SILU:
        wg = oracle.conv2d(x, w, b, stride, pad, dil, groups, act=act, out_min=lo, out_max=hi,
                           mode="wgsl", clamp_op=clamp_op)
        e2 = oracle.rel_err(y, wg)
        assert e2 <= F16_WGSL, f"vs reference f16 arithmetic: {e2}"
    return e1


def kaiming(shape, seed, dtype=np.float16):
    fan_in = int(np.prod(shape[1:]))
    (w,) = oracle.make_inputs([shape], seed=seed, dtype=np.float32)
    return (w * np.sqrt(2.0 / fan_in)).astype(dtype)


# (B, IC, H, W, OC, KH, KW, pad, dil): stride-1 dense fp16 -> tensor-core path
DENSE_F16 = [
    (1, 64, 160, 160, 128, 3, 3, 1, 1),   # BASELINE config 2 geometry, one image
    (2, 8, 7, 9, 5, 3, 3, 1, 1),
    (1, 40, 13, 11, 130, 3, 3, 1, 1),     # two output-channel tiles, IC % 32 != 0
    (3, 32, 20, 20, 16, 1, 1, 0, 1),      # 1x1
    (1, 16, 9, 33, 64, 5, 5, 2, 1),
    (1, 24, 17, 17, 33, 7, 7, 3, 1),
    (2, 64, 10, 10, 32, 3, 3, 2, 2),      # dilation 2
    (1, 256, 20, 20, 256, 3, 3, 1, 1),
    (1, 8, 1, 600, 8, 1, 3, 0, 1),        # 1-row image, KH != KW
    (1, 96, 40, 40, 96, 3, 3, 1, 1),
    (8, 64, 48, 48, 192, 3, 3, 1, 1),     # streamed weights, >1 tile per CTA
    (3, 16, 30, 30, 24, 5, 3, 2, 1),      # KH != KW with padding
    # 1x1 / stride 1 / no padding: activations read from NCHW by TMA
    (2, 40, 16, 24, 96, 1, 1, 0, 1),      # IC % 32 != 0: zero-filled channel rows
    (3, 64, 20, 20, 200, 1, 1, 0, 1),     # two output-channel tiles
    (2, 16, 32, 32, 24, 1, 1, 0, 1),      # positions on M, 16-channel stages
    # OC <= 64: positions on the MMA M side (N = 16 / 32 / 64)
    (2, 64, 40, 40, 64, 3, 3, 1, 1),
    (2, 48, 33, 35, 17, 1, 1, 0, 1),
    (1, 32, 24, 40, 1, 1, 1, 0, 1),       # one output channel
    (2, 16, 26, 26, 8, 3, 3, 1, 1),       # 16-channel stages, 8 M blocks per tile
    (1, 96, 20, 20, 40, 5, 5, 2, 1),
    # planes of at most 512 positions: N = 16 / 32 tiles of 4 M blocks
    (2, 64, 20, 20, 16, 3, 3, 1, 1),
    (3, 32, 16, 16, 32, 3, 3, 1, 1),
    (2, 24, 12, 12, 8, 3, 3, 1, 1),
]


@pytest.mark.parametrize("geom", DENSE_F16, ids=[str(g) for g in DENSE_F16])
def test_dense_f16_tensor_core(ctx, geom):
    B, IC, H, W, OC, KH, KW, pad, dil = geom
    (x,) = oracle.make_inputs([(B, IC, H, W)], seed=10)
    w = kaiming((OC, IC, KH, KW), 11)
    (b,) = oracle.make_inputs([(OC,)], seed=12, scale=0.01)
    pads = (pad if KH > 1 else 0, pad if KW > 1 else 0) if KH != KW else (pad, pad)
    y = engine_conv(ctx, x, w, b, 1, pads, dil, 1)
    check_f16(y, x, w, b, 1, pads, dil, 1)


# (B, IC, H, W, OC, pad, dil): 3x3 / stride 1 convolutions whose filter
# columns are folded into the MMA's N (N = 3 * ocp: 32 / 48 / 96 / 192), with
# 16-byte NCHW stores (OW % 8 == 0 and a padded row pitch of 8k) or 2-byte ones
KW_FOLDED_F16 = [
    (2, 32, 9, 160, 8, (1, 1), (1, 1)),      # N = 32, 8 M blocks, vector stores
    (2, 48, 13, 17, 16, (1, 1), (1, 1)),     # N = 48, odd sizes
    (1, 64, 30, 30, 24, (1, 1), (1, 1)),     # N = 96 (24 channels of 32)
    (1, 80, 9, 40, 40, (1, 1), (1, 1)),      # N = 192, one M block per tile
    (1, 32, 12, 20, 8, (2, 1), (2, 1)),      # vertical dilation
    (3, 256, 20, 20, 16, (1, 1), (1, 1)),    # YOLO26-N neck shape
    (2, 64, 20, 20, 64, (1, 1), (1, 1)),     # small plane: folded at ocp = 16 * ceil(IC/16)
    (1, 16, 5, 3, 5, (1, 1), (1, 1)),        # planes narrower than the filter rows
]


@pytest.mark.parametrize("geom", KW_FOLDED_F16, ids=[str(g) for g in KW_FOLDED_F16])
@pytest.mark.parametrize("bias", [True, False])
def test_kw_folded_f16(ctx, geom, bias):
    B, IC, H, W, OC, pad, dil = geom
    p = _lib.ConvParams(B, IC, H, W, OC, H + 2 * pad[0] - 2 * dil[0], W + 2 * pad[1] - 2 * dil[1],
                        3, 3, 1, 1, pad[0], pad[1], dil[0], dil[1], 1, int(bias), 1,
                        _lib.ACT_NONE, -np.inf, np.inf)
    buf = ctypes.create_string_buffer(256)
    _lib.check(_lib.lib.wgx_conv2d_describe(ctypes.byref(p), buf, 256))
    assert "kw-folded" in buf.value.decode(), buf.value
    (x,) = oracle.make_inputs([(B, IC, H, W)], seed=30)
    w = kaiming((OC, IC, 3, 3), 31)
    b = oracle.make_inputs([(OC,)], seed=32, scale=0.01)[0] if bias else None
    y = engine_conv(ctx, x, w, b, 1, pad, dil, 1)
    check_f16(y, x, w, b, 1, pad, dil, 1)


def test_dense_f16_no_bias_and_clamp(ctx):
    (x,) = oracle.make_inputs([(2, 48, 15, 17)], seed=20)
    w = kaiming((40, 48, 3, 3), 21)
    y = engine_conv(ctx, x, w, None, 1, 1, 1, 1)
    check_f16(y, x, w, None, 1, 1, 1, 1)
    y = engine_conv(ctx, x, w, None, 1, 1, 1, 1, clamp=(0.0, float(np.finfo(np.float64).max)))
    check_f16(y, x, w, None, 1, 1, 1, 1, act=oracle.ACT_CLAMP, lo=0.0, hi=np.inf, clamp_op=True)


# strided convolutions on the tensor cores (space-to-depth re-layout):
# (B, IC, H, W, OC, K, stride, pad)
STRIDED_F16 = [
    (1, 3, 64, 64, 16, 3, 2, 1),      # YOLO stem shape (IC = 3: 12 virtual channels)
    (2, 5, 32, 40, 24, 3, 2, 1),      # few channels, vectorised re-layout (20 virtual)
    (1, 2, 24, 24, 16, 3, 2, 0),      # 8 virtual channels, no padding
    (2, 16, 40, 40, 32, 3, 2, 1),     # vectorised re-layout (IC % 8 == 0, W % 8 == 0)
    (2, 32, 21, 19, 64, 3, 2, 1),     # odd sizes: per-slot re-layout
    (1, 64, 48, 48, 160, 3, 2, 1),    # two output-channel tiles
    (2, 32, 20, 24, 48, 5, 2, 2),     # 5x5 -> 3x3 virtual filter
    (1, 16, 30, 30, 32, 1, 2, 0),     # 1x1 stride 2: one input phase
    (1, 16, 33, 33, 24, 3, 2, 0),     # no padding
    (1, 8, 28, 28, 16, 7, 2, 3),      # 7x7 -> 4x4 virtual filter
    (1, 16, 27, 27, 16, 3, 3, 1),     # stride 3
    (2, 128, 80, 80, 128, 3, 2, 1),   # YOLO26-N downsampling shape
]


@pytest.mark.parametrize("geom", STRIDED_F16, ids=[str(g) for g in STRIDED_F16])
def test_strided_f16_tensor_core(ctx, geom):
    B, IC, H, W, OC, K, s, p = geom
    OH, OW = oracle.conv_out_hw(H, W, K, K, (s, s), (p, p), (1, 1))
    params = _lib.ConvParams(B, IC, H, W, OC, OH, OW, K, K, s, s, p, p, 1, 1, 1, 1, 1,
                             _lib.ACT_NONE, -np.inf, np.inf)
    plan = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(params), ctypes.byref(plan)))
    assert plan.variant == _lib.CONV_UMMA
    (x,) = oracle.make_inputs([(B, IC, H, W)], seed=35)
    w = kaiming((OC, IC, K, K), 36)
    (b,) = oracle.make_inputs([(OC,)], seed=37, scale=0.01)
    y = engine_conv(ctx, x, w, b, s, p, 1, 1)
    check_f16(y, x, w, b, s, p, 1, 1)


def test_strided_f16_without_bias(ctx):
    """A stride-2 tensor-core convolution with no bias tensor."""
    (x,) = oracle.make_inputs([(2, 32, 40, 40)], seed=38)
    w = kaiming((64, 32, 3, 3), 39)
    tx = ctx.tensor("float16", x.shape).setData(x)
    tw = ctx.tensor("float16", w.shape).setData(w)
    out = ctx.tensor("float16", [2, 64, 20, 20])
    ctx.recordShader(wgx.shaders.convolution,
                     [tx, tw, None, [2, 2], [1, 1], [1, 1], False, [0, 0], 1, out])
    ctx.submit()
    ctx.sync()
    check_f16(out.numpy(), x, w, None, 2, 1, 1, 1)
    ctx.reset()


@pytest.mark.parametrize("geom", [
    (1, 1, 33, 35, 8, 3, 2, 1),      # stride 2 with IC = 1 (4 virtual channels < 8)
    (1, 5, 7, 7, 3, 3, 1, 1),        # IC < 8
    (1, 16, 20, 20, 16, 3, 5, 1),    # stride 5
])
def test_dense_f16_cuda_core_fallback(ctx, geom):
    B, IC, H, W, OC, K, s, p = geom
    (x,) = oracle.make_inputs([(B, IC, H, W)], seed=30)
    w = kaiming((OC, IC, K, K), 31)
    (b,) = oracle.make_inputs([(OC,)], seed=32, scale=0.01)
    y = engine_conv(ctx, x, w, b, s, p, 1, 1)
    check_f16(y, x, w, b, s, p, 1, 1)


@pytest.mark.parametrize("geom", [
    (1, 256, 80, 80, 5, 1, 2, 1),    # BASELINE config 3 depthwise, one image
    (2, 80, 80, 80, 3, 1, 1, 1),     # YOLO shapes: one plane per CTA
    (3, 64, 40, 40, 3, 1, 1, 1),     # several planes per CTA
    (2, 24, 20, 20, 7, 1, 3, 1),
    (1, 8, 300, 300, 3, 1, 1, 1),    # banded plane
    (2, 5, 13, 21, 5, 1, 2, 1),      # unaligned rows: per-element staging
    (1, 6, 17, 16, 3, 1, 0, 1),      # no padding
    (2, 8, 9, 13, 3, 2, 1, 1),
    (1, 16, 33, 31, 7, 1, 3, 1),
    (1, 12, 24, 24, 3, 1, 2, 2),
    (3, 32, 40, 40, 3, 1, 1, 1),
    (1, 4, 224, 224, 3, 2, 1, 1),
    (2, 16, 24, 32, 7, 1, 3, 1),     # fp16 sliding-window kernel, K = 7
    (1, 4, 160, 320, 3, 1, 1, 1),    # sliding-window kernel in row bands
    (3, 5, 16, 40, 5, 1, 2, 1),      # planes that do not fill a CTA
    (3, 40, 16, 16, 3, 2, 1, 1),     # strided, many small planes per CTA (DepthART shapes)
    (2, 24, 32, 32, 5, 2, 2, 1),
])
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_depthwise(ctx, geom, dtype):
    B, C, H, W, K, s, p, d = geom
    (x,) = oracle.make_inputs([(B, C, H, W)], seed=40, dtype=dtype)
    (w, b) = oracle.make_inputs([(C, 1, K, K), (C,)], seed=41, scale=[0.1, 0.01], dtype=dtype)
    y = engine_conv(ctx, x, w, b, s, p, d, C)
    if dtype == np.float16:
        check_f16(y, x, w, b, s, p, d, C)
    else:
        ex = oracle.conv2d(x, w, b, s, p, d, C, mode="exact")
        assert oracle.rel_err(y, ex) <= F32_TOL
        assert oracle.rel_err(y, oracle.conv2d(x, w, b, s, p, d, C, mode="wgsl")) <= F32_TOL


def test_depthwise_relu6_clamp(ctx):
    (x,) = oracle.make_inputs([(2, 24, 28, 28)], seed=42)
    (w, b) = oracle.make_inputs([(24, 1, 3, 3), (24,)], seed=43, scale=[0.5, 0.1])
    y = engine_conv(ctx, x, w, b, 1, 1, 1, 24, clamp=(0.0, 6.0))
    check_f16(y, x, w, b, 1, 1, 1, 24, act=oracle.ACT_CLAMP, lo=0.0, hi=6.0, clamp_op=True)


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_grouped_direct(ctx, dtype):
    (x, w, b) = oracle.make_inputs([(2, 8, 11, 9), (6, 4, 3, 3), (6,)], seed=50, dtype=dtype)
    y = engine_conv(ctx, x, w, b, 1, 1, 1, 2)
    ex = oracle.conv2d(x, w, b, 1, 1, 1, 2, mode="exact")
    tol = F16_EXACT if dtype == np.float16 else F32_TOL
    assert oracle.rel_err(y, ex) <= tol


@pytest.mark.parametrize("geom", [(2, 16, 8, 8, 3), (1, 64, 12, 12, 5), (2, 3, 9, 9, 4)])
@pytest.mark.parametrize("dtype", [np.float32])
def test_fp32_dense(ctx, geom, dtype):
    B, IC, H, W, OC = geom
    (x, w, b) = oracle.make_inputs([(B, IC, H, W), (OC, IC, 3, 3), (OC,)], seed=60, dtype=dtype)
    y = engine_conv(ctx, x, w, b, 1, 1, 1, 1)
    assert oracle.rel_err(y, oracle.conv2d(x, w, b, 1, 1, 1, 1, mode="exact")) <= F32_TOL
    assert oracle.rel_err(y, oracle.conv2d(x, w, b, 1, 1, 1, 1, mode="wgsl")) <= F32_TOL


def test_single_channel_pointwise_f16(ctx):
    (x, w, b) = oracle.make_inputs([(3, 24, 20, 28), (1, 24, 1, 1), (1,)], seed=70)
    y = engine_conv(ctx, x, w, b, 1, 0, 1, 1, clamp=(-1.0, 1.0))
    check_f16(y, x, w, b, 1, 0, 1, 1, act=oracle.ACT_CLAMP, lo=-1.0, hi=1.0, clamp_op=True)


# ------------------------------------------------------------------ mm
def engine_mm(ctx, a, b):
    dt = dtname(a)
    ta = ctx.tensor(dt, a.shape).setData(a)
    tb = ctx.tensor(dt, b.shape).setData(b)
    out = ctx.tensor(dt, [a.shape[0], b.shape[1]])
    ctx.recordShader(wgx.shaders.mm, [ta, tb, out])
    ctx.submit()
    ctx.sync()
    r = out.numpy()
    ctx.reset()
    return r


def test_mm_fp32_config1(ctx):
    # A[512,512] @ B[512,512], U(-1,1), seed 0
    a, b = oracle.make_inputs([(512, 512), (512, 512)], seed=0, dist="uniform", dtype=np.float32)
    y = engine_mm(ctx, a, b)
    assert oracle.rel_err(y, oracle.mm(a, b, "exact")) <= F32_TOL
    assert oracle.rel_err(y, oracle.mm(a, b, "wgsl")) <= F32_TOL


@pytest.mark.parametrize("mkn", [
    (64, 4096, 64),     # one tile: K split over a cluster of 8 CTAs
    (100, 300, 72),     # K % 4 == 0, N % 4 == 0, partial tiles
    (1000, 129, 515),   # K and N not multiples of 4: scalar loads
    (7, 1000, 9),
    (640, 64, 640),     # 100 tiles, K too short to split
    (1, 2048, 1),
])
def test_mm_fp32_shapes(ctx, mkn):
    """The split-K cluster FFMA kernel against both oracle modes."""
    M, K, N = mkn
    a, b = oracle.make_inputs([(M, K), (K, N)], seed=81, dist="uniform", dtype=np.float32)
    y = engine_mm(ctx, a, b)
    assert oracle.rel_err(y, oracle.mm(a, b, "exact")) <= F32_TOL
    assert oracle.rel_err(y, oracle.mm(a, b, "wgsl")) <= F32_TOL


@pytest.mark.parametrize("mkn", [
    (1024, 512, 1024),  # 64 tiles, K split over clusters of 2
    (768, 1024, 768),   # 36 tiles, K split over clusters of 4
    (2048, 256, 1024),  # 128 tiles, K not split (8 rounds of 32 in one CTA)
    (512, 4096, 512),   # 16 tiles, K split over clusters of 4, 32 rounds each
])
@pytest.mark.parametrize("scale", [1.0, 1e3])
def test_mm_fp32_tensor_core(ctx, mkn, scale):
    """fp32 mm on tcgen05 (3xTF32: TF32 heads and fp32 tails of both
    operands; products of at least 2^29 multiply-adds take this path)
    against both oracle modes at the fp32 bound, with inputs spanning six
    orders of magnitude."""
    M, K, N = mkn
    a, b = oracle.make_inputs([(M, K), (K, N)], seed=82, dist="uniform", dtype=np.float32)
    a = (a * scale).astype(np.float32)
    b[:, ::3] *= 1e-3  # columns of mixed magnitude
    y = engine_mm(ctx, a, b)
    assert oracle.rel_err(y, oracle.mm(a, b, "exact")) <= F32_TOL
    assert oracle.rel_err(y, oracle.mm(a, b, "wgsl")) <= F32_TOL


def test_mm_fp32_tensor_core_first_call(tmp_path):
    """The tensor-core fp32 mm as the first call of a fresh process, on a
    shape whose K is not split (every per-device set-up must happen on that
    path too): the result against the exact oracle."""
    import os
    import subprocess
    import sys
    M, K, N = 2048, 256, 1024
    a, b = oracle.make_inputs([(M, K), (K, N)], seed=83, dist="uniform", dtype=np.float32)
    np.save(tmp_path / "a.npy", a)
    np.save(tmp_path / "b.npy", b)
    script = (
        "import sys, numpy as np; sys.path.insert(0, %r); import wgx\n"
        "ctx = wgx.WgpuExecutionContext(0)\n"
        "a = np.load(%r); b = np.load(%r)\n"
        "ta = ctx.tensor('float32', a.shape).setData(a)\n"
        "tb = ctx.tensor('float32', b.shape).setData(b)\n"
        "out = ctx.tensor('float32', [a.shape[0], b.shape[1]])\n"
        "ctx.recordShader(wgx.shaders.mm, [ta, tb, out]); ctx.submit(); ctx.sync()\n"
        "np.save(%r, out.numpy())\n"
    ) % (os.path.dirname(os.path.dirname(os.path.abspath(wgx.__file__))), str(tmp_path / "a.npy"),
         str(tmp_path / "b.npy"), str(tmp_path / "y.npy"))
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    y = np.load(tmp_path / "y.npy")
    assert oracle.rel_err(y, oracle.mm(a, b, "exact")) <= F32_TOL


@pytest.mark.parametrize("mkn", [(512, 512, 512), (100, 72, 300), (64, 8, 1000), (300, 200, 7),
                                 (257, 1024, 129), (5, 7, 3)])
def test_mm_fp16(ctx, mkn):
    M, K, N = mkn
    a, b = oracle.make_inputs([(M, K), (K, N)], seed=80, dist="uniform")
    y = engine_mm(ctx, a, b)
    assert oracle.rel_err(y, oracle.mm(a, b, "exact")) <= F16_EXACT
    assert oracle.rel_err(y, oracle.mm(a, b, "wgsl")) <= F16_WGSL


# ----------------------------------------------- stateless C-ABI entry
def c_conv(ctx, x, w, b, pad, act, lo=-np.inf, hi=np.inf):
    """wgx_conv2d with device pointers, a caller-provided scratch and the
    context's stream."""
    B, IC, H, W = x.shape
    OC, _, KH, KW = w.shape
    p = _lib.ConvParams(B, IC, H, W, OC, H + 2 * pad - KH + 1, W + 2 * pad - KW + 1, KH, KW, 1, 1,
                        pad, pad, 1, 1, 1, int(b is not None), 1, act, lo, hi)
    plan = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(p), ctypes.byref(plan)))
    tx = ctx.tensor("float16", x.shape).setData(x)
    tw = ctx.tensor("float16", w.shape).setData(w)
    tb = ctx.tensor("float16", b.shape).setData(b) if b is not None else None
    out = ctx.tensor("float16", [B, OC, p.OH, p.OW])
    scratch = ctx.storageBuffer(max(16, plan.scratch_bytes))
    _lib.check(_lib.lib.wgx_conv2d(ctypes.byref(p), tx.data_ptr, tw.data_ptr,
                                   tb.data_ptr if tb else None, out.data_ptr, scratch.device_ptr,
                                   scratch.size, ctx.stream))
    ctx.sync()
    return out.numpy(), plan


def test_stateless_conv_silu_config2_geometry(ctx):
    (x,) = oracle.make_inputs([(1, 64, 160, 160)], seed=90)
    w = kaiming((128, 64, 3, 3), 91)
    (b,) = oracle.make_inputs([(128,)], seed=92, scale=0.01)
    y, plan = c_conv(ctx, x, w, b, 1, _lib.ACT_SILU)
    assert plan.variant == _lib.CONV_UMMA
    check_f16(y, x, w, b, 1, 1, 1, 1, act=oracle.ACT_SILU)


def test_config2_full_batch_properties(ctx):
    """BASELINE config 2 at full size ([8,64,160,160], fused SiLU): image 0
    against the oracle, and every image equal (bit for bit) to the same
    image convolved alone."""
    x = oracle.make_inputs([(8, 64, 160, 160)], seed=0)[0]
    w = kaiming((128, 64, 3, 3), 1)
    (b,) = oracle.make_inputs([(128,)], seed=2, scale=0.01)
    y, _ = c_conv(ctx, x, w, b, 1, _lib.ACT_SILU)
    check_f16(y[:1], x[:1], w, b, 1, 1, 1, 1, act=oracle.ACT_SILU)
    for i in (3, 7):
        yi, _ = c_conv(ctx, x[i:i + 1], w, b, 1, _lib.ACT_SILU)
        np.testing.assert_array_equal(yi[0], y[i])
    # the whole batch against the exact oracle
    check_f16(y, x, w, b, 1, 1, 1, 1, act=oracle.ACT_SILU)


def test_config3_full_size_depthwise(ctx):
    """BASELINE config 3 depthwise at the benchmarked size: [16,256,80,80] x
    [256,1,5,5], stride 1, pad 2, groups 256, N(0,1) input, N(0,0.1)
    weights, against the exact oracle and the reference's f16 arithmetic."""
    (x,) = oracle.make_inputs([(16, 256, 80, 80)], seed=90)
    (w, b) = oracle.make_inputs([(256, 1, 5, 5), (256,)], seed=91, scale=[0.1, 0.01])
    y = engine_conv(ctx, x, w, b, 1, 2, 1, 256)
    check_f16(y, x, w, b, 1, 2, 1, 256)


def test_config3_full_size_pointwise(ctx):
    """BASELINE config 3's 1x1 pointwise at the benchmarked size:
    [16,256,80,80] x [256,256,1,1] (Kaiming weights), through the TMA direct
    mode, against the exact oracle and the reference's f16 arithmetic (its
    conv2d-tile64-f16 kernel for B > 1)."""
    (x,) = oracle.make_inputs([(16, 256, 80, 80)], seed=92)
    w = kaiming((256, 256, 1, 1), 93)
    (b,) = oracle.make_inputs([(256,)], seed=94, scale=0.01)
    y = engine_conv(ctx, x, w, b, 1, 0, 1, 1)
    check_f16(y, x, w, b, 1, 0, 1, 1)


# --------------------------------------------------- program fusion
def test_program_depthwise_silu_fusion_in_place(ctx):
    """A depthwise conv -> sigmoid -> mul whose output reuses the conv
    input's pool fuses (the tiled depthwise kernel stages whole planes
    before writing them): 3 commands, result equal to the oracle's."""
    C, H, W = 24, 20, 20
    (x,) = oracle.make_inputs([(2, C, H, W)], seed=110)
    (w, b) = oracle.make_inputs([(C, 1, 3, 3), (C,)], seed=111, scale=[0.3, 0.05])
    wbytes = w.tobytes() + b.tobytes()
    shape = [2, C, H, W]
    nb = 2 * C * H * W * 2
    prog = {
        "version": "1",
        "chain": [
            {"name": "aten.convolution.default", "args": [0, 1, 2, 3, 4, 5, 6, 7, 8, 9]},
            {"name": "aten.sigmoid.default", "args": [9, 10]},
            {"name": "aten.mul.Tensor", "args": [9, 10, 11]},
        ],
        "values": [
            {"type": "tensor", "shape": shape, "dtype": "float16", "memObjId": 0},
            {"type": "tensor", "shape": [C, 1, 3, 3], "dtype": "float16", "weightsOffset": 0,
             "weightsLength": w.nbytes},
            {"type": "tensor", "shape": [C], "dtype": "float16", "weightsOffset": w.nbytes,
             "weightsLength": b.nbytes},
            {"type": "list", "items": [1, 1]}, {"type": "list", "items": [1, 1]},
            {"type": "list", "items": [1, 1]}, {"type": "scalar", "value": False},
            {"type": "list", "items": [0, 0]}, {"type": "scalar", "value": C},
            {"type": "tensor", "shape": shape, "dtype": "float16", "memObjId": 1},
            {"type": "tensor", "shape": shape, "dtype": "float16", "memObjId": 2},
            {"type": "tensor", "shape": shape, "dtype": "float16", "memObjId": 0},
        ],
        "inputIds": [0], "outputIds": [11],
        "memoryPlan": {"pools": [{"id": i, "size": nb} for i in range(3)]},
    }
    tin = ctx.tensor("float16", shape).setData(x)
    tout = ctx.tensor("float16", shape)
    ctx.recordProgram(prog, wbytes, [tin, tout])
    # one convolution; input and output are bound to the caller's tensors
    assert [n for n in ctx.command_names() if n != "copy"] == [
        n for n in ctx.command_names() if n.startswith("aten.convolution")]
    assert len([n for n in ctx.command_names() if n != "copy"]) == 1
    ctx.submit()
    ctx.sync()
    ex = oracle.conv2d(x, w, b, 1, 1, 1, C, act=oracle.ACT_SILU, mode="exact")
    assert oracle.rel_err(tout.numpy(), ex) <= 5e-3


@pytest.mark.parametrize("out_pool,ic,commands", [(3, 32, 3), (0, 32, 3), (0, 4, 3)])
def test_program_conv_sigmoid_mul_fusion(ctx, out_pool, ic, commands):
    """conv -> sigmoid -> mul becomes one conv with a SiLU epilogue (input
    copy + conv + output copy = 3 commands for an unbound program). The
    program input is read from the caller's tensor, so even with the mul's
    output in the conv input's pool (out_pool 0) the output overlays no
    input and a CUDA-core conv (IC=4) fuses too."""
    (x,) = oracle.make_inputs([(2, ic, 24, 24)], seed=100)
    w = kaiming((48, ic, 3, 3), 101)
    (b,) = oracle.make_inputs([(48,)], seed=102, scale=0.01)
    wbytes = w.tobytes() + b.tobytes()
    prog = {
        "version": "1",
        "chain": [
            {"name": "aten.convolution.default", "args": [0, 1, 2, 3, 4, 5, 6, 7, 8, 9]},
            {"name": "aten.sigmoid.default", "args": [9, 10]},
            {"name": "aten.mul.Tensor", "args": [9, 10, 11]},
        ],
        "values": [
            {"type": "tensor", "shape": [2, ic, 24, 24], "dtype": "float16", "memObjId": 0},
            {"type": "tensor", "shape": [48, ic, 3, 3], "dtype": "float16", "weightsOffset": 0,
             "weightsLength": w.nbytes},
            {"type": "tensor", "shape": [48], "dtype": "float16", "weightsOffset": w.nbytes,
             "weightsLength": b.nbytes},
            {"type": "list", "items": [1, 1]},
            {"type": "list", "items": [1, 1]},
            {"type": "list", "items": [1, 1]},
            {"type": "scalar", "value": False},
            {"type": "list", "items": [0, 0]},
            {"type": "scalar", "value": 1},
            {"type": "tensor", "shape": [2, 48, 24, 24], "dtype": "float16", "memObjId": 1},
            {"type": "tensor", "shape": [2, 48, 24, 24], "dtype": "float16", "memObjId": 2},
            {"type": "tensor", "shape": [2, 48, 24, 24], "dtype": "float16",
             "memObjId": out_pool},
        ],
        "inputIds": [0],
        "outputIds": [11],
        "memoryPlan": {"pools": [{"id": 0, "size": 2 * 48 * 24 * 24 * 2},
                                 {"id": 1, "size": 2 * 48 * 24 * 24 * 2},
                                 {"id": 2, "size": 2 * 48 * 24 * 24 * 2},
                                 {"id": 3, "size": 2 * 48 * 24 * 24 * 2}]},
    }
    tin = ctx.tensor("float16", x.shape).setData(x)
    tout = ctx.tensor("float16", [2, 48, 24, 24])
    ctx.recordProgram(prog, wbytes, [tin, tout])
    ctx.submit()
    ctx.sync()
    y = tout.numpy()
    # (commands counts the caller copies of an unbound program: 2)
    assert len([n for n in ctx.command_names() if n != "copy"]) == commands - 2
    ex = oracle.conv2d(x, w, b, 1, 1, 1, 1, act=oracle.ACT_SILU, mode="exact")
    assert oracle.rel_err(y, ex) <= 5e-3


@pytest.mark.parametrize("C,H,W", [(32, 16, 20), (8, 16, 20), (8, 6, 160)])
def test_program_split_and_residual_folded_into_convs(ctx, C, H, W):
    """C2f-style block: conv1 (+SiLU) -> split [a, b]; conv2 (+SiLU) of b;
    y = b + conv2(b) (residual); cat [a, b, y]. The split and the add are
    done by the convolutions' epilogues; the result equals the program
    oracle's. (C = 8: conv2 takes the folded-column form, with 2-byte and
    16-byte residual stores.)"""
    import program_oracle
    B = 2
    rng = np.random.default_rng(120)
    x = rng.standard_normal((B, C, H, W)).astype(np.float16)
    w1 = kaiming((2 * C, C, 1, 1), 121)
    w2 = kaiming((C, C, 3, 3), 122)
    b1 = (rng.standard_normal(2 * C) * 0.01).astype(np.float16)
    b2 = (rng.standard_normal(C) * 0.01).astype(np.float16)
    wb = w1.tobytes() + b1.tobytes() + w2.tobytes() + b2.tobytes()
    o = [0, w1.nbytes, w1.nbytes + b1.nbytes, w1.nbytes + b1.nbytes + w2.nbytes]
    t = lambda shape, pool: {"type": "tensor", "shape": shape, "dtype": "float16",
                             "memObjId": pool}
    vals = [
        t([B, C, H, W], 0),                                                        # 0 x
        {"type": "tensor", "shape": [2 * C, C, 1, 1], "dtype": "float16",
         "weightsOffset": o[0], "weightsLength": w1.nbytes},                      # 1
        {"type": "tensor", "shape": [2 * C], "dtype": "float16",
         "weightsOffset": o[1], "weightsLength": b1.nbytes},                      # 2
        {"type": "list", "items": [1, 1]}, {"type": "list", "items": [0, 0]},    # 3 4
        {"type": "list", "items": [1, 1]}, {"type": "scalar", "value": False},   # 5 6
        {"type": "list", "items": [0, 0]}, {"type": "scalar", "value": 1},       # 7 8
        t([B, 2 * C, H, W], 1),                                                    # 9 v1
        t([B, 2 * C, H, W], 2),                                                    # 10 s1
        t([B, 2 * C, H, W], 3),                                                    # 11 y1
        {"type": "list", "items": [C, C]}, {"type": "scalar", "value": 1},       # 12 13
        t([B, C, H, W], 4), t([B, C, H, W], 5),                                    # 14 a, 15 b
        {"type": "tensorlist", "items": [14, 15]},                                 # 16
        {"type": "tensor", "shape": [C, C, 3, 3], "dtype": "float16",
         "weightsOffset": o[2], "weightsLength": w2.nbytes},                      # 17
        {"type": "tensor", "shape": [C], "dtype": "float16",
         "weightsOffset": o[3], "weightsLength": b2.nbytes},                      # 18
        {"type": "list", "items": [1, 1]},                                         # 19 pad 1
        t([B, C, H, W], 1), t([B, C, H, W], 2), t([B, C, H, W], 3),               # 20 v2 21 s2 22 m
        t([B, C, H, W], 6),                                                        # 23 y = b + m
        {"type": "tensorlist", "items": [14, 15, 23]},                             # 24
        t([B, 3 * C, H, W], 7),                                                    # 25 out
    ]
    chain = [
        {"name": "aten.convolution.default", "args": [0, 1, 2, 3, 4, 5, 6, 7, 8, 9]},
        {"name": "aten.sigmoid.default", "args": [9, 10]},
        {"name": "aten.mul.Tensor", "args": [9, 10, 11]},
        {"name": "aten.split_with_sizes_copy.default", "args": [11, 12, 13, 16]},
        {"name": "aten.convolution.default", "args": [15, 17, 18, 3, 19, 5, 6, 7, 8, 20]},
        {"name": "aten.sigmoid.default", "args": [20, 21]},
        {"name": "aten.mul.Tensor", "args": [20, 21, 22]},
        {"name": "aten.add.Tensor", "args": [15, 22, 8, 23]},
        {"name": "aten.cat.default", "args": [24, 13, 25]},
    ]
    nb = lambda c: B * c * H * W * 2
    prog = {"version": "1", "chain": chain, "values": vals, "inputIds": [0], "outputIds": [25],
            "memoryPlan": {"pools": [{"id": 0, "size": nb(C)}, {"id": 1, "size": nb(2 * C)},
                                     {"id": 2, "size": nb(2 * C)}, {"id": 3, "size": nb(2 * C)},
                                     {"id": 4, "size": nb(C)}, {"id": 5, "size": nb(C)},
                                     {"id": 6, "size": nb(C)}, {"id": 7, "size": nb(3 * C)}]}}
    tin = ctx.tensor("float16", x.shape).setData(x)
    tout = ctx.tensor("float16", [B, 3 * C, H, W])
    ctx.recordProgram(prog, wb, [tin, tout])
    # conv1 (split), conv2 (residual), cat (+ caller copies where not bound)
    assert len([n for n in ctx.command_names() if n != "copy"]) == 3
    ctx.submit()
    ctx.sync()
    (ref,) = program_oracle.run_program(prog, wb, [x])
    assert oracle.rel_err(tout.numpy(), ref) <= 5e-3
