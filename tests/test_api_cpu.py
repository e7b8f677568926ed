"""CPU-only checks of the C-ABI library: it loads, exports every symbol the
header declares, plans kernel variants without a GPU, and fails cleanly
when no device is present."""
import ctypes
import os
import re

import numpy as np
import pytest

import wgx
from wgx import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "wgx.h")).read()
    return sorted(set(re.findall(r"WGX_API\s+(?:const\s+)?\w+\s*\*?\s*(wgx_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = header_symbols()
    assert "wgx_record_program" in syms and "wgx_conv2d" in syms and "wgx_mm" in syms
    assert len(syms) >= 28


def test_library_exports_every_header_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(header_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_device_count():
    assert _lib.lib.wgx_version() == 1
    assert wgx.device_count() >= 0


def test_debug_inject_flags():
    """The test-only fault injection accepts its two flags and rejects
    others (host state only: no GPU call)."""
    assert _lib.lib.wgx_debug_inject(_lib.INJECT_ALLOC_FAIL | _lib.INJECT_SKIP_LOADS) == 0
    assert _lib.lib.wgx_debug_inject(0) == 0
    assert _lib.lib.wgx_debug_inject(8) == _lib.WGX_ERR_INVALID
    assert "unknown flags" in _lib.lib.wgx_last_error().decode()


def test_normal_build_reports_no_bounds_checks():
    if os.environ.get("WGX_LIBRARY") == "bounds":
        assert _lib.build_flags() == _lib.BUILD_BOUNDS
    else:
        assert _lib.build_flags() == 0


def test_bounds_build_exports_the_same_symbols():
    """lib/libwgx_bounds.so (-DWGX_BOUNDS) is a drop-in for lib/libwgx.so:
    same exports, and it says which build it is."""
    path = os.path.join(_lib.PKG_DIR, "lib", "libwgx_bounds.so")
    if not os.path.exists(path):
        pytest.skip("bounds build not compiled (make -C wgpu-executorch_b200 bounds)")
    blib = ctypes.CDLL(path)
    missing = [s for s in header_symbols() if not hasattr(blib, s)]
    assert not missing, missing
    flags = ctypes.c_uint32(7)
    assert blib.wgx_build_flags(ctypes.byref(flags)) == 0 and flags.value == _lib.BUILD_BOUNDS


@pytest.mark.skipif(wgx.device_count() > 0, reason="a GPU is present")
def test_context_without_gpu_raises_cleanly():
    with pytest.raises(wgx.WgxError, match="no CUDA device"):
        wgx.WgpuExecutionContext(0)


def test_tensor_shape_validation_messages():
    dev = wgx.Device(0)
    with pytest.raises(wgx.WgxError, match="exceeds maximum rank"):
        wgx.Tensor("float32", [1] * (wgx.MAX_NDIM + 1), dev, None)
    with pytest.raises(wgx.WgxError, match="positive integers"):
        wgx.Tensor("float32", [0, 3], dev, None)
    with pytest.raises(wgx.WgxError, match="positive integers"):
        wgx.Tensor("float32", [-1, 3], dev, None)
    with pytest.raises(wgx.WgxError, match="positive integers"):
        wgx.Tensor("float32", [1.5, 3], dev, None)


def plan(**kw):
    p = _lib.ConvParams()
    d = dict(B=1, IC=1, IH=1, IW=1, OC=1, OH=1, OW=1, KH=1, KW=1, sH=1, sW=1, pH=0, pW=0, dH=1,
             dW=1, groups=1, has_bias=1, dtype=1, act=0, out_min=-np.inf, out_max=np.inf)
    d.update(kw)
    for k, v in d.items():
        setattr(p, k, v)
    out = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(p), ctypes.byref(out)))
    return out


def test_plan_selects_tensor_core_path_for_dense_fp16():
    # [8,64,160,160] x [128,64,3,3], s1 p1
    p = plan(B=8, IC=64, IH=160, IW=160, OC=128, OH=160, OW=160, KH=3, KW=3, pH=1, pW=1)
    assert p.variant == _lib.CONV_UMMA
    # tiles of 128 output channels x 256 positions: 102 per image
    assert p.grid_ctas == 8 * 102
    assert p.scratch_bytes > 8 * 64 * 162 * 162 * 2


def test_plan_depthwise_and_pointwise_of_config3():
    dw = plan(B=16, IC=256, IH=80, IW=80, OC=256, OH=80, OW=80, KH=5, KW=5, pH=2, pW=2,
              groups=256)
    assert dw.variant == _lib.CONV_DEPTHWISE
    pw = plan(B=16, IC=256, IH=80, IW=80, OC=256, OH=80, OW=80)
    assert pw.variant == _lib.CONV_UMMA


def test_plan_fallbacks():
    assert plan(dtype=0, B=1, IC=64, IH=8, IW=8, OC=64, OH=8, OW=8).variant == _lib.CONV_SIMT_GEMM
    assert plan(IC=3, OC=1, IH=4, IW=4, OH=4, OW=4).variant == _lib.CONV_POINTWISE1
    assert plan(IC=4, OC=4, groups=2, IH=2, IW=2, OH=2, OW=2).variant == _lib.CONV_DIRECT
    # stride 2 with one input channel: 4 space-to-depth channels -> CUDA cores
    assert plan(IC=1, IH=64, IW=64, OC=16, OH=32, OW=32, KH=3, KW=3, sH=2, sW=2, pH=1,
                pW=1).variant == _lib.CONV_SIMT_GEMM
    # stride above 4 -> CUDA cores
    assert plan(IC=16, IH=20, IW=20, OC=16, OH=4, OW=4, KH=3, KW=3, sH=5, sW=5, pH=1,
                pW=1).variant == _lib.CONV_SIMT_GEMM


def test_plan_strided_convs_use_tensor_cores():
    # YOLO stem: IC=3, 3x3 stride 2 pad 1 -> 2x2 stride-1 conv over 12 channels
    stem = plan(B=64, IC=3, IH=640, IW=640, OC=16, OH=320, OW=320, KH=3, KW=3, sH=2, sW=2,
                pH=1, pW=1)
    assert stem.variant == _lib.CONV_UMMA
    # 321 virtual rows of OW + 1 columns per image, the row pitch rounded up
    # to 328 (a multiple of 8); OC = 16 puts positions on the MMA M side,
    # 8 M blocks of 128 = 1024 positions per tile
    assert stem.grid_ctas == 64 * ((319 * 328 + 320 + 1023) // 1024)
    down = plan(B=64, IC=128, IH=80, IW=80, OC=128, OH=40, OW=40, KH=3, KW=3, sH=2, sW=2,
                pH=1, pW=1)
    assert down.variant == _lib.CONV_UMMA
    # re-laid input: 4 phases x 128 channels x 41 x 41 positions (+ slack)
    assert down.scratch_bytes >= 64 * 512 * 41 * 41 * 2


def describe(**kw):
    p = _lib.ConvParams()
    d = dict(B=1, IC=1, IH=1, IW=1, OC=1, OH=1, OW=1, KH=1, KW=1, sH=1, sW=1, pH=0, pW=0, dH=1,
             dW=1, groups=1, has_bias=1, dtype=1, act=0, out_min=-np.inf, out_max=np.inf)
    d.update(kw)
    for k, v in d.items():
        setattr(p, k, v)
    buf = ctypes.create_string_buffer(256)
    _lib.check(_lib.lib.wgx_conv2d_describe(ctypes.byref(p), buf, 256))
    return buf.value.decode()


def test_describe_names_the_selected_configuration():
    # channels on M, N = 256 positions, weights resident
    d = describe(B=8, IC=64, IH=160, IW=160, OC=128, OH=160, OW=160, KH=3, KW=3, pH=1, pW=1)
    assert d.startswith("umma channels-on-M N=256") and "resident" in d
    # YOLO stem: positions on M, N = 16, 8 M blocks of 128 positions
    d = describe(B=64, IC=3, IH=640, IW=640, OC=16, OH=320, OW=320, KH=3, KW=3, sH=2, sW=2,
                 pH=1, pW=1)
    assert "positions-on-M N=16 G=8" in d
    # 3x3 / stride 2 with 64 channels: skipped all-zero taps of the space-to-depth view
    d = describe(B=64, IC=128, IH=80, IW=80, OC=128, OH=40, OW=40, KH=3, KW=3, sH=2, sW=2,
                 pH=1, pW=1)
    assert "tapskip" in d
    assert describe(B=2, IC=8, IH=9, IW=9, OC=8, OH=9, OW=9, KH=3, KW=3, pH=1, pW=1,
                    groups=8) == "depthwise"
    # 3x3 / stride 1, OC <= 64: filter columns folded into N where the MMAs
    # saved outweigh the longer epilogue (ocp < 14 * ceil(IC / 16))
    d = describe(B=64, IC=16, IH=160, IW=160, OC=8, OH=160, OW=160, KH=3, KW=3, pH=1, pW=1)
    assert "positions-on-M N=32 G=8" in d and "kw-folded" in d
    d = describe(B=64, IC=64, IH=80, IW=80, OC=16, OH=80, OW=80, KH=3, KW=3, pH=1, pW=1)
    assert "N=48 G=4" in d and "kw-folded" in d
    d = describe(B=64, IC=256, IH=20, IW=20, OC=64, OH=20, OW=20, KH=3, KW=3, pH=1, pW=1)
    assert "N=192 G=1" in d and "kw-folded" in d
    # small planes (at most 512 positions): folded up to ocp = 16 * ceil(IC / 16)
    d = describe(B=64, IC=64, IH=20, IW=20, OC=64, OH=20, OW=20, KH=3, KW=3, pH=1, pW=1)
    assert "N=192 G=1" in d and "kw-folded" in d
    for ic, oc in ((8, 16), (32, 32), (16, 16)):
        d = describe(B=64, IC=ic, IH=80, IW=80, OC=oc, OH=80, OW=80, KH=3, KW=3, pH=1, pW=1)
        assert "kw-folded" not in d, (ic, oc, d)


def test_plan_rejects_bad_geometry():
    with pytest.raises(wgx.WgxError):
        plan(IC=3, OC=4, groups=2)
