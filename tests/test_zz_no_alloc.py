"""wgx_conv2d_noalloc: the convolution entry point that allocates nothing.

Some callers cannot hand the library scratch memory: code recorded inside a
CUDA stream capture, hosts whose device memory belongs to an allocator the
call site cannot reach, loops that cannot afford cudaFree's device-wide
synchronisation. For them wgx_conv2d_noalloc takes only inputs and outputs
and uses a fixed 32 MiB scratch buffer built into the library. These tests
call it through the C ABI twice in a row and compare each result with the
existing entry point, wgx_conv2d, which uses caller-provided scratch. The
file sorts last so a run that stops at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest

import wgx
from wgx import _lib

pytestmark = pytest.mark.gpu

F16_EXACT = 2e-3  # tolerance of the fp16 parity tests (max|y-ref| / max|ref|)


def rel_err(y, ref):
    y = y.astype(np.float64)
    ref = ref.astype(np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def params(B, IC, H, W, OC, act):
    return _lib.ConvParams(B, IC, H, W, OC, H, W, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                           act, -np.inf, np.inf)


def test_noalloc_matches_wgx_conv2d_on_two_calls():
    B, IC, H, W, OC = 2, 64, 40, 36, 96
    p = params(B, IC, H, W, OC, _lib.ACT_SILU)
    plan = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(p), ctypes.byref(plan)))
    assert plan.variant == _lib.CONV_UMMA and plan.scratch_bytes > 0
    rng = np.random.default_rng(7)
    ctx = wgx.WgpuExecutionContext(0)
    try:
        w = (rng.standard_normal((OC, IC, 3, 3), dtype=np.float32) * 0.06).astype(np.float16)
        b = (rng.standard_normal((OC,), dtype=np.float32) * 0.01).astype(np.float16)
        tw = ctx.tensor("float16", w.shape).setData(w)
        tb = ctx.tensor("float16", b.shape).setData(b)
        scratch = ctx.storageBuffer(plan.scratch_bytes)
        for call in range(2):
            x = rng.standard_normal((B, IC, H, W), dtype=np.float32).astype(np.float16)
            tx = ctx.tensor("float16", x.shape).setData(x)
            ref_out = ctx.tensor("float16", [B, OC, H, W])
            out = ctx.tensor("float16", [B, OC, H, W])
            _lib.check(_lib.lib.wgx_conv2d(ctypes.byref(p), tx.data_ptr, tw.data_ptr, tb.data_ptr,
                                           ref_out.data_ptr, scratch.device_ptr, scratch.size,
                                           ctx.stream))
            _lib.check(_lib.lib.wgx_conv2d_noalloc(ctypes.byref(p), tx.data_ptr, tw.data_ptr,
                                                   tb.data_ptr, out.data_ptr, ctx.stream))
            ctx.sync()
            y, ref = out.numpy(), ref_out.numpy()
            assert np.all(np.isfinite(y.astype(np.float32)))
            assert rel_err(y, ref) <= F16_EXACT, f"call {call}: {rel_err(y, ref)}"
    finally:
        ctx.destroy()


def test_noalloc_rejects_scratch_beyond_its_buffer():
    # [8, 256, 160, 160]: the re-laid input alone is ~100 MB > 32 MiB
    p = params(8, 256, 160, 160, 64, _lib.ACT_NONE)
    rc = _lib.lib.wgx_conv2d_noalloc(ctypes.byref(p), None, None, None, None, None)
    assert rc != 0
    assert "built-in buffer holds" in _lib.lib.wgx_last_error().decode()
