"""Failure detection without a GPU fault (wgx_debug_inject).

The reference reports every failure as a synchronous Error
(src/context.ts:52-56, 226-230, 296-298). Here two failures are made on
purpose and each must come back as a status code with the context still
usable afterwards:

* an allocation failure, injected on the host in front of cudaMalloc
  (nothing is allocated): WGX_ERR_NOMEM from storageBuffer and from
  recordProgram, then the same calls succeed;
* a tensor-core convolution whose producer role is told to issue no copies:
  the MMA and epilogue roles' bounded mbarrier waits (about 2 s) run out,
  the kernel records the timeout in the device error word and returns (no
  trap, no hang), and sync() raises WGX_ERR_DEVICE; the context then runs
  the same convolution correctly.
"""
import ctypes

import numpy as np
import pytest

import oracle
import wgx
from wgx import _lib
from wgx._lib import WgxError

from test_gpu_api import PROG, _abc

pytestmark = pytest.mark.gpu


@pytest.fixture
def inject():
    yield lambda flags: _lib.check(_lib.lib.wgx_debug_inject(flags))
    _lib.check(_lib.lib.wgx_debug_inject(0))


def test_injected_allocation_failure_is_reported_and_recoverable(ctx, inject):
    inject(_lib.INJECT_ALLOC_FAIL)
    with pytest.raises(WgxError) as e:
        ctx.storageBuffer(1024)
    assert e.value.code == _lib.WGX_ERR_NOMEM
    assert "cudaMalloc" in str(e.value)
    # one shot: the next allocation succeeds
    assert ctx.storageBuffer(1024).size == 1024
    # recordProgram: its arena allocation fails, no command is left behind
    a, b, c = _abc(ctx)
    out = ctx.tensor("float32", [2, 2])
    inject(_lib.INJECT_ALLOC_FAIL)
    with pytest.raises(WgxError) as e:
        ctx.recordProgram(PROG, b"", [a, b, c, out])
    assert e.value.code == _lib.WGX_ERR_NOMEM
    assert ctx.stats()["commands"] == 0
    ctx.recordProgram(PROG, b"", [a, b, c, out])
    ctx.submit()
    ctx.sync()
    # (a + 1.5 * b) @ c  (tests/api/program.test.ts:54-68)
    assert list(out.numpy().reshape(-1)) == [112.0, 160.0, 240.0, 352.0]


def _conv(ctx, x, w, b):
    tx = ctx.tensor("float16", x.shape).setData(x)
    tw = ctx.tensor("float16", w.shape).setData(w)
    tb = ctx.tensor("float16", b.shape).setData(b)
    out = ctx.tensor("float16", [x.shape[0], w.shape[0], x.shape[2], x.shape[3]])
    ctx.recordShader(wgx.shaders.convolution,
                     [tx, tw, tb, [1, 1], [1, 1], [1, 1], False, [0, 0], 1, out])
    return out


def test_bounded_wait_timeout_is_reported_and_recoverable(ctx, inject):
    (x, w, b) = oracle.make_inputs([(2, 32, 20, 20), (96, 32, 3, 3), (96,)], seed=400,
                                   scale=[1.0, (2.0 / 288) ** 0.5, 0.01])
    # the tensor-core path (the kernel with the bounded waits) is selected
    p = _lib.ConvParams(2, 32, 20, 20, 96, 20, 20, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                        _lib.ACT_NONE, -np.inf, np.inf)
    plan = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(p), ctypes.byref(plan)))
    assert plan.variant == _lib.CONV_UMMA
    inject(_lib.INJECT_SKIP_LOADS)
    _conv(ctx, x, w, b)
    ctx.submit()  # the launch parameters are fixed here (graph capture)
    inject(0)
    with pytest.raises(WgxError) as e:
        ctx.sync()
    assert e.value.code == _lib.WGX_ERR_DEVICE
    assert "bounded wait" in str(e.value)
    # the error word was read and cleared; the context keeps working
    ctx.reset()
    out = _conv(ctx, x, w, b)
    ctx.submit()
    ctx.sync()
    ex = oracle.conv2d(x, w, b, 1, 1, 1, 1, mode="exact")
    assert oracle.rel_err(out.numpy(), ex) <= 2e-3
