"""wgx_conv2d_noalloc: the convolution entry point that allocates nothing.

Some callers cannot hand the library scratch memory: code recorded inside a
CUDA stream capture (cudaMalloc is not allowed there), hosts whose device
memory belongs to an allocator the call site cannot reach, loops that cannot
afford cudaFree's device-wide synchronisation. For them wgx_conv2d_noalloc
takes only inputs and outputs and uses a fixed 32 MiB scratch buffer built
into the library. These tests call it through the C ABI and check it

* against the CPU oracle (exact mode) and against the existing entry point,
  wgx_conv2d with caller-provided scratch, on two calls in a row with
  different inputs and weights;
* after a larger call that left non-finite values all over the shared
  buffer, on smaller convolutions of the other kernel variants (stride-2
  space-to-depth stem, positions-on-M small-OC, 1x1 direct mode,
  channels-on-M): no leftover scratch byte reaches a kept output;
* inside a CUDA-graph capture, replayed twice.

The file sorts last so a run that stops at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest

import oracle
import wgx
from wgx import _lib

pytestmark = pytest.mark.gpu

F16_EXACT = 2e-3  # fp16 tensor-core parity vs the exact oracle (max|y-ref| / max|ref|)


def params(B, IC, H, W, OC, K, s, p, act):
    OH, OW = (H + 2 * p - K) // s + 1, (W + 2 * p - K) // s + 1
    return _lib.ConvParams(B, IC, H, W, OC, OH, OW, K, K, s, s, p, p, 1, 1, 1, 1, 1,
                           act, -np.inf, np.inf)


def plan_for(p):
    plan = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(p), ctypes.byref(plan)))
    return plan


def inputs(B, IC, H, W, OC, K, seed):
    x, w, b = oracle.make_inputs([(B, IC, H, W), (OC, IC, K, K), (OC,)], seed=seed,
                                 scale=[1.0, (2.0 / (IC * K * K)) ** 0.5, 0.01])
    return x, w, b


def noalloc(ctx, p, tx, tw, tb, out):
    _lib.check(_lib.lib.wgx_conv2d_noalloc(ctypes.byref(p), tx.data_ptr, tw.data_ptr,
                                           tb.data_ptr, out.data_ptr, ctx.stream))


def test_noalloc_matches_oracle_and_wgx_conv2d_on_two_calls(ctx):
    B, IC, H, W, OC = 2, 64, 40, 36, 96
    p = params(B, IC, H, W, OC, 3, 1, 1, _lib.ACT_SILU)
    plan = plan_for(p)
    assert plan.variant == _lib.CONV_UMMA and 0 < plan.scratch_bytes
    scratch = ctx.storageBuffer(plan.scratch_bytes)
    for call in range(2):
        # new inputs AND new weights on the second call: the packed weights
        # in the shared buffer must be rebuilt, not reused
        x, w, b = inputs(B, IC, H, W, OC, 3, seed=100 + call)
        tx = ctx.tensor("float16", x.shape).setData(x)
        tw = ctx.tensor("float16", w.shape).setData(w)
        tb = ctx.tensor("float16", b.shape).setData(b)
        ref_out = ctx.tensor("float16", [B, OC, H, W])
        out = ctx.tensor("float16", [B, OC, H, W])
        _lib.check(_lib.lib.wgx_conv2d(ctypes.byref(p), tx.data_ptr, tw.data_ptr, tb.data_ptr,
                                       ref_out.data_ptr, scratch.device_ptr, scratch.size,
                                       ctx.stream))
        noalloc(ctx, p, tx, tw, tb, out)
        ctx.sync()
        y = out.numpy()
        assert np.all(np.isfinite(y.astype(np.float32)))
        ex = oracle.conv2d(x, w, b, 1, 1, 1, 1, act=oracle.ACT_SILU, mode="exact")
        assert oracle.rel_err(y, ex) <= F16_EXACT, f"call {call} vs oracle"
        assert oracle.rel_err(y, ref_out.numpy()) <= F16_EXACT, f"call {call} vs wgx_conv2d"


# smaller convolutions of every scratch-using variant, run after a large
# call that filled the buffer with non-finite values:
# (B, IC, H, W, OC, K, stride, pad, expected plan description fragment)
AFTER_POISON = [
    (1, 3, 64, 64, 16, 3, 2, 1, "positions-on-M"),    # RGB stem: space-to-depth, 16 virtual ch.
    (2, 16, 26, 26, 8, 3, 1, 1, "kw-folded"),         # small OC, folded filter columns
    (2, 48, 32, 32, 64, 1, 1, 0, "positions-on-M"),   # 1x1 direct mode (packed weights only)
    (1, 64, 20, 20, 96, 3, 1, 1, "channels-on-M"),    # OC > 64
    (2, 32, 18, 22, 128, 3, 2, 1, "channels-on-M"),   # stride 2, channels on M
]


def describe(p):
    buf = ctypes.create_string_buffer(256)
    _lib.check(_lib.lib.wgx_conv2d_describe(ctypes.byref(p), buf, 256))
    return buf.value.decode()


def test_noalloc_never_reads_leftover_scratch(ctx):
    # 1) a large call with +inf inputs and NaN weights: the re-laid input and
    #    the packed weights in the shared buffer are all non-finite afterwards
    big = params(8, 128, 64, 64, 128, 3, 1, 1, _lib.ACT_NONE)
    need = plan_for(big).scratch_bytes
    assert 8 << 20 < need <= 32 << 20
    x = np.full((8, 128, 64, 64), np.inf, dtype=np.float16)
    w = np.full((128, 128, 3, 3), np.nan, dtype=np.float16)
    b = np.zeros(128, dtype=np.float16)
    tx = ctx.tensor("float16", x.shape).setData(x)
    tw = ctx.tensor("float16", w.shape).setData(w)
    tb = ctx.tensor("float16", b.shape).setData(b)
    out = ctx.tensor("float16", [8, 128, 64, 64])
    noalloc(ctx, big, tx, tw, tb, out)
    ctx.sync()
    assert not np.any(np.isfinite(out.numpy().astype(np.float32)))
    # 2) smaller convolutions of other variants, each against the oracle
    for i, (B, IC, H, W, OC, K, s, pd, kind) in enumerate(AFTER_POISON):
        p = params(B, IC, H, W, OC, K, s, pd, _lib.ACT_SILU)
        assert plan_for(p).variant == _lib.CONV_UMMA
        assert kind in describe(p), describe(p)
        x, w, b = inputs(B, IC, H, W, OC, K, seed=200 + i)
        tx = ctx.tensor("float16", x.shape).setData(x)
        tw = ctx.tensor("float16", w.shape).setData(w)
        tb = ctx.tensor("float16", b.shape).setData(b)
        out = ctx.tensor("float16", [B, OC, p.OH, p.OW])
        noalloc(ctx, p, tx, tw, tb, out)
        ctx.sync()
        y = out.numpy()
        assert np.all(np.isfinite(y.astype(np.float32))), (B, IC, H, W, OC, K, s)
        ex = oracle.conv2d(x, w, b, s, pd, 1, 1, act=oracle.ACT_SILU, mode="exact")
        assert oracle.rel_err(y, ex) <= F16_EXACT, (B, IC, H, W, OC, K, s)


def test_noalloc_inside_cuda_graph_capture():
    """The reason the entry point exists: calls recorded in a stream capture
    (global capture mode: any allocation on any thread would end the
    capture with an error). One eager warm-up of the same calls first (the
    first call on a device looks the buffer up), then two calls captured,
    the graph replayed twice against the eager outputs."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shapes = [(2, 64, 24, 20, 96, 3, 1, 1), (2, 16, 26, 26, 8, 3, 1, 1)]
    calls = []
    for i, (B, IC, H, W, OC, K, s, pd) in enumerate(shapes):
        p = params(B, IC, H, W, OC, K, s, pd, _lib.ACT_SILU)
        x, w, b = inputs(B, IC, H, W, OC, K, seed=300 + i)
        tens = [torch.from_numpy(a).to(dev) for a in (x, w, b)]
        out = torch.empty(B, OC, p.OH, p.OW, dtype=torch.float16, device=dev)
        calls.append((p, tens, out, (x, w, b, s, pd)))
    stream = torch.cuda.Stream(device=dev)

    def launch_all():
        for p, (tx, tw, tb), out, _ in calls:
            _lib.check(_lib.lib.wgx_conv2d_noalloc(
                ctypes.byref(p), ctypes.c_void_p(tx.data_ptr()), ctypes.c_void_p(tw.data_ptr()),
                ctypes.c_void_p(tb.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(stream.cuda_stream)))

    with torch.cuda.stream(stream):
        launch_all()
    torch.cuda.synchronize()
    eager = [c[2].clone() for c in calls]
    for c in calls:
        c[2].zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream, capture_error_mode="global"):
        launch_all()
    torch.cuda.synchronize()
    for rep in range(2):
        for c in calls:
            c[2].fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for (p, _, out, (x, w, b, s, pd)), e in zip(calls, eager):
            y = out.cpu().numpy()
            assert np.all(np.isfinite(y.astype(np.float32))), f"replay {rep}"
            assert torch.equal(out, e), f"replay {rep} differs from the eager call"
            ex = oracle.conv2d(x, w, b, s, pd, 1, 1, act=oracle.ACT_SILU, mode="exact")
            assert oracle.rel_err(y, ex) <= F16_EXACT
    del graph


def test_noalloc_rejects_scratch_beyond_its_buffer():
    # [8, 256, 160, 160]: the re-laid input alone is ~100 MB > 32 MiB
    p = params(8, 256, 160, 160, 64, 3, 1, 1, _lib.ACT_NONE)
    rc = _lib.lib.wgx_conv2d_noalloc(ctypes.byref(p), None, None, None, None, None)
    assert rc != 0
    assert "built-in buffer holds" in _lib.lib.wgx_last_error().decode()
