"""API behaviour of the reference (tests/api/context.test.ts,
tests/api/tensor.test.ts, tests/api/program.test.ts) on the engine."""
import numpy as np
import pytest

import wgx
from kat_cases import literal
from wgx import GPUBufferUsage, WgpuExecutionContext, WgxError

pytestmark = pytest.mark.gpu


# -------------------------------------------------- context.test.ts
def test_allocates_storage_buffers(ctx):
    buf = ctx.storageBuffer(256)
    assert buf.size >= 256
    assert buf.usage & GPUBufferUsage.STORAGE


def test_aligns_storage_buffer_size_to_4_bytes(ctx):
    assert ctx.storageBuffer(1).size == 4


def test_creates_tensors_with_owned_buffers(ctx):
    t = ctx.tensor("float32", [2, 3])
    assert t.shape == (2, 3)
    assert t.byteLength == 24


def test_copy_validates_copy_src(ctx):
    dev = ctx.device
    src_buf = dev.createBuffer(16, GPUBufferUsage.STORAGE | GPUBufferUsage.COPY_DST)
    dst = ctx.tensor("float32", [4])
    src = wgx.Tensor("float32", [4], dev, src_buf)
    with pytest.raises(WgxError, match="COPY_SRC"):
        ctx.copy(src, dst)
    del src
    src_buf.destroy()


def test_copy_validates_copy_dst(ctx):
    dev = ctx.device
    src = ctx.tensor("float32", [4])
    dst_buf = dev.createBuffer(16, GPUBufferUsage.STORAGE | GPUBufferUsage.COPY_SRC)
    dst = wgx.Tensor("float32", [4], dev, dst_buf)
    with pytest.raises(WgxError, match="COPY_DST"):
        ctx.copy(src, dst)
    del dst
    dst_buf.destroy()


def test_copy_validates_destination_size(ctx):
    with pytest.raises(WgxError, match="< source"):
        ctx.copy(ctx.tensor("float32", [4]), ctx.tensor("float32", [2]))


def test_copy_submit_transfers_data(ctx):
    src = ctx.tensor("float32", [4])
    dst = ctx.tensor("float32", [4])
    src.setData(np.array([1, 2, 3, 4], np.float32))
    ctx.copy(src, dst)
    ctx.submit()
    ctx.sync()
    assert list(dst.numpy()) == [1, 2, 3, 4]


def test_destroy_prevents_further_use():
    c = WgpuExecutionContext(0)
    c.destroy()
    with pytest.raises(WgxError, match="destroyed"):
        c.storageBuffer(16)
    with pytest.raises(WgxError, match="destroyed"):
        c.sync()


def test_destroy_is_idempotent():
    c = WgpuExecutionContext(0)
    c.destroy()
    c.destroy()


def test_submit_with_no_commands_is_noop(ctx):
    ctx.submit()


def test_sync_without_submit(ctx):
    ctx.sync()


def test_submit_replays_all_commands_until_reset(ctx):
    a = ctx.tensor("float32", [4]).setData(np.ones(4, np.float32))
    b = ctx.tensor("float32", [4]).setData(np.zeros(4, np.float32))
    out = ctx.tensor("float32", [4])
    ctx.recordShader(wgx.shaders.add, [a, b, 1.0, out])
    ctx.copy(out, b)  # b <- a + b: grows by one per submit
    for _ in range(3):
        ctx.submit()
    ctx.sync()
    assert list(b.numpy()) == [3, 3, 3, 3]
    ctx.reset()
    ctx.submit()
    ctx.sync()
    assert list(b.numpy()) == [3, 3, 3, 3]


# ---------------------------------------------------- tensor.test.ts
def test_tensor_valid_shape(ctx):
    t = ctx.tensor("float32", [2, 3])
    assert (t.shape, t.numel, t.byteLength, t.dtype) == ((2, 3), 6, 24, "float32")


def test_tensor_rejects_bad_shapes(ctx):
    with pytest.raises(WgxError, match="exceeds maximum rank"):
        ctx.tensor("float32", [1] * (wgx.MAX_NDIM + 1))
    with pytest.raises(WgxError, match="positive integers"):
        ctx.tensor("float32", [0, 3])
    with pytest.raises(WgxError, match="positive integers"):
        ctx.tensor("float32", [1.5, 3])


def test_tensor_rejects_small_buffer_and_missing_storage(ctx):
    dev = ctx.device
    buf = dev.createBuffer(4, GPUBufferUsage.STORAGE | GPUBufferUsage.COPY_DST)
    with pytest.raises(WgxError, match="< required"):
        wgx.Tensor("float32", [2, 3], dev, buf)
    buf.destroy()
    buf = dev.createBuffer(24, GPUBufferUsage.COPY_DST | GPUBufferUsage.COPY_SRC)
    with pytest.raises(WgxError, match="STORAGE flag"):
        wgx.Tensor("float32", [2, 3], dev, buf)
    buf.destroy()


def test_set_get_roundtrip_and_prefix(ctx):
    t = ctx.tensor("float32", [2, 3])
    t.setData(np.arange(1, 7, dtype=np.float32))
    assert list(t.numpy().reshape(-1)) == [1, 2, 3, 4, 5, 6]
    t.setData(np.array([7, 8], np.float32))
    assert list(t.numpy().reshape(-1)) == [7, 8, 3, 4, 5, 6]
    t.setData(np.array([1, 2, 3, 4], np.float32).tobytes())
    assert list(t.numpy().reshape(-1)) == [1, 2, 3, 4, 5, 6]


def test_set_data_rejects_larger_source(ctx):
    with pytest.raises(WgxError, match="pass a view"):
        ctx.tensor("float32", [2, 3]).setData(np.zeros(8, np.float32))


def test_set_data_requires_copy_dst(ctx):
    dev = ctx.device
    buf = dev.createBuffer(24, GPUBufferUsage.STORAGE | GPUBufferUsage.COPY_SRC)
    t = wgx.Tensor("float32", [2, 3], dev, buf)
    with pytest.raises(WgxError, match="COPY_DST"):
        t.setData(np.zeros(6, np.float32))
    del t
    buf.destroy()


def test_unaligned_byte_sizes(ctx):
    t = ctx.tensor("uint8", [3])
    t.setData(np.array([7, 42, 99], np.uint8))
    assert list(np.frombuffer(t.getData(), np.uint8)) == [7, 42, 99]


# --------------------------------------------------- program.test.ts
PROG = {
    "version": "1",
    "chain": [{"name": "aten.add.Tensor", "args": [0, 1, 2, 3]},
              {"name": "aten.mm.default", "args": [3, 4, 5]}],
    "values": [
        {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 0},
        {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 1},
        {"type": "scalar", "value": 1.5},
        {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 2},
        {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 3},
        {"type": "tensor", "shape": [2, 2], "dtype": "float32", "memObjId": 0},
    ],
    "inputIds": [0, 1, 4],
    "outputIds": [5],
    "memoryPlan": {"pools": [{"id": i, "size": 16} for i in range(4)]},
}


def _abc(ctx):
    a = ctx.tensor("float32", [2, 2]).setData(np.array([1, 2, 3, 4], np.float32))
    b = ctx.tensor("float32", [2, 2]).setData(np.array([10, 20, 30, 40], np.float32))
    c = ctx.tensor("float32", [2, 2]).setData(np.array([1, 2, 3, 4], np.float32))
    return a, b, c


def test_program_runs_with_buffer_reuse(ctx):
    a, b, c = _abc(ctx)
    out = ctx.tensor("float32", [2, 2])
    ctx.recordProgram(PROG, b"", [a, b, c, out])
    ctx.submit()
    ctx.sync()
    exp, tol = literal("program", "runs a 2-kernel program")
    assert np.max(np.abs(out.numpy().reshape(-1) - exp)) <= tol


def test_program_rejects_wrong_arg_count(ctx):
    a, b, c = _abc(ctx)
    with pytest.raises(WgxError, match="expected 4 args"):
        ctx.recordProgram(PROG, b"", [a, b, c])


def test_program_rejects_non_tensor_output(ctx):
    a, b, c = _abc(ctx)
    with pytest.raises(WgxError, match="output 0 must be a Tensor"):
        ctx.recordProgram(PROG, b"", [a, b, c, 42])


def test_program_rejects_unknown_operator(ctx):
    a, b, c = _abc(ctx)
    bad = dict(PROG, chain=[{"name": "aten.nonexistent.default", "args": [0, 1, 2, 3]}])
    with pytest.raises(WgxError, match="unknown operator"):
        ctx.recordProgram(bad, b"", [a, b, c, ctx.tensor("float32", [2, 2])])


def test_program_rejects_missing_pool(ctx):
    a, b, c = _abc(ctx)
    vals = [dict(PROG["values"][0], memObjId=99)] + PROG["values"][1:]
    with pytest.raises(WgxError, match="no memory pool 99"):
        ctx.recordProgram(dict(PROG, values=vals), b"", [a, b, c, ctx.tensor("float32", [2, 2])])


def test_failed_record_leaves_no_commands(ctx):
    a, b, c = _abc(ctx)
    bad = dict(PROG, chain=PROG["chain"] + [{"name": "aten.nope", "args": []}])
    with pytest.raises(WgxError):
        ctx.recordProgram(bad, b"", [a, b, c, ctx.tensor("float32", [2, 2])])
    assert ctx.stats()["commands"] == 0


def _conv_program(B=2, C=16, H=12, W=12, OC=8, seed=5):
    """One-input, one-output program: a 3x3 convolution with constant weights."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((OC, C, 3, 3)) * 0.1).astype(np.float16)
    b = (rng.standard_normal(OC) * 0.01).astype(np.float16)
    vals = [{"type": "tensor", "shape": [B, C, H, W], "dtype": "float16", "memObjId": 0},
            {"type": "tensor", "shape": [OC, C, 3, 3], "dtype": "float16", "weightsOffset": 0,
             "weightsLength": w.nbytes},
            {"type": "tensor", "shape": [OC], "dtype": "float16", "weightsOffset": w.nbytes,
             "weightsLength": b.nbytes},
            {"type": "list", "items": [1, 1]}, {"type": "list", "items": [1, 1]},
            {"type": "list", "items": [1, 1]}, {"type": "scalar", "value": False},
            {"type": "list", "items": [0, 0]}, {"type": "scalar", "value": 1},
            {"type": "tensor", "shape": [B, OC, H, W], "dtype": "float16", "memObjId": 1}]
    prog = {"version": "1",
            "chain": [{"name": "aten.convolution.default", "args": list(range(10))}],
            "values": vals, "inputIds": [0], "outputIds": [9],
            "memoryPlan": {"pools": [{"id": 0, "size": B * C * H * W * 2},
                                     {"id": 1, "size": B * OC * H * W * 2}]}}
    return prog, w.tobytes() + b.tobytes(), (B, C, H, W), (B, OC, H, W)


@pytest.mark.parametrize("depth,steps", [(2, 5), (3, 7)])
def test_pipeline_matches_serial_steps(ctx, depth, steps):
    """Pipelined steps (upload, compute and download of neighbouring steps
    overlapping, device slots reused) give exactly the outputs of
    setData / submit / getData run step by step on the same inputs."""
    prog, wb, xs_shape, ys_shape = _conv_program()
    inp = ctx.tensor("float16", xs_shape)
    out = ctx.tensor("float16", ys_shape)
    ctx.recordProgram(prog, wb, [inp, out])
    rng = np.random.default_rng(9)
    xs = [rng.standard_normal(xs_shape).astype(np.float16) for _ in range(steps)]
    ref = []
    for x in xs:
        inp.setData(x)
        ctx.submit()
        ref.append(out.numpy().copy())
    pipe = ctx.pipeline(inp, out, depth)
    try:
        hout = [np.full(ys_shape, np.nan, np.float16) for _ in range(steps)]
        for i, x in enumerate(xs):
            pipe.step(x, hout[i])
        pipe.sync()
        for i in range(steps):
            np.testing.assert_array_equal(hout[i], ref[i])
    finally:
        pipe.destroy()


def test_pipeline_rejects_bad_arguments(ctx):
    prog, wb, xs_shape, ys_shape = _conv_program()
    inp = ctx.tensor("float16", xs_shape)
    out = ctx.tensor("float16", ys_shape)
    ctx.recordProgram(prog, wb, [inp, out])
    with pytest.raises(wgx.WgxError, match="depth"):
        ctx.pipeline(inp, out, 1)
    pipe = ctx.pipeline(inp, out, 2)
    with pytest.raises(wgx.WgxError, match="smaller"):
        pipe.step(np.zeros(4, np.float16), np.zeros(ys_shape, np.float16))
    pipe.destroy()
    pipe.destroy()  # idempotent
