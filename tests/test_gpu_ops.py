"""The program-executor operators around the convolutions (cat, split,
permute, bmm, max-pool, upsampling, softmax, mean, pad, flat copies),
recorded one by one through the ``shaders`` registry and compared with
numpy restatements of the reference kernels' arithmetic
(src/shaders/<op>/*.wgsl.ts): data movement bit-exact, arithmetic in fp32
with one rounding (fp16: within one fp16 ulp of the fp64 result)."""
import numpy as np
import pytest

import wgx

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(7)


def T(ctx, a):
    return ctx.tensor("float16" if a.dtype == np.float16 else
                      "int32" if a.dtype == np.int32 else "float32", list(a.shape)).setData(a)


def empty(ctx, shape, dt):
    return ctx.tensor(dt, list(shape))


def run(ctx, shader, args):
    ctx.recordShader(shader, args)
    ctx.submit()
    ctx.sync()
    ctx.reset()


def rnd(shape, dt=np.float16):
    return RNG.standard_normal(shape).astype(dt)


@pytest.mark.parametrize("dt", [np.float16, np.float32])
@pytest.mark.parametrize("shapes,dim", [
    ([(4, 16, 20, 20), (4, 16, 20, 20), (4, 32, 20, 20)], 1),    # 16-byte pieces
    ([(2, 3, 5, 7), (2, 1, 5, 7)], 1),                           # unaligned pieces
    ([(3, 4, 6400), (3, 4, 1600), (3, 4, 400)], -1),
    ([(2, 8, 8)] * 10, 1),                                       # more than 8 pieces
])
def test_cat(ctx, shapes, dim, dt):
    xs = [rnd(s, dt) for s in shapes]
    ref = np.concatenate(xs, axis=dim)
    out = empty(ctx, ref.shape, "float16" if dt == np.float16 else "float32")
    run(ctx, wgx.shaders.cat, [[T(ctx, x) for x in xs], dim, out])
    np.testing.assert_array_equal(out.numpy(), ref)


@pytest.mark.parametrize("shape,sizes,dim", [
    ((4, 64, 20, 20), [32, 32], 1),
    ((3, 2, 128, 40), [32, 32, 64], 2),
    ((2, 5, 3), [2, 3], 1),
])
def test_split(ctx, shape, sizes, dim):
    x = rnd(shape)
    outs = [empty(ctx, tuple(s if d == dim else shape[d] for d in range(len(shape))), "float16")
            for s in sizes]
    run(ctx, wgx.shaders.splitWithSizesCopy, [T(ctx, x), sizes, dim, outs])
    refs = np.split(x, np.cumsum(sizes)[:-1], axis=dim)
    for o, r in zip(outs, refs):
        np.testing.assert_array_equal(o.numpy(), r)


@pytest.mark.parametrize("shape,perm", [
    ((3, 2, 400, 400), [0, 1, 3, 2]),   # tiled transpose
    ((2, 2, 32, 400), [0, 1, 3, 2]),
    ((5, 33, 17), [0, 2, 1]),
    ((2, 3, 4, 5), [2, 0, 3, 1]),       # generic index remap
])
def test_permute(ctx, shape, perm):
    x = rnd(shape)
    ref = np.transpose(x, perm)
    out = empty(ctx, ref.shape, "float16")
    run(ctx, wgx.shaders.permuteCopy, [T(ctx, x), perm, out])
    np.testing.assert_array_equal(out.numpy(), ref)


@pytest.mark.parametrize("dt", [np.float16, np.float32])
@pytest.mark.parametrize("bmkn", [(8, 400, 32, 400), (8, 64, 400, 400), (3, 5, 7, 9),
                                  (2, 65, 17, 130)])
def test_bmm(ctx, bmkn, dt):
    b, m, k, n = bmkn
    a, bb = rnd((b, m, k), dt), rnd((b, k, n), dt)
    out = empty(ctx, (b, m, n), "float16" if dt == np.float16 else "float32")
    run(ctx, wgx.shaders.bmm, [T(ctx, a), T(ctx, bb), out])
    ref = np.matmul(a.astype(np.float64), bb.astype(np.float64))
    err = np.abs(out.numpy().astype(np.float64) - ref).max() / np.abs(ref).max()
    assert err <= (2e-3 if dt == np.float16 else 1e-5)


@pytest.mark.parametrize("bmkn", [
    (2, 400, 32, 400),   # YOLO26-N PSA shapes of one image: channels on the MMA M side
    (2, 64, 400, 400),   # positions on M (M <= 64), TMA reads of the [K][N] images
    (3, 96, 64, 50),     # N % 8 != 0: re-laid input
    (4, 130, 24, 72),    # two M tiles, K not a multiple of 16
    (5, 16, 8, 64),
])
def test_bmm_fp16_tensor_cores(ctx, bmkn):
    """fp16 aten.bmm on the tcgen05 pipeline (per-image weights): one weight
    pack + the tensor-core kernel (+ re-layout when N % 8 != 0), against the
    exact oracle batch by batch (fp16 bound of the tensor-core path)."""
    import oracle
    b, m, k, n = bmkn
    a, bb = oracle.make_inputs([(b, m, k), (b, k, n)], seed=95, dist="uniform")
    out = empty(ctx, (b, m, n), "float16")
    ctx.recordShader(wgx.shaders.bmm, [T(ctx, a), T(ctx, bb), out])
    assert ctx.stats()["kernel_launches"] == (2 if n % 8 == 0 else 3)
    ctx.submit()
    ctx.sync()
    # after the submit: counted from the captured graph's kernel nodes
    assert ctx.stats()["kernel_launches"] == (2 if n % 8 == 0 else 3)
    y = out.numpy()
    ctx.reset()
    for i in range(b):
        assert oracle.rel_err(y[i], oracle.mm(a[i], bb[i], "exact")) <= 2e-3, i


def maxpool_ref(x, k, s, p, d, ceil_mode, f16):
    N, C, H, W = x.shape
    def osz(n, kk, ss, pp, dd):
        num = n + 2 * pp - (dd * (kk - 1) + 1)
        q = num / ss
        return int(np.ceil(q) if ceil_mode else np.floor(q)) + 1
    OH, OW = osz(H, k[0], s[0], p[0], d[0]), osz(W, k[1], s[1], p[1], d[1])
    y = np.empty((N, C, OH, OW), np.float32)
    idx = np.zeros((N, C, OH, OW), np.int32)
    start = -65504.0 if f16 else -3.4028234663852886e38
    xf = x.astype(np.float32)
    for oh in range(OH):
        for ow in range(OW):
            best = np.full((N, C), start, np.float32)
            bi = np.zeros((N, C), np.int32)
            for kh in range(k[0]):
                ih = oh * s[0] - p[0] + kh * d[0]
                if ih < 0 or ih >= H:
                    continue
                for kw in range(k[1]):
                    iw = ow * s[1] - p[1] + kw * d[1]
                    if iw < 0 or iw >= W:
                        continue
                    v = xf[:, :, ih, iw]
                    m = v > best
                    best = np.where(m, v, best)
                    bi = np.where(m, ih * W + iw, bi)
            y[:, :, oh, ow] = best
            idx[:, :, oh, ow] = bi
    return y, idx


@pytest.mark.parametrize("geom", [
    ((3, 16, 20, 20), (5, 5), (1, 1), (2, 2), (1, 1), False),   # YOLO SPPF, plane kernel
    ((2, 4, 9, 11), (3, 3), (2, 2), (1, 1), (1, 1), True),      # ceil mode
    ((1, 2, 70, 70), (2, 2), (2, 2), (0, 0), (1, 1), False),    # plane > 4096: generic
    ((1, 3, 12, 12), (3, 3), (1, 1), (0, 0), (2, 2), False),    # dilation
    ((2, 9, 13, 17), (3, 3), (1, 1), (1, 1), (1, 1), False),    # row kernel, K = 3
    ((1, 5, 11, 9), (7, 7), (1, 1), (3, 3), (1, 1), False),     # row kernel, K = 7
    ((2, 40, 20, 20), (5, 5), (1, 1), (0, 0), (1, 1), False),   # row kernel, no padding
])
@pytest.mark.parametrize("ties", [False, True])
def test_maxpool(ctx, geom, ties):
    shape, k, s, p, d, ceil_mode = geom
    x = rnd(shape)
    if ties:  # coarse values: many equal maxima, the first one in window order wins
        x = (np.round(x.astype(np.float32) * 2) / 2).astype(x.dtype)
    y, idx = maxpool_ref(x, k, s, p, d, ceil_mode, True)
    vals = empty(ctx, y.shape, "float16")
    ind = empty(ctx, y.shape, "int32")
    run(ctx, wgx.shaders.maxPool2d, [T(ctx, x), list(k), list(s), list(p), list(d), ceil_mode,
                                     [vals, ind]])
    np.testing.assert_array_equal(vals.numpy().astype(np.float32), y)
    np.testing.assert_array_equal(ind.numpy(), idx)


@pytest.mark.parametrize("shape,out_hw", [((2, 16, 20, 20), (40, 40)), ((1, 3, 5, 7), (11, 13)),
                                          ((2, 8, 40, 40), (80, 80))])
def test_upsample_nearest(ctx, shape, out_hw):
    x = rnd(shape)
    N, C, H, W = shape
    ih = (np.arange(out_hw[0]) * H) // out_hw[0]
    iw = (np.arange(out_hw[1]) * W) // out_hw[1]
    ref = x[:, :, ih][:, :, :, iw]
    out = empty(ctx, (N, C) + out_hw, "float16")
    run(ctx, wgx.shaders.upsampleNearest2d, [T(ctx, x), list(out_hw), None, out])
    np.testing.assert_array_equal(out.numpy(), ref)


@pytest.mark.parametrize("align", [True, False])
def test_upsample_bilinear(ctx, align):
    x = rnd((2, 5, 14, 14), np.float32)
    OH, OW = 28, 21
    def src(o, n_in, n_out):
        o = np.arange(o, dtype=np.float64)
        if align:
            return o * (n_in - 1) / (n_out - 1)
        return (o + 0.5) * n_in / n_out - 0.5
    sh, sw = src(OH, 14, OH), src(OW, 14, OW)
    h0, w0 = np.floor(sh).astype(int), np.floor(sw).astype(int)
    lh, lw = sh - h0, sw - w0
    c = lambda v, n: np.clip(v, 0, n - 1)
    xd = x.astype(np.float64)
    v00 = xd[:, :, c(h0, 14)][:, :, :, c(w0, 14)]
    v01 = xd[:, :, c(h0, 14)][:, :, :, c(w0 + 1, 14)]
    v10 = xd[:, :, c(h0 + 1, 14)][:, :, :, c(w0, 14)]
    v11 = xd[:, :, c(h0 + 1, 14)][:, :, :, c(w0 + 1, 14)]
    top = v00 + (v01 - v00) * lw
    bot = v10 + (v11 - v10) * lw
    ref = top + (bot - top) * lh[:, None]
    out = empty(ctx, (2, 5, OH, OW), "float32")
    run(ctx, wgx.shaders.upsampleBilinear2d, [T(ctx, x), [OH, OW], align, None, out])
    assert np.abs(out.numpy() - ref).max() <= 1e-5


@pytest.mark.parametrize("align", [True, False])
@pytest.mark.parametrize("shape,out_hw", [((2, 6, 32, 40), (64, 80)),    # 16-byte row groups
                                          ((16, 24, 128, 128), (256, 256)),  # DepthART decoder
                                          ((2, 5, 14, 14), (28, 21))])   # per-element path
def test_upsample_bilinear_f16(ctx, align, shape, out_hw):
    """fp16 bilinear (fp32 interpolation, one rounding) against an fp64
    restatement of the same source-index rule."""
    x = rnd(shape)
    N, C, H, W = shape
    OH, OW = out_hw
    def src(o, n_in, n_out):
        o = np.arange(o, dtype=np.float64)
        if align:
            return o * (n_in - 1) / (n_out - 1)
        return (o + 0.5) * n_in / n_out - 0.5
    sh, sw = src(OH, H, OH), src(OW, W, OW)
    h0, w0 = np.floor(sh).astype(int), np.floor(sw).astype(int)
    lh, lw = sh - h0, sw - w0
    c = lambda v, n: np.clip(v, 0, n - 1)
    xd = x.astype(np.float64)
    v00 = xd[:, :, c(h0, H)][:, :, :, c(w0, W)]
    v01 = xd[:, :, c(h0, H)][:, :, :, c(w0 + 1, W)]
    v10 = xd[:, :, c(h0 + 1, H)][:, :, :, c(w0, W)]
    v11 = xd[:, :, c(h0 + 1, H)][:, :, :, c(w0 + 1, W)]
    top = v00 + (v01 - v00) * lw
    bot = v10 + (v11 - v10) * lw
    ref = top + (bot - top) * lh[:, None]
    out = empty(ctx, (N, C, OH, OW), "float16")
    run(ctx, wgx.shaders.upsampleBilinear2d, [T(ctx, x), [OH, OW], align, None, out])
    y = out.numpy().astype(np.float64)
    assert np.abs(y - ref).max() <= 2e-3 * np.abs(ref).max()


def test_softmax_and_mean(ctx):
    x = rnd((2, 2, 40, 400))
    out = empty(ctx, x.shape, "float16")
    run(ctx, wgx.shaders.softmax, [T(ctx, x), -1, False, out])
    xd = x.astype(np.float64)
    e = np.exp(xd - xd.max(-1, keepdims=True))
    ref = e / e.sum(-1, keepdims=True)
    assert np.abs(out.numpy().astype(np.float64) - ref).max() <= 1e-3
    m = empty(ctx, (2, 2, 1, 1), "float16")
    run(ctx, wgx.shaders.meanDim, [T(ctx, x), [2, 3], True, None, m])
    np.testing.assert_allclose(m.numpy().astype(np.float64), xd.mean((2, 3), keepdims=True),
                               atol=2e-3)


def test_constant_pad_and_flat_copies(ctx):
    x = rnd((1, 3, 5, 6))
    out = empty(ctx, (1, 3, 6, 9), "float16")
    run(ctx, wgx.shaders.constantPadNd, [T(ctx, x), [1, 2, 0, 1], 0.5, out])
    ref = np.pad(x.astype(np.float32), ((0, 0), (0, 0), (0, 1), (1, 2)), constant_values=0.5)
    np.testing.assert_array_equal(out.numpy().astype(np.float32), ref)
    for shader, args_tail in [(wgx.shaders.viewCopy, [[3, 30]]), (wgx.shaders.clone, [None]),
                              (wgx.shaders.squeezeCopy, [[0]])]:
        shape = (3, 30) if shader is wgx.shaders.viewCopy else (3, 5, 6) if shader is \
            wgx.shaders.squeezeCopy else (1, 3, 5, 6)
        o = empty(ctx, shape, "float16")
        run(ctx, shader, [T(ctx, x)] + args_tail + [o])
        np.testing.assert_array_equal(o.numpy().reshape(-1), x.reshape(-1))


def attention_program(n, L, dq, dv):
    """The PSA attention spelling of the YOLO26-N export: bmm(Q, K^T) ->
    view -> softmax(-1) -> permute(0,1,3,2) -> squeeze -> bmm(V^T, P^T)."""
    h = 2
    b = n // h
    vals = [
        {"type": "tensor", "shape": [n, L, dq], "dtype": "float16", "memObjId": 0},      # 0 Q
        {"type": "tensor", "shape": [n, dq, L], "dtype": "float16", "memObjId": 1},      # 1 K^T
        {"type": "tensor", "shape": [n, dv, L], "dtype": "float16", "memObjId": 2},      # 2 V^T
        {"type": "tensor", "shape": [n, L, L], "dtype": "float16", "memObjId": 3},       # 3 S
        {"type": "list", "items": [b, h, L, L]},                                           # 4
        {"type": "tensor", "shape": [b, h, L, L], "dtype": "float16", "memObjId": 4},    # 5
        {"type": "scalar", "value": -1},                                                   # 6
        {"type": "scalar", "value": False},                                                # 7
        {"type": "tensor", "shape": [b, h, L, L], "dtype": "float16", "memObjId": 3},    # 8 P
        {"type": "list", "items": [0, 1, 3, 2]},                                           # 9
        {"type": "tensor", "shape": [b, h, L, L], "dtype": "float16", "memObjId": 4},    # 10 P^T
        {"type": "list", "items": [0]},                                                    # 11
        {"type": "tensor", "shape": [n, L, L], "dtype": "float16", "memObjId": 3},       # 12
        {"type": "tensor", "shape": [n, dv, L], "dtype": "float16", "memObjId": 5},      # 13 O^T
    ]
    chain = [
        {"name": "aten.bmm.default", "args": [0, 1, 3]},
        {"name": "aten.view_copy.default", "args": [3, 4, 5]},
        {"name": "aten._softmax.default", "args": [5, 6, 7, 8]},
        {"name": "aten.permute_copy.default", "args": [8, 9, 10]},
        {"name": "aten.view_copy.default", "args": [10, [n, L, L] and 4, 12]},
        {"name": "aten.bmm.default", "args": [2, 12, 13]},
    ]
    vals.append({"type": "list", "items": [n, L, L]})                                    # 14
    chain[4]["args"] = [10, 14, 12]
    sizes = [n * L * dq * 2, n * dq * L * 2, n * dv * L * 2, n * L * L * 2, n * L * L * 2,
             n * dv * L * 2]
    return {"version": "1", "chain": chain, "values": vals, "inputIds": [0, 1, 2],
            "outputIds": [13],
            "memoryPlan": {"pools": [{"id": i, "size": sz} for i, sz in enumerate(sizes)]}}


@pytest.mark.parametrize("n,L,dq,dv", [(4, 400, 32, 64), (2, 37, 16, 32), (6, 129, 32, 96)])
def test_fused_attention_program(ctx, n, L, dq, dv):
    q = (RNG.standard_normal((n, L, dq)) * 0.3).astype(np.float16)
    kt = (RNG.standard_normal((n, dq, L)) * 0.3).astype(np.float16)
    vt = RNG.standard_normal((n, dv, L)).astype(np.float16)
    out = empty(ctx, (n, dv, L), "float16")
    ctx.recordProgram(attention_program(n, L, dq, dv), b"", [T(ctx, q), T(ctx, kt), T(ctx, vt), out])
    # one fused kernel; the rest are input copies (inputs not bound to the
    # caller's tensors, which copy without a kernel)
    st = ctx.stats()
    assert st["kernel_launches"] == 1
    names = [n for n, _ in ctx.profile()]
    assert names.count("attention (bmm -> softmax -> bmm)") == 1
    assert all(n == "attention (bmm -> softmax -> bmm)" or n == "copy" for n in names), names
    ctx.submit()
    ctx.sync()
    s = np.matmul(q.astype(np.float64), kt.astype(np.float64))
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref = np.matmul(vt.astype(np.float64), np.swapaxes(p, 1, 2))
    err = np.abs(out.numpy().astype(np.float64) - ref).max() / np.abs(ref).max()
    assert err <= 5e-3, err


# Elementwise operators (src/shaders/add, sub, mul, sigmoid): same shapes
# (16-byte path), leading-dimension broadcasts (the repeating-operand path),
# other broadcasts and odd sizes (element paths). alpha = 1 keeps the fp32
# arithmetic exactly that of numpy (one rounding), so those cases are
# compared bit for bit; alpha = 2.5 within one fp16 ulp of the result.
@pytest.mark.gpu
@pytest.mark.parametrize("dt", [np.float16, np.float32])
@pytest.mark.parametrize("op", ["add", "sub", "mul"])
@pytest.mark.parametrize("sa,sb", [
    ((4, 3, 40), (4, 3, 40)),       # same shape
    ((6, 4, 8400), (1, 8400)),      # the detection head's anchor scaling
    ((1, 2, 24), (5, 2, 24)),       # broadcast first operand
    ((3, 5, 7), (7,)),              # odd sizes
    ((2, 3, 4, 8), (3, 1, 8)),      # broadcast in the middle
])
def test_elementwise_binary(ctx, dt, op, sa, sb):
    a, b = rnd(sa, dt), rnd(sb, dt)
    out_shape = np.broadcast_shapes(sa, sb)
    out = empty(ctx, out_shape, "float16" if dt == np.float16 else "float32")
    shader = getattr(wgx.shaders, op)
    for alpha in ([1.0, 2.5] if op != "mul" else [None]):
        args = [T(ctx, a), T(ctx, b)] + ([alpha] if alpha is not None else []) + [out]
        run(ctx, shader, args)
        af, bf = a.astype(np.float32), b.astype(np.float32)
        ref = (af + np.float32(alpha) * bf if op == "add" else
               af - np.float32(alpha) * bf if op == "sub" else af * bf).astype(dt)
        got = out.numpy().reshape(out_shape)
        if alpha in (1.0, None):
            np.testing.assert_array_equal(got, ref)
        else:
            err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
            assert np.all(err <= np.abs(ref.astype(np.float64)) * (1e-3 if dt == np.float16 else 1e-6) + 1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,scale", [((4, 80, 400), 1.0), ((3, 5, 7), 1.0),
                                         ((2, 80, 8400), 6.0)])
def test_sigmoid(ctx, shape, scale):
    """(scale 6: inputs out to about +-25, both tails saturated; the vector
    fp16 path evaluates 0.5 * tanh(x / 2) + 0.5)"""
    x = (rnd(shape).astype(np.float32) * scale).astype(np.float16)
    out = empty(ctx, shape, "float16")
    run(ctx, wgx.shaders.sigmoid, [T(ctx, x), out])
    ref = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    assert np.max(np.abs(out.numpy().reshape(shape).astype(np.float64) - ref)) <= 1e-3


def pool_chain_program(shape, K, n, idx_out=True):
    """n chained max_pool2d_with_indices (K x K, stride 1, same padding), the
    SPPF spelling; outputs every stage's values and (idx_out) the last
    indices."""
    vals = [{"type": "tensor", "shape": list(shape), "dtype": "float16", "memObjId": 0},
            {"type": "list", "items": [K, K]}, {"type": "list", "items": [1, 1]},
            {"type": "list", "items": [(K - 1) // 2] * 2}, {"type": "list", "items": [1, 1]},
            {"type": "scalar", "value": False}]
    chain, outs = [], []
    src = 0
    for s in range(n):
        v = len(vals)
        vals += [{"type": "tensor", "shape": list(shape), "dtype": "float16", "memObjId": 1 + 2 * s},
                 {"type": "tensor", "shape": list(shape), "dtype": "int32", "memObjId": 2 + 2 * s},
                 {"type": "tensorlist", "items": [v, v + 1]}]
        chain.append({"name": "aten.max_pool2d_with_indices.default",
                      "args": [src, 1, 2, 3, 4, 5, v + 2]})
        outs.append(v)
        src = v
    nb = int(np.prod(shape)) * 4
    return {"version": "1", "chain": chain, "values": vals, "inputIds": [0],
            "outputIds": outs + ([outs[-1] + 1] if idx_out else []),
            "memoryPlan": {"pools": [{"id": i, "size": nb} for i in range(1 + 2 * n)]}}


@pytest.mark.parametrize("shape,K,n,idx_out,ties", [((2, 8, 20, 20), 5, 3, True, False),
                                                    ((1, 6, 9, 13), 3, 2, True, False),
                                                    ((3, 16, 20, 20), 5, 3, False, False),
                                                    ((2, 8, 12, 16), 5, 3, False, True),
                                                    ((2, 5, 11, 7), 7, 2, False, False)])
def test_maxpool_cascade_program(ctx, shape, K, n, idx_out, ties):
    """(idx_out False: no operator reads the indices and none is a program
    output, so the cascade writes none and tracks no maximising position;
    fp16 planes of even width then take the packed half2 kernel. ties: a
    few integer values and -inf, so equal maxima are everywhere.)"""
    if ties:
        rng = np.random.default_rng(77)
        x = rng.integers(-2, 3, size=shape).astype(np.float16)
        x[rng.random(shape) < 0.1] = -np.inf
    else:
        x = rnd(shape)
    ys = [empty(ctx, shape, "float16") for _ in range(n)]
    last_idx = empty(ctx, shape, "int32")
    ctx.recordProgram(pool_chain_program(shape, K, n, idx_out), b"",
                      [T(ctx, x)] + ys + ([last_idx] if idx_out else []))
    names = ctx.command_names()
    assert sum(nm.endswith("(cascade)") for nm in names) == 1, names
    ctx.submit()
    ctx.sync()
    p = (K - 1) // 2
    cur = x
    for s in range(n):
        y, idx = maxpool_ref(cur, (K, K), (1, 1), (p, p), (1, 1), False, True)
        np.testing.assert_array_equal(ys[s].numpy().reshape(shape).astype(np.float32), y)
        cur = y.astype(np.float16)
    if idx_out:
        np.testing.assert_array_equal(last_idx.numpy().reshape(shape), idx)


@pytest.mark.parametrize("k", [1, 3])
def test_launch_count_is_the_graph_kernel_nodes(ctx, k):
    """Before the first submit the stats give the recorders' counts (a
    tensor-core convolution counts a re-layout launch, which the 1x1
    direct mode, reading NCHW through TMA, does without); after it, the
    kernel nodes of the captured graph, never more."""
    x = rnd((2, 64, 32, 32))
    w = rnd((32, 64, k, k)) * 0.05
    y = empty(ctx, (2, 32, 32, 32), "float16")
    ctx.recordShader(wgx.shaders.convolution, [T(ctx, x), T(ctx, w), None, [1, 1],
                                               [k // 2, k // 2], [1, 1], False, [0, 0], 1, y])
    before = ctx.stats()["kernel_launches"]
    ctx.submit()
    ctx.sync()
    after = ctx.stats()["kernel_launches"]
    ctx.reset()
    assert 1 <= after <= before
