"""TEST INFRASTRUCTURE ONLY: CPU executor of the reference's Program JSON.

Only tests/ and bench.py's CPU-baseline / reference legs import this module,
as the checker and the timed CPU baseline of whole-model runs; the product
never does.

It follows the reference's recordProgram (src/context.ts:219-317) and
resolveArgs (src/program.ts:188-224): one array per tensor value, constants
sliced out of the weights image (weightsOffset / weightsLength), program
inputs bound in ``inputIds`` order, each chain op reading its arguments by
value id and writing its output tensor(s) (the last argument). Every
operator computes in fp64 and rounds once to the storage dtype; the
convolutions and mm call the C restatement (wgsl_oracle.c) in its exact
mode. Operator semantics per reference shader directory:

  convolution / conv_with_clamp  src/shaders/convolution, conv-with-clamp
  mm, bmm                        src/shaders/mm, bmm
  add / sub (alpha), mul         src/shaders/add, sub, mul (numpy broadcasting)
  sigmoid, relu, hardswish       src/shaders/sigmoid, relu, hardswish
  cat, split_with_sizes_copy     src/shaders/cat, split-with-sizes
  permute_copy                   src/shaders/permute
  view/clone/squeeze/unsqueeze/prepack  flat copies (src/shaders/utils/flat-copy.ts)
  max_pool2d_with_indices        src/shaders/max-pool-2d (-65504 / -FLT_MAX start,
                                 strict '>', index ih*IW+iw, floor/ceil size)
  _softmax                       src/shaders/softmax
  upsample_nearest2d             src/shaders/upsample-nearest-2d (src = dst*in/out)
  upsample_bilinear2d            src/shaders/upsample-bilinear2d (align_corners rule)
  mean.dim                       src/shaders/mean-dim
  constant_pad_nd                src/shaders/constant-pad-nd
"""
from __future__ import annotations

import math
from typing import Dict, List, Sequence

import numpy as np

import oracle

_NP = {"float32": np.float32, "float16": np.float16, "int32": np.int32, "int8": np.int8,
       "uint8": np.uint8, "bool": np.bool_, "float64": np.float64, "int64": np.int64}


def _round(x, dt):
    return np.asarray(x).astype(dt)


def _hw(v):
    v = list(v)
    return (int(v[0]), int(v[-1]))


class _Env:
    def __init__(self, program: dict, weights: bytes):
        self.values = program["values"]
        self.arrays: Dict[int, np.ndarray] = {}
        raw = np.frombuffer(bytes(weights), dtype=np.uint8)
        for i, v in enumerate(self.values):
            if v["type"] == "tensor" and v.get("weightsOffset") is not None:
                dt = _NP[v["dtype"]]
                o, n = int(v["weightsOffset"]), int(v["weightsLength"])
                shape = [int(s) for s in v["shape"]]
                count = int(np.prod(shape)) if shape else 1
                self.arrays[i] = raw[o:o + n].view(dt)[:count].reshape(shape).copy()

    def arg(self, i: int):
        v = self.values[i]
        t = v["type"]
        if t == "tensor":
            return self.arrays[i]
        if t == "scalar":
            return v["value"]
        if t == "list":
            return [int(x) if float(x).is_integer() else float(x) for x in v["items"]]
        if t == "tensorlist":
            return [self.arrays.get(int(j)) for j in v["items"]]
        return None

    def out_ids(self, i: int) -> List[int]:
        v = self.values[i]
        return [int(j) for j in v["items"]] if v["type"] == "tensorlist" else [i]

    def spec(self, i: int):
        v = self.values[i]
        return [int(s) for s in v["shape"]], _NP[v["dtype"]]


def _maxpool(x, k, s, p, d, ceil_mode):
    N, C, H, W = x.shape
    def osz(n, kk, ss, pp, dd):
        q = (n + 2 * pp - (dd * (kk - 1) + 1)) / ss
        return max(0, int(math.ceil(q) if ceil_mode else math.floor(q)) + 1)
    OH, OW = osz(H, k[0], s[0], p[0], d[0]), osz(W, k[1], s[1], p[1], d[1])
    start = -65504.0 if x.dtype == np.float16 else -3.4028234663852886e38
    best = np.full((N, C, OH, OW), start, np.float64)
    idx = np.zeros((N, C, OH, OW), np.int32)
    xf = x.astype(np.float64)
    oh = np.arange(OH)[:, None]
    ow = np.arange(OW)[None, :]
    for kh in range(k[0]):
        ih = oh * s[0] - p[0] + kh * d[0]
        for kw in range(k[1]):
            iw = ow * s[1] - p[1] + kw * d[1]
            ok = (ih >= 0) & (ih < H) & (iw >= 0) & (iw < W)
            v = xf[:, :, np.clip(ih, 0, H - 1), np.clip(iw, 0, W - 1)]
            m = (v > best) & ok
            best = np.where(m, v, best)
            idx = np.where(m, (ih * W + iw).astype(np.int32), idx)
    return best.astype(x.dtype), idx


def _bilinear_src(o, n_in, n_out, align):
    o = np.arange(o, dtype=np.float64)
    if align:
        return o * (n_in - 1) / (n_out - 1) if n_out > 1 else np.zeros_like(o)
    return (o + 0.5) * n_in / n_out - 0.5


def _bilinear(x, OH, OW, align):
    N, C, H, W = x.shape
    sh, sw = _bilinear_src(OH, H, OH, align), _bilinear_src(OW, W, OW, align)
    h0, w0 = np.floor(sh).astype(int), np.floor(sw).astype(int)
    lh, lw = (sh - h0)[:, None], sw - w0
    c = lambda v, n: np.clip(v, 0, n - 1)
    xd = x.astype(np.float64)
    def g(hh, ww):
        return xd[:, :, c(hh, H)][:, :, :, c(ww, W)]
    top = g(h0, w0) + (g(h0, w0 + 1) - g(h0, w0)) * lw
    bot = g(h0 + 1, w0) + (g(h0 + 1, w0 + 1) - g(h0 + 1, w0)) * lw
    return (top + (bot - top) * lh).astype(x.dtype)


def _exec(env: _Env, name: str, args: Sequence[int], conv_mode: str):
    A = lambda i: env.arg(args[i])
    out_spec = env.spec(env.out_ids(args[-1])[0])
    shape, dt = out_spec
    if name in ("aten.convolution.default", "et_vk.conv_with_clamp.default"):
        x, w, b = A(0), A(1), A(2)
        stride, pad, dil, transposed = A(3), A(4), A(5), bool(A(6))
        groups = int(A(8))
        if transposed:
            return oracle.conv_transpose2d(x, w, b, _hw(stride), _hw(pad), _hw(dil), _hw(A(7)),
                                           groups, mode=conv_mode)
        if name.startswith("et_vk"):
            lo = -np.inf if A(9) is None else float(A(9))
            hi = np.inf if A(10) is None else float(A(10))
            return oracle.conv2d(x, w, b, _hw(stride), _hw(pad), _hw(dil), groups,
                                 act=oracle.ACT_CLAMP, out_min=lo, out_max=hi, mode=conv_mode,
                                 clamp_op=True)
        return oracle.conv2d(x, w, b, _hw(stride), _hw(pad), _hw(dil), groups, mode=conv_mode)
    if name == "aten.mm.default":
        return oracle.mm(A(0), A(1), conv_mode)
    if name == "aten.bmm.default":
        return _round(np.matmul(A(0).astype(np.float64), A(1).astype(np.float64)), dt)
    if name in ("aten.add.Tensor", "aten.sub.Tensor"):
        alpha = float(A(2)) if len(args) == 4 and A(2) is not None else 1.0
        a, b = A(0).astype(np.float64), A(1).astype(np.float64)
        return _round(a + alpha * b if name == "aten.add.Tensor" else a - alpha * b, dt)
    if name == "aten.mul.Tensor":
        return _round(A(0).astype(np.float64) * A(1).astype(np.float64), dt)
    if name == "aten.sigmoid.default":
        return _round(1.0 / (1.0 + np.exp(-A(0).astype(np.float64))), dt)
    if name == "aten.relu.default":
        return _round(np.maximum(A(0).astype(np.float64), 0.0), dt)
    if name == "aten.hardswish.default":
        x = A(0).astype(np.float64)
        return _round(x * np.clip(x + 3.0, 0.0, 6.0) / 6.0, dt)
    if name == "aten.cat.default":
        return np.concatenate(A(0), axis=int(A(1)))
    if name == "aten.split_with_sizes_copy.default":
        sizes = A(1)
        return np.split(A(0), np.cumsum(sizes)[:-1], axis=int(A(2)))
    if name == "aten.permute_copy.default":
        return np.ascontiguousarray(np.transpose(A(0), [int(p) for p in A(1)]))
    if name in ("aten.view_copy.default", "aten.clone.default", "aten.squeeze_copy.dims",
                "aten.unsqueeze_copy.default", "et_vk.prepack.default"):
        return A(0).reshape(shape).copy()
    if name == "aten.max_pool2d_with_indices.default":
        stride = A(2) or A(1)
        return list(_maxpool(A(0), _hw(A(1)), _hw(stride), _hw(A(3)), _hw(A(4)), bool(A(5))))
    if name == "aten._softmax.default":
        x = A(0).astype(np.float64)
        d = int(A(1))
        e = np.exp(x - x.max(axis=d, keepdims=True))
        return _round(e / e.sum(axis=d, keepdims=True), dt)
    if name == "aten.upsample_nearest2d.vec":
        x = A(0)
        H, W = x.shape[2:]
        ih = (np.arange(shape[2]) * H) // shape[2]
        iw = (np.arange(shape[3]) * W) // shape[3]
        return x[:, :, ih][:, :, :, iw].copy()
    if name == "aten.upsample_bilinear2d.vec":
        return _bilinear(A(0), shape[2], shape[3], bool(A(2)))
    if name == "aten.mean.dim":
        dims = tuple(int(d) for d in A(1))
        return _round(A(0).astype(np.float64).mean(axis=dims, keepdims=True).reshape(shape), dt)
    if name == "aten.constant_pad_nd.default":
        x, pad = A(0), A(1)
        value = float(A(2)) if len(args) == 4 and A(2) is not None else 0.0
        widths = [(0, 0)] * x.ndim
        for k in range(len(pad) // 2):
            widths[x.ndim - 1 - k] = (int(pad[2 * k]), int(pad[2 * k + 1]))
        return np.pad(x, widths, constant_values=value).astype(dt)
    raise NotImplementedError(name)


class ProgramRunner:
    """A program bound to its weights and inputs. ``run()`` executes the
    whole chain; afterwards every value is held, so ``run_op(i)`` can re-run
    chain op i alone on its recorded inputs (used to time bounded samples
    of the program's work)."""

    def __init__(self, program: dict, weights: bytes, inputs: Sequence[np.ndarray],
                 conv_mode: str = "exact"):
        self.program = program
        self.conv_mode = conv_mode
        self.env = _Env(program, weights)
        tensor_inputs = [int(i) for i in program["inputIds"]
                         if self.env.values[int(i)]["type"] == "tensor"]
        if len(tensor_inputs) != len(inputs):
            raise ValueError(f"expected {len(tensor_inputs)} inputs, got {len(inputs)}")
        for i, x in zip(tensor_inputs, inputs):
            shape, dt = self.env.spec(i)
            self.env.arrays[i] = np.asarray(x).astype(dt).reshape(shape)

    def run_op(self, index: int) -> None:
        op = self.program["chain"][index]
        res = _exec(self.env, op["name"], [int(a) for a in op["args"]], self.conv_mode)
        outs = self.env.out_ids(int(op["args"][-1]))
        res = res if isinstance(res, list) else [res]
        if len(res) != len(outs):
            raise ValueError(f"{op['name']}: {len(res)} results for {len(outs)} outputs")
        for o, r in zip(outs, res):
            shape, dt = self.env.spec(o)
            self.env.arrays[o] = np.asarray(r).astype(dt).reshape(shape)

    def run(self) -> List[np.ndarray]:
        for i in range(len(self.program["chain"])):
            self.run_op(i)
        return [self.env.arrays[int(i)] for i in self.program["outputIds"]]


def run_program(program: dict, weights: bytes, inputs: Sequence[np.ndarray],
                conv_mode: str = "exact") -> List[np.ndarray]:
    """Outputs of ``program`` (in ``outputIds`` order) for ``inputs`` (one
    array per tensor input id, in ``inputIds`` order)."""
    return ProgramRunner(program, weights, inputs, conv_mode).run()
