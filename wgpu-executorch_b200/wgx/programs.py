"""Program JSON transforms: fp16 conversion, batch lift, spatial re-shape and
seeded random-init weights.

A program is the reference's ExecuTorch export format (src/program.ts:26-165):
``values`` (tensor / scalar / list / tensorlist / null), ``chain`` of
``{name, args}`` with args ``[...inputs, ...outputs]``, ``inputIds``,
``outputIds`` and ``memoryPlan.pools``. Every function here takes a program
dict (and the weights image where it matters) and returns new ones; the
inputs are not modified.

* ``convert_to_fp16`` restates utils/convert_model_to_fp16.mjs:52-122
  (float32 -> float16 dtypes, 4-byte aligned fp16 weights image, pool sizes
  re-derived from their member tensors) including the DepthART decoder
  rebalance (x1/16 on the penultimate conv, x16 on the last one,
  convert_model_to_fp16.mjs:23-46).
* ``batch_lift`` turns a batch-1 export into a batch-B program by following
  the data flow from the inputs: every tensor that depends on an input gets
  its leading dimension multiplied by B, view shapes are re-derived, and the
  pools grow with their members. Constants stay shared.
* ``respatial`` changes the input's height/width of a fully convolutional
  program (DepthART 448x448 -> 256x256), re-deriving every activation's
  spatial size and the explicit ``upsample_*`` output sizes.
* ``random_init`` writes seeded Kaiming-normal weights and N(0, 0.01) biases
  into every convolution's constant slots and keeps all other constants
  (the detector's anchor and stride tables).
"""
from __future__ import annotations

import copy
import math
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np

DTYPE_BYTES = {"float32": 4, "float16": 2, "int32": 4, "int8": 1, "uint8": 1, "bool": 1,
               "float64": 8, "int64": 8}

CONV_OPS = ("aten.convolution.default", "et_vk.conv_with_clamp.default")


def _numel(shape: Sequence[int]) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def tensor_bytes(v: dict) -> int:
    return _numel(v["shape"]) * DTYPE_BYTES[v["dtype"]]


def _tensor_ids(values: List[dict], arg: int) -> List[int]:
    """The tensor value ids an argument names (a tensor or a tensorlist)."""
    if arg < 0 or arg >= len(values):
        return []
    v = values[arg]
    if v["type"] == "tensor":
        return [arg]
    if v["type"] == "tensorlist":
        return [int(i) for i in v["items"] if values[int(i)]["type"] == "tensor"]
    return []


def _is_constant(v: dict) -> bool:
    return v.get("weightsOffset") is not None and v.get("weightsLength") is not None


def _resize_pools(prog: dict) -> None:
    """Every pool at least as large as its largest member (4-byte rounded)."""
    need: Dict[int, int] = {}
    for v in prog["values"]:
        if v["type"] == "tensor" and v.get("memObjId") is not None:
            b = (tensor_bytes(v) + 3) & ~3
            need[int(v["memObjId"])] = max(need.get(int(v["memObjId"]), 0), b)
    for pool in prog["memoryPlan"]["pools"]:
        pool["size"] = max(int(pool["size"]), need.get(int(pool["id"]), 0))


# ----------------------------------------------------------------- fp16
def convert_to_fp16(program: dict, weights: bytes, depthart_rebalance: bool = False
                    ) -> Tuple[dict, bytes]:
    """float32 program + weights -> float16 program + weights, as
    utils/convert_model_to_fp16.mjs:52-122 does. ``depthart_rebalance``
    applies the DepthART decoder scaling of convert_model_to_fp16.mjs:23-46
    (and its structural checks)."""
    prog = copy.deepcopy(program)
    values = prog["values"]
    scales: Dict[int, float] = {}
    if depthart_rebalance:
        hidden, output = prog["chain"][-2], prog["chain"][-1]
        hidden_out = hidden["args"][-1]
        ok = (hidden["name"] == "et_vk.conv_with_clamp.default"
              and output["name"] == "et_vk.conv_with_clamp.default"
              and output["args"][0] == hidden_out
              and values[hidden["args"][9]].get("value") == 0
              and values[hidden["args"][10]].get("value", 0) >= 1e30
              and all(d == 1 for d in values[output["args"][1]]["shape"][2:])
              and sum(1 for op in prog["chain"] if hidden_out in op["args"][:-1]) == 1)
        if not ok:
            raise ValueError("DepthART decoder changed: verify FP16 range balancing before "
                             "conversion")
        scales[hidden["args"][1]] = 1.0 / 16
        scales[hidden["args"][2]] = 1.0 / 16
        scales[output["args"][1]] = 16.0
    src = np.frombuffer(bytes(weights), dtype=np.uint8)
    chunks: List[bytes] = []
    offset = 0
    for i, v in enumerate(values):
        if v["type"] != "tensor":
            continue
        if v["dtype"] == "float32":
            v["dtype"] = "float16"
        if _is_constant(v):
            aligned = (offset + 3) & ~3
            if aligned > offset:
                chunks.append(bytes(aligned - offset))
                offset = aligned
            n = int(v["weightsLength"]) // 4
            o = int(v["weightsOffset"])
            f32 = src[o:o + 4 * n].view(np.float32)
            s = scales.get(i, 1.0)
            if s != 1.0:
                f32 = (f32 * np.float32(s)).astype(np.float32)
            f16 = f32.astype(np.float16).tobytes()   # round to nearest even
            v["weightsOffset"] = offset
            v["weightsLength"] = len(f16)
            chunks.append(f16)
            offset += len(f16)
    if prog.get("memoryPlan") and prog["memoryPlan"].get("pools") is not None:
        sizes: Dict[int, int] = {int(p["id"]): 0 for p in prog["memoryPlan"]["pools"]}
        for v in values:
            if v["type"] == "tensor" and v.get("memObjId") is not None:
                b = (_numel(v["shape"]) * DTYPE_BYTES.get(v["dtype"], 2) + 3) & ~3
                sizes[int(v["memObjId"])] = max(sizes.get(int(v["memObjId"]), 0), b)
        for p in prog["memoryPlan"]["pools"]:
            p["size"] = sizes.get(int(p["id"])) or math.ceil(int(p["size"]) / 2)
    return prog, b"".join(chunks)


# ----------------------------------------------------------- data flow
def _dependent_values(prog: dict) -> Set[int]:
    """Tensor ids that depend on a program input (the last argument of each
    op is its output, a tensor or a tensorlist)."""
    values = prog["values"]
    dep: Set[int] = set()
    for i in prog["inputIds"]:
        dep.update(_tensor_ids(values, int(i)))
    for op in prog["chain"]:
        ins = [t for a in op["args"][:-1] for t in _tensor_ids(values, int(a))]
        if any(t in dep for t in ins):
            dep.update(_tensor_ids(values, int(op["args"][-1])))
    return dep


def _replace_list(prog: dict, op: dict, pos: int, items: List[int]) -> None:
    """Point argument ``pos`` of ``op`` at a fresh list value."""
    prog["values"].append({"type": "list", "items": [int(x) for x in items]})
    op["args"][pos] = len(prog["values"]) - 1


def _dim_arg(prog: dict, op: dict, pos: int, ndim: int) -> int:
    v = prog["values"][op["args"][pos]]
    d = int(v["value"]) if v["type"] == "scalar" else 0
    return d + ndim if d < 0 else d


def batch_lift(program: dict, batch: int) -> dict:
    """A batch-``batch`` version of a batch-1 program.

    Every input-dependent tensor's leading dimension is multiplied by
    ``batch`` (a [1,C,H,W] activation becomes [B,C,H,W]; the [2,400,32]
    attention operand squeezed out of [1,2,...] becomes [2B,400,32], which
    keeps the images outermost in memory). ``view_copy`` shapes follow. Ops
    that would mix images along the leading dimension (cat / split /
    softmax / mean over dim 0, a permute that moves dim 0) are rejected.
    """
    if batch < 1:
        raise ValueError("batch must be >= 1")
    prog = copy.deepcopy(program)
    if batch == 1:
        return prog
    values = prog["values"]
    dep = _dependent_values(prog)
    for i in prog["inputIds"]:
        v = values[int(i)]
        if v["type"] == "tensor" and int(v["shape"][0]) != 1:
            raise ValueError(f"batch_lift: input {i} has leading dimension {v['shape'][0]}, "
                             "expected 1")
    for op in prog["chain"]:
        name, args = op["name"], op["args"]
        ins = [t for a in args[:-1] for t in _tensor_ids(values, int(a))]
        if not any(t in dep for t in ins):
            continue
        x = values[args[0]] if values[args[0]]["type"] == "tensor" else None
        nd = len(x["shape"]) if x else 0
        if name == "aten.view_copy.default":
            items = [int(s) for s in values[args[1]]["items"]]
            if items and items[0] > 0:
                items[0] *= batch
            _replace_list(prog, op, 1, items)
        elif name in ("aten.cat.default",):
            first = values[_tensor_ids(values, args[0])[0]]
            if _dim_arg(prog, op, 1, len(first["shape"])) == 0:
                raise ValueError("batch_lift: cat along the batch dimension")
        elif name == "aten.split_with_sizes_copy.default":
            if _dim_arg(prog, op, 2, nd) == 0:
                raise ValueError("batch_lift: split along the batch dimension")
        elif name == "aten._softmax.default":
            if _dim_arg(prog, op, 1, nd) == 0:
                raise ValueError("batch_lift: softmax along the batch dimension")
        elif name == "aten.permute_copy.default":
            perm = [int(p) % nd for p in values[args[1]]["items"]]
            if perm[0] != 0:
                raise ValueError("batch_lift: permute moves the batch dimension")
        elif name == "aten.mean.dim":
            dims = [int(d) % nd for d in values[args[1]]["items"]]
            if 0 in dims:
                raise ValueError("batch_lift: mean over the batch dimension")
        elif name == "aten.unsqueeze_copy.default":
            if _dim_arg(prog, op, 1, nd + 1) == 0:
                raise ValueError("batch_lift: unsqueeze in front of the batch dimension")
    for t in dep:
        v = values[t]
        if not v["shape"]:
            raise ValueError(f"batch_lift: scalar tensor {t} depends on the input")
        v["shape"] = [int(v["shape"][0]) * batch] + [int(s) for s in v["shape"][1:]]
    _resize_pools(prog)
    return prog


# ------------------------------------------------------------ spatial
def _conv_out(n: int, k: int, s: int, p: int, d: int) -> int:
    return (n + 2 * p - d * (k - 1) - 1) // s + 1


def _hw(values: List[dict], idx: int) -> Tuple[int, int]:
    items = [int(x) for x in values[idx]["items"]]
    return (items[0], items[1] if len(items) > 1 else items[0])


def respatial(program: dict, height: int, width: int) -> dict:
    """The program for a ``height`` x ``width`` input (fully convolutional
    programs: convolutions, elementwise ops, pooling and upsampling).

    Activation sizes are propagated op by op from the new input size; an
    ``upsample_*`` op with an explicit output size keeps its ratio to the
    input it upsamples, which must come out integral.
    """
    prog = copy.deepcopy(program)
    values = prog["values"]
    (inp,) = [int(i) for i in prog["inputIds"] if values[int(i)]["type"] == "tensor"]
    old_in = values[inp]["shape"]
    if len(old_in) != 4:
        raise ValueError("respatial: input must be NCHW")
    new_shape: Dict[int, List[int]] = {inp: [old_in[0], old_in[1], int(height), int(width)]}

    def cur(t: int) -> List[int]:
        return new_shape.get(t, [int(s) for s in values[t]["shape"]])

    for op in prog["chain"]:
        name, args = op["name"], op["args"]
        outs = _tensor_ids(values, int(args[-1]))
        ins = [t for a in args[:-1] for t in _tensor_ids(values, int(a))]
        if not any(t in new_shape for t in ins):
            continue
        x = cur(args[0])
        if name in CONV_OPS:
            w = values[args[1]]["shape"]
            (sh, sw), (ph, pw), (dh, dw) = (_hw(values, args[3]), _hw(values, args[4]),
                                            _hw(values, args[5]))
            if values[args[6]].get("value"):
                raise ValueError("respatial: transposed convolution")
            oh = _conv_out(x[2], int(w[2]), sh, ph, dh)
            ow = _conv_out(x[3], int(w[3]), sw, pw, dw)
            shape = [x[0], int(values[outs[0]]["shape"][1]), oh, ow]
        elif name in ("aten.upsample_bilinear2d.vec", "aten.upsample_nearest2d.vec"):
            size_pos = 1
            old_x = values[args[0]]["shape"]
            v = values[args[size_pos]]
            if v["type"] == "list":
                oh0, ow0 = (int(s) for s in v["items"])
                if (oh0 * x[2]) % old_x[2] or (ow0 * x[3]) % old_x[3]:
                    raise ValueError("respatial: upsample size does not scale to an integer")
                oh, ow = oh0 * x[2] // old_x[2], ow0 * x[3] // old_x[3]
                _replace_list(prog, op, size_pos, [oh, ow])
            else:
                f = values[args[-2]]["items"]
                oh, ow = int(math.floor(x[2] * float(f[0]))), int(math.floor(x[3] * float(f[1])))
            shape = [x[0], x[1], oh, ow]
        elif name in ("aten.add.Tensor", "aten.sub.Tensor", "aten.mul.Tensor", "aten.relu.default",
                      "aten.sigmoid.default", "aten.hardswish.default", "aten.clone.default"):
            shape = list(x)
            for t in ins:
                s = cur(t)
                if len(s) == len(shape):
                    shape = [max(a, b) if 1 in (a, b) else a for a, b in zip(shape, s)]
        else:
            raise ValueError(f"respatial: {name} is not supported")
        for t in outs:
            new_shape[t] = shape
    for t, s in new_shape.items():
        values[t]["shape"] = s
    _resize_pools(prog)
    return prog


# ------------------------------------------------------------ weights
def random_init(program: dict, weights: bytes, seed: int = 0) -> bytes:
    """A weights image with every convolution's weight drawn from
    N(0, 2 / fan_in) (Kaiming normal, fan_in = IC/groups * KH * KW) and its
    bias from N(0, 0.01^2), seeded; other constants are kept."""
    out = bytearray(weights)
    values = program["values"]
    rng = np.random.default_rng(seed)
    done: Set[int] = set()
    for op in program["chain"]:
        if op["name"] not in CONV_OPS:
            continue
        for pos in (1, 2):
            vid = int(op["args"][pos])
            v = values[vid]
            if vid in done or v["type"] != "tensor" or not _is_constant(v):
                continue
            done.add(vid)
            n = _numel(v["shape"])
            if pos == 1:
                fan_in = _numel(v["shape"][1:])
                data = rng.standard_normal(n) * math.sqrt(2.0 / fan_in)
            else:
                data = rng.standard_normal(n) * 0.01
            dt = np.float16 if v["dtype"] == "float16" else np.float32
            raw = data.astype(dt).tobytes()
            o = int(v["weightsOffset"])
            if len(raw) != int(v["weightsLength"]):
                raise ValueError(f"random_init: value {vid} length mismatch")
            out[o:o + len(raw)] = raw
    return bytes(out)
