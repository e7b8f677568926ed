"""Host-side mirror of the wgpu-executorch TypeScript API over the wgx C ABI.

The reference's public surface (src/index.ts) is re-exported with the same
names, argument meaning and error behaviour:

* ``WgpuExecutionContext`` (src/context.ts:17): ``storageBuffer``, ``tensor``,
  ``copy``, ``recordShader``, ``recordProgram``, ``submit``, ``sync``,
  ``reset``, ``destroy``;
* ``Tensor`` (src/tensor.ts:43): ``dtype``, ``shape``, ``numel``,
  ``byteLength``, ``setData``, ``getData``;
* ``Shader`` (src/shader.ts:10-34) and the ``shaders`` / ``shaderRegistry``
  tables (src/shaders/index.ts:39-60);
* ``MAX_NDIM``, ``DTYPE_BYTESIZE``, ``GPUBufferUsage``.

Errors are raised as ``WgxError`` (an ``Exception``) carrying the reference's
message text. ``sync()`` and ``getData()`` are blocking here (the reference
returns Promises). All device work runs in the CUDA library; this module only
marshals arguments.
"""
from __future__ import annotations

import ctypes
import json
from ctypes import byref, c_int, c_int64, c_uint32, c_uint64, c_void_p
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Mapping, Sequence, Union

import numpy as np

from ._lib import (ARG_BOOL, ARG_INT_LIST, ARG_NULL, ARG_NUMBER, ARG_STRING, ARG_TENSOR,
                   ARG_TENSOR_LIST, DTYPE_BYTESIZE, DTYPE_CODE, DTYPES, WGX_ERR_INVALID, WgxArg,
                   WgxError, check,
                   device_count, lib)

MAX_NDIM = 8


class GPUBufferUsage:
    """The GPUBufferUsage bits the reference checks."""
    MAP_READ = 0x0001
    COPY_SRC = 0x0004
    COPY_DST = 0x0008
    UNIFORM = 0x0040
    STORAGE = 0x0080


class Device:
    """Stand-in for a GPUDevice: a CUDA device ordinal. ``features`` lists
    'shader-f16' because fp16 is native on sm_100a."""

    def __init__(self, ordinal: int = 0):
        self.ordinal = int(ordinal)
        self.features = frozenset({"shader-f16"})

    def createBuffer(self, size: int, usage: int) -> "Buffer":
        h = c_void_p()
        check(lib.wgx_buffer_create(self.ordinal, int(size), int(usage), byref(h)))
        return Buffer(h, owner=None)


def requestDevice(ordinal: int = 0) -> Device:
    return Device(ordinal)


class Buffer:
    """A device allocation (GPUBuffer stand-in): ``size``, ``usage``."""

    def __init__(self, handle: c_void_p, owner: Any):
        self._h = handle
        self._owner = owner  # the context when owned; keeps it alive
        size, usage, ptr = c_uint64(), c_uint32(), c_void_p()
        check(lib.wgx_buffer_info(handle, byref(size), byref(usage), byref(ptr)))
        self.size = size.value
        self.usage = usage.value
        self.device_ptr = ptr.value or 0

    def destroy(self) -> None:
        if self._owner is None and self._h:
            check(lib.wgx_buffer_destroy(self._h))
            self._h = None


def _np_bytes(src: Any) -> np.ndarray:
    if isinstance(src, (bytes, bytearray, memoryview)):
        return np.frombuffer(src, dtype=np.uint8)
    arr = np.ascontiguousarray(src)
    return arr.view(np.uint8).reshape(-1)


class Tensor:
    """Non-owning typed view over a device buffer (src/tensor.ts:43)."""

    def __init__(self, dtype: str, shape: Sequence[int], device: Device, buffer: Buffer,
                 _ctx: "WgpuExecutionContext" = None):
        self._init(dtype, shape, buffer, _ctx)

    def _init(self, dtype, shape, buffer, ctx):
        if dtype not in DTYPE_CODE:
            raise WgxError(1, f"unknown dtype {dtype}")
        shape = list(shape)
        if len(shape) > MAX_NDIM:
            raise WgxError(1, f"Tensor rank {len(shape)} exceeds maximum rank of {MAX_NDIM}")
        if any((not float(d).is_integer()) or d <= 0 for d in shape):
            raise WgxError(1, "Tensor dimensions must be positive integers")
        shape = [int(d) for d in shape]
        arr = (c_int64 * max(1, len(shape)))(*shape)
        h = c_void_p()
        check(lib.wgx_tensor_create(ctx._h if ctx is not None else None, DTYPE_CODE[dtype], arr,
                                    len(shape), buffer._h if buffer is not None else None,
                                    byref(h)))
        self._h = h
        self._ctx = ctx
        self._dtype = dtype
        self._shape = tuple(shape)
        self._numel = int(np.prod(shape)) if shape else 1
        if buffer is None:
            binfo = c_void_p()
            ptr = c_void_p()
            check(lib.wgx_tensor_info(h, None, None, None, None, byref(ptr)))
            self._buffer = None
            self._ptr = ptr.value or 0
        else:
            self._buffer = buffer
            self._ptr = buffer.device_ptr

    @classmethod
    def _create(cls, ctx, dtype, shape, buffer=None) -> "Tensor":
        t = cls.__new__(cls)
        t._init(dtype, shape, buffer, ctx)
        return t

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and lib is not None:  # module globals may be gone at interpreter exit
            lib.wgx_tensor_release(h)
            self._h = None

    @property
    def dtype(self) -> str:
        return self._dtype

    @property
    def shape(self) -> tuple:
        return self._shape

    @property
    def numel(self) -> int:
        return self._numel

    @property
    def byteLength(self) -> int:
        return self._numel * DTYPE_BYTESIZE[self._dtype]

    @property
    def data_ptr(self) -> int:
        """Device address of the tensor's first byte."""
        return self._ptr

    def setData(self, src: Any) -> "Tensor":
        b = _np_bytes(src)
        check(lib.wgx_tensor_set_data(self._h, b.ctypes.data_as(c_void_p), b.nbytes))
        return self

    def getData(self) -> bytes:
        out = np.empty(self.byteLength, dtype=np.uint8)
        check(lib.wgx_tensor_get_data(self._h, out.ctypes.data_as(c_void_p), out.nbytes))
        return out.tobytes()

    def getDataInto(self, dst: np.ndarray) -> np.ndarray:
        """getData into a caller-owned (e.g. pinned) host array."""
        check(lib.wgx_tensor_get_data(self._h, dst.ctypes.data_as(c_void_p), dst.nbytes))
        return dst

    def numpy(self) -> np.ndarray:
        npdt = {"float32": np.float32, "float16": np.float16, "float64": np.float64,
                "int32": np.int32, "int64": np.int64, "int8": np.int8, "uint8": np.uint8,
                "bool": np.bool_}[self._dtype]
        return np.frombuffer(self.getData(), dtype=npdt).reshape(self._shape)


@dataclass(frozen=True)
class Shader:
    """Operator plugin (src/shader.ts:10-34): ExecuTorch ``name``, ``code``
    (here: the CUDA kernel variants the op may launch), ``recordIn``."""
    name: str
    code: Mapping[str, str]
    recordIn: Callable[["WgpuExecutionContext", Sequence[Any]], None]


class _ArgPack:
    """Keeps the ctypes storage behind a wgx_arg array alive."""

    def __init__(self, args: Sequence[Any]):
        self.keep = []
        self.arr = (WgxArg * max(1, len(args)))()
        for i, a in enumerate(args):
            self._fill(self.arr[i], a)
        self.n = len(args)

    def _fill(self, x: WgxArg, a: Any) -> None:
        if a is None:
            x.kind = ARG_NULL
        elif isinstance(a, Tensor):
            x.kind = ARG_TENSOR
            x.v.tensor = a._h
        elif isinstance(a, (bool, np.bool_)):
            x.kind = ARG_BOOL
            x.v.boolean = int(bool(a))
        elif isinstance(a, (int, float, np.integer, np.floating)):
            x.kind = ARG_NUMBER
            x.v.number = float(a)
        elif isinstance(a, str):
            s = a.encode()
            self.keep.append(s)
            x.kind = ARG_STRING
            x.v.string = s
        elif isinstance(a, (list, tuple)):
            if all(isinstance(e, Tensor) for e in a) and len(a) > 0:
                arr = (c_void_p * len(a))(*[e._h.value for e in a])
                self.keep.append(arr)
                x.kind = ARG_TENSOR_LIST
                x.count = len(a)
                x.v.tensors = ctypes.cast(arr, ctypes.POINTER(c_void_p))
            else:
                arr = (c_int64 * max(1, len(a)))(*[int(e) for e in a])
                self.keep.append(arr)
                x.kind = ARG_INT_LIST
                x.count = len(a)
                x.v.ints = ctypes.cast(arr, ctypes.POINTER(c_int64))
        else:
            raise WgxError(1, f"unsupported argument type {type(a).__name__}")


def _native_shader(name: str, variants: Dict[str, str]) -> Shader:
    def recordIn(ctx: "WgpuExecutionContext", args: Sequence[Any]) -> None:
        ctx._assert_alive()
        pack = _ArgPack(args)
        check(lib.wgx_record_op(ctx._h, name.encode(), pack.arr, pack.n))
        ctx._keep.append(list(a for a in args if isinstance(a, Tensor)))

    return Shader(name=name, code=dict(variants), recordIn=recordIn)


_CONV_VARIANTS = {
    "umma": "tcgen05/TMEM implicit GEMM (fp16)",
    "simtGemm": "FFMA implicit GEMM (fp32)",
    "depthwise": "shared-memory row-band depthwise",
    "direct": "grouped direct conv",
    "pointwiseSingle": "1x1 single output channel",
    "transposed": "transposed conv gather",
}


class _Shaders:
    """``shaders`` namespace (src/shaders/index.ts:39-60): every operator of
    the reference's registry, recorded through wgx_record_op."""
    mm = _native_shader("aten.mm.default", {"umma": "tcgen05 GEMM (fp16)",
                                            "simt": "FFMA GEMM (fp32)"})
    convolution = _native_shader("aten.convolution.default", _CONV_VARIANTS)
    convWithClamp = _native_shader("et_vk.conv_with_clamp.default", _CONV_VARIANTS)
    add = _native_shader("aten.add.Tensor", {"elementwise": "", "broadcast": ""})
    sub = _native_shader("aten.sub.Tensor", {"elementwise": "", "broadcast": ""})
    mul = _native_shader("aten.mul.Tensor", {"elementwise": "", "broadcast": ""})
    sigmoid = _native_shader("aten.sigmoid.default", {"elementwise": ""})
    relu = _native_shader("aten.relu.default", {"elementwise": ""})
    hardswish = _native_shader("aten.hardswish.default", {"elementwise": ""})
    # linear algebra & reductions
    bmm = _native_shader("aten.bmm.default", {"simt64": "64x64 FFMA tiles"})
    meanDim = _native_shader("aten.mean.dim", {"warpPerLine": ""})
    softmax = _native_shader("aten._softmax.default", {"warpPerLine": ""})
    # pooling & resampling
    maxPool2d = _native_shader("aten.max_pool2d_with_indices.default",
                               {"plane": "whole plane in shared memory", "generic": ""})
    upsampleBilinear2d = _native_shader("aten.upsample_bilinear2d.vec", {"generic": ""})
    upsampleNearest2d = _native_shader("aten.upsample_nearest2d.vec",
                                       {"vec8": "16-byte stores", "generic": ""})
    # shape & data movement
    cat = _native_shader("aten.cat.default", {"multiCopy": "one 16-byte gather launch"})
    constantPadNd = _native_shader("aten.constant_pad_nd.default", {"generic": ""})
    splitWithSizesCopy = _native_shader("aten.split_with_sizes_copy.default",
                                        {"multiCopy": "one 16-byte gather launch"})
    permuteCopy = _native_shader("aten.permute_copy.default",
                                 {"transpose": "32x32 shared-memory tiles", "generic": ""})
    viewCopy = _native_shader("aten.view_copy.default", {"flatCopy": ""})
    clone = _native_shader("aten.clone.default", {"flatCopy": ""})
    squeezeCopy = _native_shader("aten.squeeze_copy.dims", {"flatCopy": ""})
    unsqueezeCopy = _native_shader("aten.unsqueeze_copy.default", {"flatCopy": ""})
    prepack = _native_shader("et_vk.prepack.default", {"flatCopy": ""})

    def __iter__(self):
        for k, v in vars(type(self)).items():
            if isinstance(v, Shader):
                yield k, v


shaders = _Shaders()
shaderRegistry: Dict[str, Shader] = {s.name: s for _, s in shaders}


class WgpuExecutionContext:
    """Execution context (src/context.ts:17) on one CUDA device."""

    def __init__(self, device: Union[Device, int] = 0):
        self._device = device if isinstance(device, Device) else Device(int(device))
        h = c_void_p()
        check(lib.wgx_context_create(self._device.ordinal, byref(h)))
        self._h = h
        self._keep = []  # tensors referenced by recorded commands
        self._destroyed = False

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and lib is not None:  # module globals may be gone at interpreter exit
            lib.wgx_context_release(h)
            self._h = None

    @property
    def device(self) -> Device:
        return self._device

    def _assert_alive(self):
        if self._destroyed:
            raise WgxError(3, "WgpuExecutionContext is destroyed")

    def destroy(self) -> None:
        if self._destroyed:
            return
        check(lib.wgx_context_destroy(self._h))
        self._destroyed = True
        self._keep.clear()

    def storageBuffer(self, size: int) -> Buffer:
        self._assert_alive()
        h = c_void_p()
        check(lib.wgx_storage_buffer(self._h, int(size), byref(h)))
        return Buffer(h, owner=self)

    def tensor(self, dtype: str, shape: Sequence[int], buffer: Buffer = None) -> Tensor:
        self._assert_alive()
        return Tensor._create(self, dtype, shape, buffer)

    def copy(self, src: Tensor, dst: Tensor) -> "WgpuExecutionContext":
        self._assert_alive()
        check(lib.wgx_copy(self._h, src._h, dst._h))
        self._keep.append((src, dst))
        return self

    def recordShader(self, shader: Shader, args: Sequence[Any]) -> "WgpuExecutionContext":
        self._assert_alive()
        shader.recordIn(self, args)
        return self

    def recordProgram(self, program: Union[Mapping, str, bytes], weights: Union[bytes, np.ndarray],
                      args: Sequence[Any]) -> "WgpuExecutionContext":
        self._assert_alive()
        if isinstance(program, Mapping):
            text = json.dumps(program).encode()
        elif isinstance(program, str):
            text = program.encode()
        else:
            text = bytes(program)
        w = _np_bytes(weights) if weights is not None else np.zeros(0, np.uint8)
        pack = _ArgPack(args)
        check(lib.wgx_record_program(self._h, text, len(text), w.ctypes.data_as(c_void_p),
                                     w.nbytes, pack.arr, pack.n))
        self._keep.append([a for a in args if isinstance(a, Tensor)])
        return self

    def submit(self) -> None:
        self._assert_alive()
        check(lib.wgx_submit(self._h))

    def sync(self) -> None:
        self._assert_alive()
        check(lib.wgx_sync(self._h))

    def reset(self) -> None:
        self._assert_alive()
        check(lib.wgx_reset(self._h))
        self._keep.clear()

    def stats(self) -> Dict[str, int]:
        """Recorded commands and kernel launches one submit replays."""
        n, k = c_int64(), c_int64()
        check(lib.wgx_context_stats(self._h, byref(n), byref(k)))
        return {"commands": n.value, "kernel_launches": k.value}

    def command_names(self) -> list:
        """Labels of the recorded commands in recording order (the names
        ``profile`` reports), without running them."""
        self._assert_alive()
        n = self.stats()["commands"]
        return [lib.wgx_context_command_name(self._h, i).decode() for i in range(n)]

    def profile(self, repeats: int = 1) -> list:
        """Per-command device time: the recorded commands replayed eagerly
        ``repeats`` times with CUDA events around each one. Returns
        ``[(op_name, mean_ms), ...]`` in recording order."""
        self._assert_alive()
        n = c_int(self.stats()["commands"])
        if n.value == 0:
            return []
        ms = (ctypes.c_double * n.value)()
        check(lib.wgx_context_profile(self._h, int(repeats), ms, n.value, byref(n)))
        return [(lib.wgx_context_command_name(self._h, i).decode(), ms[i]) for i in range(n.value)]

    @property
    def stream(self) -> int:
        s = c_void_p()
        check(lib.wgx_context_stream(self._h, byref(s)))
        return s.value or 0

    def pipeline(self, input: Tensor, output: Tensor, depth: int = 2) -> "Pipeline":
        """Pipelined serving steps of the recorded program (wgx_pipeline_* in
        wgx.h): each ``step(host_in, host_out)`` uploads one input, replays
        the recorded commands and downloads the output, overlapping the
        copies of neighbouring steps with this step's compute. ``input`` and
        ``output`` are the tensors the program was recorded with."""
        self._assert_alive()
        return Pipeline(self, input, output, depth)


class Pipeline:
    """Overlapped upload / compute / download of consecutive steps. The host
    arrays of a step (pinned for the copies to overlap) stay in use until
    ``depth`` further steps have been issued or ``sync()`` has returned."""

    def __init__(self, ctx: "WgpuExecutionContext", input: Tensor, output: Tensor, depth: int):
        self._ctx = ctx
        self._in_bytes = input.byteLength
        self._out_bytes = output.byteLength
        h = c_void_p()
        check(lib.wgx_pipeline_create(ctx._h, input._h, output._h, int(depth), byref(h)))
        self._h = h
        self._keep = [input, output]

    def step(self, host_in: np.ndarray, host_out: np.ndarray) -> None:
        if self._h is None:
            raise WgxError(WGX_ERR_INVALID, "pipeline is destroyed")
        if not (host_in.flags.c_contiguous and host_out.flags.c_contiguous):
            raise WgxError(WGX_ERR_INVALID, "pipeline: host arrays must be contiguous")
        if host_in.nbytes < self._in_bytes or host_out.nbytes < self._out_bytes:
            raise WgxError(WGX_ERR_INVALID, "pipeline: host array smaller than its tensor")
        check(lib.wgx_pipeline_step(self._h, host_in.ctypes.data_as(c_void_p),
                                    host_out.ctypes.data_as(c_void_p)))

    def sync(self) -> None:
        if self._h is not None:
            check(lib.wgx_pipeline_sync(self._h))

    def destroy(self) -> None:
        if self._h is not None:
            check(lib.wgx_pipeline_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


__all__ = ["WgpuExecutionContext", "Tensor", "Shader", "Buffer", "Device", "requestDevice",
           "shaders", "shaderRegistry", "MAX_NDIM", "DTYPE_BYTESIZE", "GPUBufferUsage",
           "WgxError", "device_count", "DTYPES", "Pipeline"]
