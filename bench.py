#!/usr/bin/env python3
"""Benchmark of the B200 hot path (one JSON line on rank 0).

Workload: BASELINE config 2, the single fp16 aten.convolution with fused
SiLU: input [8,64,160,160] N(0,1), weight [128,64,3,3] Kaiming-normal, bias
N(0,0.01), stride 1, pad 1; 8 images per GPU (weak scaling, batch-sharded,
no collective on the data path).

* ``value``: TFLOP/s of the whole job with inputs resident in HBM. One step =
  one call of the C-ABI entry point ``wgx_conv2d`` (weight packing, input
  re-layout, tcgen05 implicit GEMM + bias + SiLU epilogue). Before every
  step, outside the per-step CUDA events, L2 is flushed: a 256 MiB buffer is
  written (evicting the step's data) and a second 256 MiB buffer is read
  (forcing the write-back of those dirty lines), so the step starts with an
  L2 that holds none of its inputs and owes no write-back.
* ``e2e``: the same metric through the public API a user calls: a Program
  (convolution -> sigmoid -> mul, fused by the engine into one kernel)
  recorded with recordProgram; every step uploads the input from pinned
  host memory (setData), submits, and reads the output back (getData).
* ``roofline``: the tcgen05 conv kernel's own CUDA-event time inside the
  timed region against the measured dense bf16 peak.
* ``cpu_baseline``: the CPU port of the reference's WGSL arithmetic
  (oracle/, fp16 per-operation rounding, all host threads) on a bounded
  sample of the same workload, rank 0 at N = 1 only.

``--impl reference`` times only that CPU port of the reference
implementation (rank 0; other ranks exit), on the same metric and config.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "wgpu-executorch_b200"))

METRIC = None
with open(os.path.join(ROOT, "BASELINE.json")) as _f:
    METRIC = json.load(_f)["metric"]

B, IC, H, W, OC, K, PAD = 8, 64, 160, 160, 128, 3, 1
FLOP_PER_IMAGE = 2.0 * OC * H * W * IC * K * K
FLOP_PER_STEP = FLOP_PER_IMAGE * B
IN_BYTES, OUT_BYTES = B * IC * H * W * 2, B * OC * H * W * 2
W_BYTES, BIAS_BYTES = OC * IC * K * K * 2, OC * 2
WORKLOAD = ("BASELINE configs[1]: aten.convolution fp16 NCHW [8,64,160,160] x [128,64,3,3] "
            "stride 1 pad 1 + bias + fused SiLU, 8 images per GPU")
DATA = "synthetic: seeded N(0,1) input, Kaiming-normal weight, N(0,0.01) bias (numpy PCG64)"
FLUSH_BYTES = 256 << 20


def synthetic_inputs(seed: int):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, IC, H, W), dtype=np.float32).astype(np.float16)
    w = (rng.standard_normal((OC, IC, K, K), dtype=np.float32) *
         np.sqrt(2.0 / (IC * K * K))).astype(np.float16)
    b = (rng.standard_normal((OC,), dtype=np.float32) * 0.01).astype(np.float16)
    return x, w, b


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the conv kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "umma_conv_kernel_config2.md")
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(p).read())
    return int(m.group(1)) if m else None


# ------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = gpu_indices
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [t.strip() for t in line.split(",")]
            if len(f) < 9:
                continue
            try:
                if int(f[0]) in self.gpus:
                    rows.append(f)
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        loaded = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------ distributed
def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def reduce_max(vals, ws):
    if ws == 1:
        return vals
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def barrier(ws):
    import torch
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------- CPU baselines
def cpu_port_sample(x, w, b, target_s: float):
    """Times the CPU port of the reference WGSL arithmetic (fp16 rounding per
    operation, the conv2d-tile64-f16 summation order, sigmoid+mul in f16) on
    one image and a slice of output channels sized to ~target_s seconds.
    Returns (flops, seconds, sample text, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    x1 = x[:1]
    t0 = time.perf_counter()
    oracle.conv2d(x1, w[:8], b[:8], 1, PAD, 1, 1, act=oracle.ACT_SILU, mode="wgsl")
    t8 = time.perf_counter() - t0
    oc = int(max(1, min(OC, round(8 * target_s / max(t8, 1e-6)))))
    t0 = time.perf_counter()
    oracle.conv2d(x1, w[:oc], b[:oc], 1, PAD, 1, 1, act=oracle.ACT_SILU, mode="wgsl")
    dt = time.perf_counter() - t0
    flops = FLOP_PER_IMAGE * oc / OC
    return flops, dt, f"1 image x {oc} of {OC} output channels of the config", \
        oracle.num_threads()


def run_reference(args, ws, rank):
    if rank != 0:
        return 0
    x, w, b = synthetic_inputs(0)
    per_step = max(0.02, min(1.0, 90.0 / max(1, args.steps + args.warmup)))
    total_f, total_t, sample, threads = 0.0, 0.0, "", 1
    for i in range(args.warmup + args.steps):
        f, t, sample, threads = cpu_port_sample(x, w, b, per_step)
        if i >= args.warmup:
            total_f += f
            total_t += t
    v = total_f / total_t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": DATA,
        "config": {"workload": WORKLOAD, "global_batch": B, "per_gpu_batch": B,
                   "parallelism": "host cores of rank 0"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample + " per step (the reference's WGSL arithmetic "
                                            "restated in C; WebGPU is unavailable on this box)"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------- our engine
def program_json():
    """conv -> sigmoid -> mul over config 2 (the reference's SiLU spelling)."""
    shape_out = [B, OC, H, W]
    nbytes = B * OC * H * W * 2
    return {
        "version": "1",
        "chain": [
            {"name": "aten.convolution.default", "args": [0, 1, 2, 3, 4, 5, 6, 7, 8, 9]},
            {"name": "aten.sigmoid.default", "args": [9, 10]},
            {"name": "aten.mul.Tensor", "args": [9, 10, 11]},
        ],
        "values": [
            {"type": "tensor", "shape": [B, IC, H, W], "dtype": "float16", "memObjId": 0},
            {"type": "tensor", "shape": [OC, IC, K, K], "dtype": "float16", "weightsOffset": 0,
             "weightsLength": W_BYTES},
            {"type": "tensor", "shape": [OC], "dtype": "float16", "weightsOffset": W_BYTES,
             "weightsLength": BIAS_BYTES},
            {"type": "list", "items": [1, 1]}, {"type": "list", "items": [PAD, PAD]},
            {"type": "list", "items": [1, 1]}, {"type": "scalar", "value": False},
            {"type": "list", "items": [0, 0]}, {"type": "scalar", "value": 1},
            {"type": "tensor", "shape": shape_out, "dtype": "float16", "memObjId": 1},
            {"type": "tensor", "shape": shape_out, "dtype": "float16", "memObjId": 2},
            {"type": "tensor", "shape": shape_out, "dtype": "float16", "memObjId": 3},
        ],
        "inputIds": [0], "outputIds": [11],
        "memoryPlan": {"pools": [{"id": 0, "size": IN_BYTES}, {"id": 1, "size": nbytes},
                                 {"id": 2, "size": nbytes}, {"id": 3, "size": nbytes}]},
    }


def run_ours(args, ws, rank, local):
    import torch

    import wgx
    from wgx import _lib

    torch.cuda.set_device(local)
    x, w, b = synthetic_inputs(rank)
    ctx = wgx.WgpuExecutionContext(local)
    ext = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))

    # ---- device-resident stateless path
    prm = _lib.ConvParams(B, IC, H, W, OC, H, W, K, K, 1, 1, PAD, PAD, 1, 1, 1, 1, 1,
                          _lib.ACT_SILU, -np.inf, np.inf)
    plan = _lib.ConvPlan()
    _lib.check(_lib.lib.wgx_conv2d_plan_for(ctypes.byref(prm), ctypes.byref(plan)))
    tx = ctx.tensor("float16", x.shape).setData(x)
    tw = ctx.tensor("float16", w.shape).setData(w)
    tb = ctx.tensor("float16", b.shape).setData(b)
    tout = ctx.tensor("float16", [B, OC, H, W])
    scratch = ctx.storageBuffer(plan.scratch_bytes)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=f"cuda:{local}")
    flush_rd = torch.ones(FLUSH_BYTES // 4, dtype=torch.int32, device=f"cuda:{local}")

    def flush_l2(i):
        flush.fill_(i)
        flush_rd.max()
    pp = ctypes.byref(prm)
    args_c = (tx.data_ptr, tw.data_ptr, tb.data_ptr, tout.data_ptr, scratch.device_ptr,
              scratch.size, ctx.stream)

    def step():
        _lib.check(_lib.lib.wgx_conv2d(pp, *args_c))

    # ---- public API path (Program, host buffers)
    e2e_ctx = wgx.WgpuExecutionContext(local)
    weights = w.tobytes() + b.tobytes()
    pin_in = torch.empty(IN_BYTES, dtype=torch.uint8, pin_memory=True).numpy()
    pin_out = torch.empty(OUT_BYTES, dtype=torch.uint8, pin_memory=True).numpy()
    pin_in[:] = x.view(np.uint8).reshape(-1)
    ein = e2e_ctx.tensor("float16", [B, IC, H, W])
    eout = e2e_ctx.tensor("float16", [B, OC, H, W])
    e2e_ctx.recordProgram(program_json(), weights, [ein, eout])
    e2e_launches = e2e_ctx.stats()["kernel_launches"]

    def e2e_step():
        ein.setData(pin_in)
        e2e_ctx.submit()
        eout.getDataInto(pin_out)

    # ---- warm-up
    for i in range(args.warmup):
        with torch.cuda.stream(ext):
            flush_l2(i)
        step()
        e2e_step()
    torch.cuda.synchronize()

    gpus = [int(g) for g in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if g.strip()]
    sampler = ClockSampler(gpus if gpus else list(range(max(ws, 1)))) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)

    # ---- timed: device-resident
    barrier(ws)
    _lib.check(_lib.lib.wgx_kernel_timing(1))
    _lib.check(_lib.lib.wgx_kernel_timing_read(b"", None, None, 1))
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        with torch.cuda.stream(ext):
            flush_l2(i + 1)
            starts[i].record(ext)
        step()
        ends[i].record(ext)
    barrier(ws)
    dev_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    kms, kcnt = ctypes.c_double(), ctypes.c_int64()
    _lib.check(_lib.lib.wgx_kernel_timing_read(b"umma_conv_kernel", ctypes.byref(kms),
                                                ctypes.byref(kcnt), 1))
    _lib.check(_lib.lib.wgx_kernel_timing(0))

    # ---- timed: end to end through the public API
    barrier(ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    barrier(ws)
    e2e_s = time.perf_counter() - t0
    clocks = sampler.stop() if sampler else None

    dev_ms, e2e_s, k_ms = reduce_max([dev_ms, e2e_s, kms.value], ws)
    total_flops = FLOP_PER_STEP * args.steps * ws
    value = total_flops / (dev_ms * 1e-3) / 1e12
    e2e_value = total_flops / e2e_s / 1e12
    kernel_avg_ms = k_ms / max(1, kcnt.value)
    peak_tf, peak_hbm, peak_kind = peaks()
    achieved = FLOP_PER_STEP / (kernel_avg_ms * 1e-3) / 1e12
    traffic = profiled_traffic()

    if rank != 0:
        return 0
    cpu = None
    if ws == 1:
        f, t, sample, threads = cpu_port_sample(x, w, b, 10.0)
        cpu = {"value": f / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": sample + " (CPU port of the reference WGSL kernels, fp16 per-op "
                                  "rounding; WebGPU/SwiftShader unavailable on this box)"}
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": DATA,
        "config": {"workload": WORKLOAD, "global_batch": B * ws, "per_gpu_batch": B,
                   "accumulate": "fp32 (TMEM)",
                   "l2": "flushed before every step (256 MiB write + 256 MiB read, untimed)",
                   "parallelism": f"dp{ws} (independent batch shards, no collective)",
                   "value_path": "wgx_conv2d C-ABI call, device buffers",
                   "e2e_path": "recordProgram(conv->sigmoid->mul) + setData/submit/getData, "
                               "pinned host buffers"},
        "roofline": {"bound": "tensor", "kernel": "umma_conv_kernel", "achieved": achieved,
                     "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                     "peak_source": f"{peak_kind} bf16 dense (burst)",
                     "flop_per_launch": FLOP_PER_STEP, "launches": kcnt.value,
                     "avg_launch_ms": kernel_avg_ms,
                     "algorithmic_bytes_per_launch": IN_BYTES + OUT_BYTES + W_BYTES + BIAS_BYTES,
                     "traffic": traffic},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": IN_BYTES,
                "d2h_bytes_per_step": OUT_BYTES, "ms_per_step": e2e_s / args.steps * 1e3},
        "gpu_launches": args.steps * (plan.n_launches + e2e_launches) * ws,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    e2e_ctx.destroy()
    ctx.destroy()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
    ws, rank, local = dist_setup()
    try:
        return run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
