"""Benchmark of the b200 linear-algebra path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload gemv_dot|gemm1024|batched|norm|norm_rows|gemm_f32|gemm_f64|vecmat
                                |elementwise|reduce]

Default workload = BASELINE config 2 (the metric's memory-bound BLAS-1/2
config): one step is y = A @ x with A 16384x16384 float32 plus one DOT of two
2^26 float32 vectors, inputs uniform[-1,1] from default_rng(1) (A, x, then the
two DOT vectors from the same stream).  value = algorithmic bytes / time
(GB/s), whole job over all ranks; inputs (1.6 GB) are far larger than L2.

Other workloads are BASELINE configs 1, 3, 4 and 5 (TFLOP/s or GB/s), and
vecmat: x @ A (vector @ matrix, float32 16384^2, GB/s), and the operations
around the path on 2^28 float32 values: elementwise (x + y) and reduce (sum).  Sharded
ones split across ranks (batch dim for config 3, row blocks of A for config 5,
contiguous slices + NCCL merge for config 4); config 1 and 2 run one replica
per rank.  Multi-GPU: one process per GPU under torchrun; barriers and the
max-over-ranks time go through a gloo process group (host side only), data
collectives through the library's own NCCL communicator.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "open-pacho_b200"))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# Tensor-pipe ceilings for the GEMM workloads, measured on this pool's B200 with
# cuBLAS (8192^3, best of 10): TF32 737.7 TFLOP/s -> 3xTF32 ceiling 245.9 logical;
# FP64 DGEMM 35.5 TFLOP/s.  MEASURED_PEAKS.json carries bf16 only.
TENSOR_CEILINGS = {
    "gemm1024": (737.7 / 3, "measured cuBLAS TF32 / 3"),
    "gemm_f32": (737.7 / 3, "measured cuBLAS TF32 / 3"),
    "batched": (737.7 / 3, "measured cuBLAS TF32 / 3"),
    "gemm_f64": (35.5, "measured cuBLAS DGEMM"),
}
L2_BYTES = 126 * 1024 * 1024


# ------------------------------------------------------------- workloads --

def gen_gemv_dot():
    rng = np.random.default_rng(1)
    A = rng.uniform(-1, 1, (16384, 16384)).astype(np.float32)
    x = rng.uniform(-1, 1, 16384).astype(np.float32)
    u = rng.uniform(-1, 1, 1 << 26).astype(np.float32)
    v = rng.uniform(-1, 1, 1 << 26).astype(np.float32)
    return A, x, u, v


def gen_gemm(seed, n, dtype):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, n), dtype=np.float32 if dtype == np.float32 else np.float64),
            rng.standard_normal((n, n), dtype=np.float32 if dtype == np.float32 else np.float64))


def gen_batched():
    rng = np.random.default_rng(2)
    A = rng.standard_normal((8, 16, 512, 256)).astype(np.float32)
    B = rng.standard_normal((1, 16, 256, 384)).astype(np.float32)
    return A, B


def gen_norm(n=1 << 28, dtype=np.float32, span=35):
    rng = np.random.default_rng(3)
    out = np.empty(n, dtype)
    step = 1 << 24
    for i in range(0, n, step):  # bounded host memory
        m = min(step, n - i)
        out[i:i + m] = rng.standard_normal(m) * 10.0 ** rng.uniform(-span, span, m)
    return out


# ------------------------------------------------------------- plumbing --

class Dist:
    """Rank info + host-side (gloo) barrier/max for torchrun launches."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
            # Bound the library's own collective waits too (default 300 s).
            os.environ.setdefault("PB_COMM_TIMEOUT_S", "60")
            self.dist = dist
            self.pg = True

    def barrier(self):
        if self.pg:
            self.dist.barrier()

    def max(self, value: float) -> float:
        if not self.pg:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def broadcast_bytes(self, data: bytes | None, size: int) -> bytes:
        if not self.pg:
            return data
        import torch

        t = torch.zeros(size, dtype=torch.uint8)
        if self.rank == 0:
            t[:] = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        self.dist.broadcast(t, 0)
        return bytes(t.numpy().tobytes())

    def all_gather_bytes(self, data: bytes, size: int) -> list[bytes]:
        """Every rank's `size`-byte record, in rank order."""
        if not self.pg:
            return [data]
        import torch

        t = torch.zeros(size, dtype=torch.uint8)
        t[: len(data)] = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        out = [torch.zeros(size, dtype=torch.uint8) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [bytes(o.numpy().tobytes()) for o in out]

    def close(self):
        if self.pg:
            self.dist.destroy_process_group()


class Clocks:
    """Samples nvidia-smi during the timed region."""

    def __init__(self, index):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def traffic_per_launch(kernel: str, workload: str):
    """DRAM bytes (read + write) per launch from the committed ncu summary."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(f"{workload}:{kernel}")
    return None if entry is None else entry.get("dram_bytes_per_launch")


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "source": "measured"}
    return {**PEAKS_FALLBACK, "source": "fallback"}


# ----------------------------------------------------------- b200 arm --

class Gpu:
    def __init__(self, device):
        from pacho_b200 import B200Backend, _lib

        self.lib = _lib
        self.backend = B200Backend(device)
        self.raw = self.backend._lib
        self.ctx = self.backend._ctx

    def upload(self, host):
        return self.backend.upload(host)

    def empty(self, shape, dtype):
        return self.backend.empty(shape, dtype)

    def check(self, status, what):
        self.lib.check(status, what)

    def busy(self, fn, dist, seconds=0.5):
        """Untimed steps for about `seconds`, so the clock sampler sees the GPU
        under this workload's load before the timed region.  The step count is
        calibrated per rank and agreed (max) across ranks: steps may contain
        collectives, so every rank must run exactly the same number."""
        t0 = time.perf_counter()
        for _ in range(8):
            fn()
        self.check(self.raw.pb_sync(self.ctx, 0), "sync")
        per8 = max(time.perf_counter() - t0, 1e-6)
        rounds = int(dist.max(float(min(max(1, int(seconds / per8)), 4096))))
        for _ in range(rounds):
            for _ in range(8):
                fn()
            self.check(self.raw.pb_sync(self.ctx, 0), "sync")

    def timer(self, fn, reps):
        self.check(self.raw.pb_sync(self.ctx, 0), "sync")
        self.check(self.raw.pb_timer_start(self.ctx, 0), "timer")
        for _ in range(reps):
            fn()
        ms = C.c_float()
        self.check(self.raw.pb_timer_stop(self.ctx, 0, C.byref(ms)), "timer")
        return ms.value / 1e3

    def launches(self):
        return self.backend.launch_count()


def p_(buf):
    return C.c_void_p(buf.ptr)


def run_gemv_dot(gpu: Gpu, args, dist: Dist, result: dict):
    A, x, u, v = gen_gemv_dot()
    M, K = A.shape
    n = u.size
    bytes_gemv = 4 * (M * K + K + M)
    bytes_dot = 2 * 4 * n
    step_bytes = bytes_gemv + bytes_dot
    dA, dx, du, dv = (gpu.upload(t) for t in (A, x, u, v))
    dy, dd = gpu.empty((M,), np.float32), gpu.empty((1,), np.float32)
    raw, ctx, F32 = gpu.raw, gpu.ctx, gpu.lib.PB_F32

    def gemv():
        gpu.check(raw.pb_gemv(ctx, 0, F32, M, K, p_(dA), p_(dx), p_(dy)), "pb_gemv")

    def dot():
        gpu.check(raw.pb_dot(ctx, 0, F32, n, p_(du), p_(dv), p_(dd)), "pb_dot")

    def step():
        gemv()
        dot()

    for _ in range(args.warmup):
        step()
    dist.barrier()
    with Clocks(gpu.backend.ordinal) as clocks:
        gpu.busy(step, dist)
        l0 = gpu.launches()
        seconds = gpu.timer(step, args.steps)
    launches = gpu.launches() - l0
    seconds = dist.max(seconds)
    # Per-kernel live timing for the roofline (dominant kernel: GEMV, 1.07 GB/launch).
    t_gemv = gpu.timer(gemv, args.steps) / args.steps
    t_dot = gpu.timer(dot, args.steps) / args.steps

    # Parity spot check of this run's outputs against the oracle (rank 0).
    y = np.empty(M, np.float32)
    d = np.empty(1, np.float32)
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(y.ctypes.data), p_(dy), y.nbytes), "d2h")
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(d.ctypes.data), p_(dd), 4), "d2h")

    # End to end through the public API: pinned host inputs copied in every step,
    # results read back every step.
    e2e = e2e_gemv_dot(gpu, A, x, u, v, args, dist)

    total = step_bytes * args.steps * dist.world
    result.update({
        "metric": "GEMV 16384x16384 + DOT 2^26 float32 HBM throughput",
        "value": total / seconds / 1e9,
        "unit": "GB/s",
        "ms_per_step": seconds / args.steps * 1e3,
        "scaling": "weak",
        "dtype": "f32",
        "config": {"workload": "BASELINE config 2: y = A@x (A 16384x16384 f32) + DOT of two 2^26 f32 "
                               "vectors, U[-1,1], default_rng(1)",
                   "step_bytes": step_bytes, "parallelism": f"replicas x{dist.world}",
                   "l2": "inputs (1.6 GB) larger than the 126 MB L2; no flush needed"},
        "clocks": clocks.summary(),
        "gpu_launches": launches,
        "kernels": {"gemv_ms": t_gemv * 1e3, "gemv_gbs": bytes_gemv / t_gemv / 1e9,
                    "dot_ms": t_dot * 1e3, "dot_gbs": bytes_dot / t_dot / 1e9},
        "roofline_kernel": ("gemv", bytes_gemv, t_gemv),
        "e2e": e2e,
        "_check": ("gemv_dot", A, x, u, v, y, d),
    })


def e2e_gemv_dot(gpu, A, x, u, v, args, dist):
    raw, ctx, F32 = gpu.raw, gpu.ctx, gpu.lib.PB_F32
    host = [np.ascontiguousarray(t) for t in (A, x, u, v)]
    for t in host:
        gpu.check(raw.pb_host_register(C.c_void_p(t.ctypes.data), t.nbytes), "pin")
    y = np.empty(A.shape[0], np.float32)
    d = np.empty(1, np.float32)
    for t in (y, d):
        gpu.check(raw.pb_host_register(C.c_void_p(t.ctypes.data), t.nbytes), "pin")
    dev = [gpu.empty(t.shape, t.dtype) for t in host]
    dy, dd = gpu.empty(y.shape, np.float32), gpu.empty((1,), np.float32)
    M, K = A.shape

    def step():
        for h, dbuf in zip(host, dev):
            gpu.check(raw.pb_h2d(ctx, 0, p_(dbuf), C.c_void_p(h.ctypes.data), h.nbytes, 0), "h2d")
        gpu.check(raw.pb_gemv(ctx, 0, F32, M, K, p_(dev[0]), p_(dev[1]), p_(dy)), "gemv")
        gpu.check(raw.pb_dot(ctx, 0, F32, u.size, p_(dev[2]), p_(dev[3]), p_(dd)), "dot")
        gpu.check(raw.pb_d2h_async(ctx, 0, C.c_void_p(y.ctypes.data), p_(dy), y.nbytes), "d2h")
        gpu.check(raw.pb_d2h_async(ctx, 0, C.c_void_p(d.ctypes.data), p_(dd), 4), "d2h")

    step()
    dist.barrier()
    seconds = dist.max(gpu.timer(step, args.steps))
    for t in (*host, y, d):
        raw.pb_host_unregister(C.c_void_p(t.ctypes.data))
    step_bytes = 4 * (A.size + x.size + A.shape[0]) + 8 * u.size
    h2d = sum(t.nbytes for t in host)
    return {"value": step_bytes * args.steps * dist.world / seconds / 1e9, "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": y.nbytes + 4,
            "ms_per_step": seconds / args.steps * 1e3}


def run_gemm(gpu: Gpu, args, dist: Dist, result: dict, which: str):
    raw, ctx = gpu.raw, gpu.ctx
    if which == "gemm1024":
        A, B = gen_gemm(0, args.n or 1024, np.float32)
        dtype, shard = np.float32, False
    elif which == "gemm_f32":
        A, B = gen_gemm(4, args.n or 16384, np.float32)
        dtype, shard = np.float32, True
    else:
        A, B = gen_gemm(4, args.n or 8192, np.float64)
        dtype, shard = np.float64, True
    n = A.shape[0]
    rows = n // dist.world if shard else n
    r0 = dist.rank * rows if shard else 0
    Aloc = np.ascontiguousarray(A[r0:r0 + rows])
    dA, dB = gpu.upload(Aloc), gpu.upload(B)
    dC = gpu.empty((rows, n), dtype)
    code = gpu.lib.dtype_code(dtype)
    ns = gpu.lib.i64_array([])

    def step():
        gpu.check(raw.pb_gemm(ctx, 0, code, 0, ns, ns, ns, rows, n, n, p_(dA), p_(dB), p_(dC)), "gemm")

    for _ in range(args.warmup):
        step()
    dist.barrier()
    with Clocks(gpu.backend.ordinal) as clocks:
        gpu.busy(step, dist)
        l0 = gpu.launches()
        seconds = gpu.timer(step, args.steps)
    launches = gpu.launches() - l0
    seconds = dist.max(seconds)
    flops = 2.0 * rows * n * n
    total = flops * args.steps * dist.world
    Cl = np.empty((rows, n), dtype)
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(Cl.ctypes.data), p_(dC), Cl.nbytes), "d2h")
    result.update({
        "metric": f"{np.dtype(dtype).name} GEMM {n}^3 TFLOP/s",
        "value": total / seconds / 1e12, "unit": "TFLOP/s",
        "ms_per_step": seconds / args.steps * 1e3,
        "scaling": "strong" if shard else "weak",
        "dtype": "f32 (3xTF32)" if dtype == np.float32 else "f64",
        "config": {"workload": f"GEMM {n}^3 {np.dtype(dtype).name}",
                   "parallelism": f"row blocks x{dist.world}" if shard else f"replicas x{dist.world}"},
        "clocks": clocks.summary(), "gpu_launches": launches,
        "roofline_kernel": ("gemm", flops, seconds / args.steps),
        "_check": ("gemm", Aloc, B, Cl),
    })


def run_vecmat(gpu: Gpu, args, dist: Dist, result: dict):
    """x @ A (vector @ matrix, float32): the skinny kernel, HBM bound."""
    raw, ctx = gpu.raw, gpu.ctx
    n = args.n or 16384
    rng = np.random.default_rng(5)
    A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    dx, dA = gpu.upload(x), gpu.upload(A)
    dy = gpu.empty((n,), np.float32)
    ns = gpu.lib.i64_array([])
    F32 = gpu.lib.PB_F32

    def step():
        gpu.check(raw.pb_gemm(ctx, 0, F32, 0, ns, ns, ns, 1, n, n, p_(dx), p_(dA), p_(dy)), "gemm")

    for _ in range(args.warmup):
        step()
    dist.barrier()
    with Clocks(gpu.backend.ordinal) as clocks:
        gpu.busy(step, dist)
        l0 = gpu.launches()
        seconds = gpu.timer(step, args.steps)
    launches = gpu.launches() - l0
    seconds = dist.max(seconds)
    step_bytes = 4 * (n * n + 2 * n)
    y = np.empty(n, np.float32)
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(y.ctypes.data), p_(dy), y.nbytes), "d2h")
    result.update({
        "metric": f"vector @ matrix ({n} @ {n}x{n}) float32 HBM throughput",
        "value": step_bytes * args.steps * dist.world / seconds / 1e9, "unit": "GB/s",
        "ms_per_step": seconds / args.steps * 1e3, "scaling": "weak", "dtype": "f32",
        "config": {"workload": f"x @ A, A {n}x{n} f32, U[-1,1], default_rng(5)",
                   "step_bytes": step_bytes, "parallelism": f"replicas x{dist.world}",
                   "l2": "A (1.07 GB) larger than the 126 MB L2; no flush needed"},
        "clocks": clocks.summary(), "gpu_launches": launches,
        "roofline_kernel": ("skinny", step_bytes, seconds / args.steps),
        "_check": ("gemm", x.reshape(1, n), A, y.reshape(1, n)),
    })


def run_around(gpu: Gpu, args, dist: Dist, result: dict, which: str):
    """Operations around the path on 2^28 float32 values (HBM bound):
    elementwise add of two arrays (pb_elementwise) or their full sum (pb_reduce)."""
    raw, ctx = gpu.raw, gpu.ctx
    n = args.n or (1 << 28)
    rng = np.random.default_rng(6)
    x = rng.standard_normal(n, dtype=np.float32)
    dx = gpu.upload(x)
    F32 = gpu.lib.PB_F32
    y = None
    if which == "elementwise":
        y = rng.standard_normal(n, dtype=np.float32)
        dy, dz = gpu.upload(y), gpu.empty((n,), np.float32)
        ptrs = (C.c_void_p * 2)(dx.ptr, dy.ptr)
        codes = (C.c_int * 2)(F32, F32)
        strides, shape = gpu.lib.i64_array([1, 1]), gpu.lib.i64_array([n])
        add = gpu.lib.EW_OPS["add"]

        def step():
            gpu.check(raw.pb_elementwise(ctx, 0, add, 2, ptrs, codes, strides, 1, shape, F32,
                                         p_(dz)), "elementwise")
        step_bytes = 12 * n
    else:
        dz = gpu.empty((1,), np.float32)
        shape = gpu.lib.i64_array([n])

        def step():
            gpu.check(raw.pb_reduce(ctx, 0, gpu.lib.PB_REDUCE_SUM, F32, p_(dx), 1, shape, 1, F32,
                                    p_(dz)), "reduce")
        step_bytes = 4 * n + 4

    for _ in range(args.warmup):
        step()
    dist.barrier()
    with Clocks(gpu.backend.ordinal) as clocks:
        gpu.busy(step, dist)
        l0 = gpu.launches()
        seconds = gpu.timer(step, args.steps)
    launches = gpu.launches() - l0
    seconds = dist.max(seconds)
    z = np.empty(n if which == "elementwise" else 1, np.float32)
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(z.ctypes.data), p_(dz), z.nbytes), "d2h")
    what = "elementwise add of two float32 arrays" if which == "elementwise" else "sum of float32 values"
    result.update({
        "metric": f"{what} (n = {n}) HBM throughput",
        "value": step_bytes * args.steps * dist.world / seconds / 1e9, "unit": "GB/s",
        "ms_per_step": seconds / args.steps * 1e3, "scaling": "weak", "dtype": "f32",
        "config": {"workload": f"{which}, n = {n} float32, N(0,1), default_rng(6)",
                   "step_bytes": step_bytes, "parallelism": f"replicas x{dist.world}",
                   "l2": "operands (1 GB each) larger than the 126 MB L2; no flush needed"},
        "clocks": clocks.summary(), "gpu_launches": launches,
        "roofline_kernel": (which, step_bytes, seconds / args.steps),
        "_check": (which, x, y, z),
    })


def run_batched(gpu: Gpu, args, dist: Dist, result: dict):
    raw, ctx = gpu.raw, gpu.ctx
    A, B = gen_batched()
    per = A.shape[0] // dist.world
    Aloc = np.ascontiguousarray(A[dist.rank * per:(dist.rank + 1) * per])
    dA, dB = gpu.upload(Aloc), gpu.upload(B)
    batch = (per, 16)
    dC = gpu.empty(batch + (512, 384), np.float32)
    L = gpu.lib

    def step():
        gpu.check(raw.pb_gemm(ctx, 0, L.PB_F32, 2, L.i64_array(batch), L.i64_array([16, 1]),
                              L.i64_array([0, 1]), 512, 384, 256, p_(dA), p_(dB), p_(dC)), "gemm")

    for _ in range(args.warmup):
        step()
    dist.barrier()
    with Clocks(gpu.backend.ordinal) as clocks:
        gpu.busy(step, dist)
        l0 = gpu.launches()
        seconds = gpu.timer(step, args.steps)
    launches = gpu.launches() - l0
    seconds = dist.max(seconds)
    flops = 2.0 * per * 16 * 512 * 384 * 256
    Cl = np.empty(batch + (512, 384), np.float32)
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(Cl.ctypes.data), p_(dC), Cl.nbytes), "d2h")
    result.update({
        "metric": "batched broadcast GEMM (8,16,512,256)@(1,16,256,384) f32 TFLOP/s",
        "value": flops * args.steps * dist.world / seconds / 1e12, "unit": "TFLOP/s",
        "ms_per_step": seconds / args.steps * 1e3, "scaling": "strong", "dtype": "f32 (3xTF32)",
        "config": {"workload": "BASELINE config 3", "parallelism": f"batch split x{dist.world}"},
        "clocks": clocks.summary(), "gpu_launches": launches,
        "roofline_kernel": ("gemm", flops, seconds / args.steps),
        "_check": ("gemm", Aloc, B, Cl),
    })


def run_norm(gpu: Gpu, args, dist: Dist, result: dict, rows: bool):
    raw, ctx = gpu.raw, gpu.ctx
    dtype = np.float64 if args.dtype == "f64" else np.float32
    span = 300 if dtype == np.float64 else 35
    n = 1 << 28
    x = gen_norm(n, dtype, span)
    code = gpu.lib.dtype_code(dtype)
    if rows:
        shape = (65536, 4096)
        nrows = shape[0] // dist.world
        xl = np.ascontiguousarray(x.reshape(shape)[dist.rank * nrows:(dist.rank + 1) * nrows])
        dx, dout = gpu.upload(xl), gpu.empty((nrows,), dtype)

        def step():
            gpu.check(raw.pb_norm(ctx, 0, code, nrows, shape[1], 1, p_(dx), p_(dout)), "norm")
    else:
        per = n // dist.world
        xl = np.ascontiguousarray(x[dist.rank * per:(dist.rank + 1) * per])
        dx, dout = gpu.upload(xl), gpu.empty((1,), dtype)
        if dist.world > 1:
            uid = C.create_string_buffer(128)
            if dist.rank == 0:
                gpu.check(raw.pb_comm_unique_id(uid), "unique id")
            data = dist.broadcast_bytes(uid.raw if dist.rank == 0 else None, 128)
            gpu.check(raw.pb_comm_init(ctx, 0, dist.world, dist.rank, data), "comm init")
            # Peer mailboxes: the partial pairs then travel over NVLink from
            # the norm kernel itself; every rank agrees, else NCCL all-gather.
            handle = C.create_string_buffer(64)
            ok = raw.pb_peer_export(ctx, 0, dist.world, dist.rank, handle) == 0
            handles = dist.all_gather_bytes(handle.raw if ok else bytes(64), 64)
            ok = ok and raw.pb_peer_import(ctx, 0, dist.world, b"".join(handles)) == 0
            p2p = all(v == b"\x01" for v in dist.all_gather_bytes(b"\x01" if ok else b"\x00", 1))
            if not p2p:
                raw.pb_peer_close(ctx, 0)
            exchange = "NVLink peer mailboxes" if p2p else "NCCL all-gather"

            def step():
                gpu.check(raw.pb_norm_sharded(ctx, 0, code, per, p_(dx), p_(dout)), "norm")
        else:
            def step():
                gpu.check(raw.pb_norm(ctx, 0, code, 1, per, 1, p_(dx), p_(dout)), "norm")

    for _ in range(args.warmup):
        step()
    dist.barrier()
    with Clocks(gpu.backend.ordinal) as clocks:
        gpu.busy(step, dist)
        l0 = gpu.launches()
        seconds = gpu.timer(step, args.steps)
    launches = gpu.launches() - l0
    seconds = dist.max(seconds)
    nbytes = xl.nbytes
    out = np.empty(nrows if rows else 1, dtype)
    gpu.check(raw.pb_d2h(ctx, 0, C.c_void_p(out.ctypes.data), p_(dout), out.nbytes), "d2h")
    result.update({
        "metric": f"scaled norm {'rows (65536,4096)' if rows else 'full 2^28'} {np.dtype(dtype).name} GB/s",
        "value": nbytes * args.steps * dist.world / seconds / 1e9, "unit": "GB/s",
        "ms_per_step": seconds / args.steps * 1e3, "scaling": "strong",
        "dtype": "f64" if dtype == np.float64 else "f32",
        "config": {"workload": "BASELINE config 4" + ("b" if rows else "a"),
                   "parallelism": f"slices x{dist.world}"
                   + (f", pairs merged through {exchange}" if not rows and dist.world > 1 else "")},
        "clocks": clocks.summary(), "gpu_launches": launches,
        "roofline_kernel": ("norm", nbytes, seconds / args.steps),
        "_check": ("norm_rows", xl, out) if rows else ("norm", x, out),
    })
    if not rows and dist.world > 1:
        raw.pb_peer_close(ctx, 0)
        raw.pb_comm_destroy(ctx, 0)


# ------------------------------------------------------ reference arm --

def cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        info = [i for i in threadpool_info() if i.get("user_api") == "blas"]
        if info:
            return int(info[0]["num_threads"])
    except Exception:  # noqa: BLE001
        pass
    return len(os.sched_getaffinity(0))


def cpu_gemv_dot(budget_s: float):
    """The reference's NumPy backend on this workload: A @ x and u @ v."""
    from oracle import numpy_backend

    A, x, u, v = gen_gemv_dot()
    numpy_backend.matmul(A, x)
    numpy_backend.dot(u, v)
    step_bytes = 4 * (A.size + x.size + A.shape[0]) + 8 * u.size
    reps, t0 = 0, time.perf_counter()
    while True:
        numpy_backend.matmul(A, x)
        numpy_backend.dot(u, v)
        reps += 1
        if time.perf_counter() - t0 > budget_s or reps >= 200:
            break
    seconds = (time.perf_counter() - t0) / reps
    return {"value": step_bytes / seconds / 1e9, "unit": "GB/s", "cores": cpu_threads(),
            "kind": "port", "sample": f"{reps} full steps (GEMV 16384^2 + DOT 2^26) with NumPy/OpenBLAS",
            "ms_per_step": seconds * 1e3}


def reference_arm(args, dist: Dist):
    if dist.rank != 0:
        return 0
    if args.workload != "gemv_dot":
        print(json.dumps({"impl": "reference", "unavailable": "reference arm implemented for the "
                          "default workload only"}))
        return 0
    from oracle import numpy_backend

    A, x, u, v = gen_gemv_dot()
    for _ in range(max(1, args.warmup)):
        numpy_backend.matmul(A, x)
        numpy_backend.dot(u, v)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        numpy_backend.matmul(A, x)
        numpy_backend.dot(u, v)
        times.append(time.perf_counter() - t0)
    step_bytes = 4 * (A.size + x.size + A.shape[0]) + 8 * u.size
    seconds = sum(times)
    value = step_bytes * args.steps / seconds / 1e9
    print(json.dumps({
        "impl": "reference", "metric": "GEMV 16384x16384 + DOT 2^26 float32 HBM throughput",
        "value": value, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": seconds / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "BASELINE config 2 (see the b200 arm)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cpu_threads(), "kind": "port",
                         "sample": f"{args.steps} full steps through the NumPy-backend restatement "
                                   "(NumPy @ -> OpenBLAS sgemv + sdot)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


# ----------------------------------------------------------------- main --

def exact_norm(x: np.ndarray) -> float:
    """Near-exact norm for the full-norm parity check (chunked, bounded host
    memory): float32 input squared and summed in float64; float64 input scaled
    by a power of two and summed in long double."""
    flat = x.reshape(-1)
    if not flat.size:
        return 0.0
    step = 1 << 24
    if flat.dtype == np.float32:
        total = 0.0
        for i in range(0, flat.size, step):
            c = flat[i:i + step].astype(np.float64)
            total += float(np.dot(c, c))
        return float(np.sqrt(total))
    finite = flat[np.isfinite(flat)]
    if finite.size != flat.size:
        return float("nan") if np.isnan(flat).any() else float("inf")
    top = float(np.max(np.abs(finite)))
    if top == 0.0:
        return 0.0
    e = np.frexp(top)[1]
    total = np.longdouble(0)
    for i in range(0, flat.size, step):
        c = np.ldexp(flat[i:i + step], -e).astype(np.longdouble)
        total += np.sum(c * c)
    return float(np.sqrt(total) * np.longdouble(2.0) ** e)


def parity_check(check):
    from oracle import numpy_backend, tolerance

    kind = check[0]
    if kind == "gemv_dot":
        _, A, x, u, v, y, d = check
        bad = tolerance.gemm_violations(y, numpy_backend.matmul(A, x), A, x)
        bad += tolerance.gemm_violations(d.reshape(()), numpy_backend.dot(u, v), u, v)
        return bad
    if kind == "gemm":
        _, A, B, Cm = check
        rows = np.random.default_rng(0).choice(A.shape[-2], size=min(64, A.shape[-2]), replace=False)
        a = A[..., rows, :]
        return tolerance.gemm_violations(Cm[..., rows, :], numpy_backend.matmul(a, B), a, B)
    if kind == "elementwise":
        _, x, y, z = check
        return int(np.sum(numpy_backend.elementwise("add", (x, y), np.float32).view(np.uint32)
                          != z.view(np.uint32)))
    if kind == "reduce":
        _, x, _, z = check
        want = numpy_backend.reduce(x, (0,), False, np.float32)
        bound = 4 * x.size * tolerance.unit_roundoff(np.float32) * float(np.sum(np.abs(x), dtype=np.float64))
        return int(abs(float(z[0]) - float(want)) > bound)
    if kind == "norm_rows":
        _, x, out = check
        sel = np.arange(0, x.shape[0], max(1, x.shape[0] // 256))
        return tolerance.norm_violations(out[sel], numpy_backend.norm(x[sel], axis=1))
    if kind == "norm":  # the full (possibly sharded) norm against the whole input
        _, x, out = check
        return tolerance.norm_violations(out.reshape(()), numpy_backend.norm(x),
                                         exact=exact_norm(x))
    return None


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--workload", default="gemv_dot",
                        choices=("gemv_dot", "gemm1024", "batched", "norm", "norm_rows", "gemm_f32",
                                 "gemm_f64", "vecmat", "elementwise", "reduce"))
    parser.add_argument("--dtype", choices=("f32", "f64"), default="f32", help="norm workloads")
    parser.add_argument("--n", type=int, default=0,
                        help="GEMM size override (profiling captures); 0 = the BASELINE size")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    dist = Dist()
    try:
        if args.impl == "reference":
            return reference_arm(args, dist)
        gpu = Gpu(dist.local)
        result: dict = {}
        if args.workload == "gemv_dot":
            run_gemv_dot(gpu, args, dist, result)
        elif args.workload in ("gemm1024", "gemm_f32", "gemm_f64"):
            run_gemm(gpu, args, dist, result, args.workload)
        elif args.workload == "batched":
            run_batched(gpu, args, dist, result)
        elif args.workload == "vecmat":
            run_vecmat(gpu, args, dist, result)
        elif args.workload in ("elementwise", "reduce"):
            run_around(gpu, args, dist, result, args.workload)
        else:
            run_norm(gpu, args, dist, result, rows=args.workload == "norm_rows")
        check = result.pop("_check")
        name, work, sec = result.pop("roofline_kernel")
        pk = peaks()
        bad = parity_check(check) if dist.rank == 0 else None
        if dist.rank != 0:
            return 0
        if result["unit"] == "GB/s" or name in ("gemv", "norm", "skinny", "elementwise", "reduce"):
            achieved = work / sec / 1e9
            roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / pk["hbm_gbs"], "kernel": name, "peak_source": pk["source"],
                    "traffic": traffic_per_launch(name, args.workload),
                    "algorithmic_bytes": work}
        else:
            achieved = work / sec / 1e12
            ceiling = TENSOR_CEILINGS.get(args.workload)
            roof = {"bound": "tensor", "achieved": achieved,
                    "peak": ceiling[0] if ceiling else None, "unit": "TFLOP/s",
                    "frac": achieved / ceiling[0] if ceiling else None, "kernel": name,
                    "peak_source": ceiling[1] if ceiling else None,
                    "traffic": traffic_per_launch(name, args.workload)}
        line = {
            "metric": result.pop("metric"), "value": result.pop("value"), "unit": result.pop("unit"),
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": result.pop("ms_per_step"), "higher_is_better": True,
            "scaling": result.pop("scaling"), "vs_baseline": None, "dtype": result.pop("dtype"),
            "data": "synthetic (seeded numpy default_rng, BASELINE distributions)",
            "config": result.pop("config"), "roofline": roof,
        }
        line.update(result)
        line["parity_violations"] = bad
        if args.workload == "gemv_dot" and dist.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_gemv_dot(10.0)
        print(json.dumps(line))
        return 0
    finally:
        dist.close()


if __name__ == "__main__":
    sys.exit(main())
