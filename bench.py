"""Benchmark of the b200 linear-algebra path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload suite|batched|gemm1024|gemv_dot|norm|norm_rows|gemm_f32|gemm_f64
                                |vecmat|elementwise|reduce|residual] [--dtype f32|f64] [--n SIZE]

Default (``suite``): every BASELINE config in one run, one JSON line.  The
headline ``value`` is config 3 -- the batched broadcast float32 GEMM
(8,16,512,256) @ (1,16,256,384), N(0,1) from default_rng(2), split along the
leading batch dimension across ranks (strong scaling, TFLOP/s over all
ranks).  ``configs`` carries one sub-record per other config, each with its own
value, roofline, parity count, end-to-end figure and (N = 1) CPU baseline:

  config1_gemm_f32_1024   float32 1024^3, default_rng(0); one replica per rank
  config2_gemv_dot_f32    y = A @ x (A 16384^2) + DOT of two 2^26 vectors, U[-1,1],
                          default_rng(1); one replica per rank
  config4a_norm_f32/_f64  full norm of 2^28 values N(0,1) * 10^U(-35,35)
                          (f64: 10^U(-300,300)), default_rng(3); contiguous slices,
                          partial (scale, ssq) pairs merged through NVLink peer mailboxes
  config4b_rows_f32/_f64  axis=1 norms of the same values as (65536, 4096); row blocks
  config5_gemm_f32_16384  float32 16384^3, default_rng(4); row blocks of A, B broadcast
  config5_gemm_f64_8192   float64 8192^3, default_rng(4); row blocks of A, B broadcast
  vecmat_f32_16384        x @ A (vector @ matrix), A 16384^2 f32, default_rng(5)
  residual_f32_16384      b - A @ x (the compiled-plan residual, GEMV epilogue), default_rng(7)

Multi-GPU: one process per GPU under torchrun.  Barriers and the
max-over-ranks time go through a gloo process group (host side only); data
collectives use the library's own NCCL communicator (B broadcast for configs 3
and 5) and NVLink peer mailboxes (config 4a partials).  Every record's inputs
are larger than the 126 MB L2 or state otherwise in ``config.l2``.
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

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# Tensor ceilings besides MEASURED_PEAKS.json (which carries bf16 and HBM only):
# cuBLAS on this pool's B200 (8192^3, best of 10): TF32 737.7 TFLOP/s, DGEMM
# 35.5 TFLOP/s; B200 specification FP64 (tensor) 40 TFLOP/s.
CUBLAS_TF32_TFLOPS = 737.7
CUBLAS_DGEMM_TFLOPS = 35.5
SPEC_FP64_TFLOPS = 40.0
L2_BYTES = 126 * 1024 * 1024


# ------------------------------------------------------------- inputs --
# Seeds and distributions exactly as BASELINE.json's configs state.

def gen_gemv_dot():
    rng = np.random.default_rng(1)
    A = rng.uniform(-1, 1, (16384, 16384)).astype(np.float32)
    x = rng.uniform(-1, 1, 16384).astype(np.float32)
    u = rng.uniform(-1, 1, 1 << 26).astype(np.float32)
    v = rng.uniform(-1, 1, 1 << 26).astype(np.float32)
    return A, x, u, v


def gen_gemm(seed, n, dtype):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n, n), dtype=dtype), rng.standard_normal((n, n), dtype=dtype)


def gen_batched():
    rng = np.random.default_rng(2)
    A = rng.standard_normal((8, 16, 512, 256)).astype(np.float32)
    B = rng.standard_normal((1, 16, 256, 384)).astype(np.float32)
    return A, B


def gen_norm(n=1 << 28, dtype=np.float32, span=35):
    rng = np.random.default_rng(3)
    out = np.empty(n, dtype)
    step = 1 << 24
    for i in range(0, n, step):  # bounded host temporaries
        m = min(step, n - i)
        out[i:i + m] = rng.standard_normal(m) * 10.0 ** rng.uniform(-span, span, m)
    return out


_NORM_CACHE: dict = {}


def norm_input(dtype):
    """Config 4 values for ``dtype`` (shared by the full and the row norms)."""
    key = np.dtype(dtype).name
    if key not in _NORM_CACHE:
        _NORM_CACHE.clear()
        _NORM_CACHE[key] = gen_norm(1 << 28, dtype, 300 if key == "float64" else 35)
    return _NORM_CACHE[key]


def shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rank's [lo, hi) of n items, as np.array_split divides them."""
    q, r = divmod(n, world)
    lo = rank * q + min(rank, r)
    return lo, lo + q + (1 if rank < r else 0)


# ---------------------------------------------------------- plumbing --

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

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
            # Bound the library's own collective waits too (default 300 s).
            os.environ.setdefault("PB_COMM_TIMEOUT_S", "60")
            self.dist = dist
            self.pg = True

    def barrier(self):
        if self.pg:
            self.dist.barrier()

    def _reduce(self, value: float, op) -> float:
        import torch

        t = torch.tensor([value], dtype=torch.float64)
        self.dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, value: float) -> float:
        return self._reduce(value, self.dist.ReduceOp.MAX) if self.pg else value

    def sum(self, value: float) -> float:
        return self._reduce(value, self.dist.ReduceOp.SUM) if self.pg else value

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


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {**PEAKS_FALLBACK, "source": "fallback"}


def traffic_entry(key: str):
    """The committed ncu DRAM figure for a (workload, kernel) key, if any."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    return json.loads(path.read_text()).get(key)


def traffic_per_launch(key: str, units: float):
    """DRAM bytes (read + write) per launch of the main kernel: the ncu figure
    if it was captured at this launch's size, scaled by the units processed
    when the kernel's traffic grows in proportion to them (streaming
    kernels), else None."""
    entry = traffic_entry(key)
    if not entry:
        return None, None
    captured = float(entry.get("units_per_launch") or 0)
    bytes_ = float(entry["dram_bytes_per_launch"])
    if captured and abs(captured - units) <= 1e-9 * captured:
        return bytes_, "captured at this size"
    if captured and entry.get("proportional"):
        return bytes_ * units / captured, f"scaled from the capture at {captured:.4g} units"
    return None, None


def cpu_cores() -> int:
    return len(os.sched_getaffinity(0))


def blas_threads_all():
    """Let OpenBLAS use every core this process may run on, whatever
    OMP_NUM_THREADS torchrun set; returns the limiter (keep it alive) and the
    thread count in effect."""
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        limiter = threadpool_limits(limits=cpu_cores(), user_api="blas")
        info = [i for i in threadpool_info() if i.get("user_api") == "blas"]
        return limiter, int(info[0]["num_threads"]) if info else cpu_cores()
    except Exception:  # noqa: BLE001 - threadpoolctl absent: numpy's own default
        return None, cpu_cores()


# ----------------------------------------------------------- the GPU --

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

    def sync(self):
        self.check(self.raw.pb_sync(self.ctx, 0), "sync")

    def busy(self, fn, dist, seconds=0.5):
        """Untimed steps for about `seconds`, so the clock sampler sees the GPU
        under this workload's load before the timed region.  The step count is
        calibrated per rank and agreed (max) across ranks: steps may contain
        collectives, so every rank must run exactly the same number."""
        t0 = time.perf_counter()
        for _ in range(4):
            fn()
        self.sync()
        per4 = max(time.perf_counter() - t0, 1e-6)
        rounds = int(dist.max(float(min(max(1, int(seconds / per4)), 4096))))
        for _ in range(rounds):
            for _ in range(4):
                fn()
            self.sync()

    def timer(self, fn, reps):
        """Seconds for `reps` calls, by CUDA events on the library's stream."""
        self.sync()
        self.check(self.raw.pb_timer_start(self.ctx, 0), "timer")
        for _ in range(reps):
            fn()
        ms = C.c_float()
        self.check(self.raw.pb_timer_stop(self.ctx, 0, C.byref(ms)), "timer")
        return ms.value / 1e3

    def kernel_seconds(self, fn, reps, graph=False):
        """Average duration of the main kernel of `fn` (CUDA events around each
        launch on the library's stream) and the launches seen.  With `graph`,
        `fn` is captured with the events inside the graph and replayed `reps`
        times, so the host's submission gaps between an event and its kernel
        cannot enter the time."""
        self.sync()
        total, count = C.c_double(), C.c_uint64()
        if not graph:
            self.check(self.raw.pb_ktimer_enable(self.ctx, 0, 1), "ktimer")
            try:
                for _ in range(reps):
                    fn()
                self.check(self.raw.pb_ktimer_read(self.ctx, 0, C.byref(total), C.byref(count)), "ktimer")
            finally:
                self.raw.pb_ktimer_enable(self.ctx, 0, 0)
            return (total.value / 1e3 / count.value if count.value else None), count.value
        self.check(self.raw.pb_ktimer_enable(self.ctx, 0, 2), "ktimer")
        try:
            with self.backend.capture(fn) as g:
                ms, launches = 0.0, 0
                for _ in range(reps):
                    g.launch()
                    self.check(self.raw.pb_ktimer_read(self.ctx, 0, C.byref(total), C.byref(count)), "ktimer")
                    ms += total.value
                    launches += count.value
        finally:
            self.raw.pb_ktimer_enable(self.ctx, 0, 0)
        return (ms / 1e3 / launches if launches else None), launches

    def launches(self):
        return self.backend.launch_count()

    def pin(self, arrays):
        for a in arrays:
            self.check(self.raw.pb_host_register(C.c_void_p(a.ctypes.data), max(a.nbytes, 1)), "pin")

    def unpin(self, arrays):
        for a in arrays:
            self.raw.pb_host_unregister(C.c_void_p(a.ctypes.data))

    def h2d(self, dst, host):
        self.check(self.raw.pb_h2d(self.ctx, 0, p_(dst), C.c_void_p(host.ctypes.data), host.nbytes, 0),
                   "h2d")

    def d2h_async(self, host, src):
        self.check(self.raw.pb_d2h_async(self.ctx, 0, C.c_void_p(host.ctypes.data), p_(src),
                                         host.nbytes), "d2h")

    def d2h(self, host, src):
        self.check(self.raw.pb_d2h(self.ctx, 0, C.c_void_p(host.ctypes.data), p_(src), host.nbytes),
                   "d2h")


def p_(buf):
    return C.c_void_p(buf.ptr)


class Comm:
    """The library's NCCL communicator and NVLink peer mailboxes (N > 1)."""

    def __init__(self, gpu: Gpu, dist: Dist):
        self.gpu, self.dist = gpu, dist
        self.active = dist.world > 1
        self.exchange = None
        if not self.active:
            return
        raw, ctx = gpu.raw, gpu.ctx
        uid = C.create_string_buffer(128)
        if dist.rank == 0:
            gpu.check(raw.pb_comm_unique_id(uid), "unique id")
        data = dist.broadcast_bytes(uid.raw if dist.rank == 0 else None, 128)
        gpu.check(raw.pb_comm_init(ctx, 0, dist.world, dist.rank, data), "comm init")
        handle = C.create_string_buffer(64)
        ok = raw.pb_peer_export(ctx, 0, dist.world, dist.rank, handle) == 0
        handles = dist.all_gather_bytes(handle.raw if ok else bytes(64), 64)
        ok = ok and raw.pb_peer_import(ctx, 0, dist.world, b"".join(handles)) == 0
        p2p = all(v == b"\x01" for v in dist.all_gather_bytes(b"\x01" if ok else b"\x00", 1))
        if not p2p:
            raw.pb_peer_close(ctx, 0)
        self.exchange = "NVLink peer mailboxes" if p2p else "NCCL all-gather"

    def broadcast(self, buf, nbytes):
        self.gpu.check(self.gpu.raw.pb_broadcast(self.gpu.ctx, 0, p_(buf), nbytes, 0), "broadcast")

    def close(self):
        if self.active:
            self.gpu.raw.pb_peer_close(self.gpu.ctx, 0)
            self.gpu.raw.pb_comm_destroy(self.gpu.ctx, 0)


# -------------------------------------------------------- workloads --
#
# A workload holds one config's host inputs and device buffers on this rank.
#   setup()        host inputs (this rank's share) and resident device buffers
#   step()         one pass over the resident inputs (what `value` times)
#   kernel_step()  the calls whose main kernel the roofline times
#   e2e_step()     one pass from pinned host inputs to host results
#   violations()   parity of this rank's outputs against the oracle
#   cpu_step()     the reference's CPU path on a bounded sample -> units done

class Workload:
    name = ""
    unit = "GB/s"
    bound = "hbm"
    scaling = "weak"
    dtype = "f32"
    e2e_steps_cap = 20

    def __init__(self, args, dist: Dist):
        self.args, self.dist = args, dist
        self.world, self.rank = dist.world, dist.rank

    # Units (flops or bytes) this rank processes per step, and per launch of
    # the main kernel (main_launches launches per kernel_step).
    units = 0.0
    kernel_units = 0.0
    kernel_key = ""
    main_launches = 1
    extra: dict = {}

    def graphable(self):
        """Whether one step can be captured into a CUDA graph (no exchange
        whose sequence numbers advance per call, nothing allocated)."""
        return True

    def scale(self):
        return 1e12 if self.unit == "TFLOP/s" else 1e9

    def kernel_step(self):
        self.step()

    def e2e_bytes(self):
        return 0, 0


class Batched(Workload):
    """BASELINE config 3, split along the leading batch dimension."""

    name, unit, bound, scaling, dtype = "config3_batched_f32", "TFLOP/s", "tensor", "strong", "f32 (3xTF32)"

    def metric(self):
        return "batched broadcast GEMM (8,16,512,256)@(1,16,256,384) float32 TFLOP/s"

    def config(self):
        return {"workload": "BASELINE config 3: (8,16,512,256) @ (1,16,256,384) float32, N(0,1), "
                            "default_rng(2)",
                "parallelism": f"batch split x{self.world} (B broadcast from rank 0 by NCCL)",
                "l2": "per step 176 MB of operands and output (1 GPU) > 126 MB L2; at N > 1 the "
                      "shards are smaller than L2 and no flush is made (strong scaling)"}

    def host(self):
        self.A, self.B = gen_batched()
        lo, hi = shard(8, self.world, self.rank)
        self.Aloc = np.ascontiguousarray(self.A[lo:hi])
        self.per = hi - lo

    def setup(self, gpu, comm):
        self.gpu, self.comm = gpu, comm
        self.host()
        L = gpu.lib
        self.dA = gpu.upload(self.Aloc)
        if comm.active:
            self.dB = gpu.upload(self.B) if self.rank == 0 else gpu.empty(self.B.shape, np.float32)
            t0 = time.perf_counter()
            comm.broadcast(self.dB, self.B.nbytes)
            gpu.sync()
            self.extra = {"b_broadcast_ms_once": (time.perf_counter() - t0) * 1e3}
        else:
            self.dB = gpu.upload(self.B)
        self.dC = gpu.empty((self.per, 16, 512, 384), np.float32)
        self.args_gemm = (L.PB_F32, 2, L.i64_array((self.per, 16)), L.i64_array([16, 1]),
                          L.i64_array([0, 1]), 512, 384, 256)
        self.units = self.kernel_units = 2.0 * self.per * 16 * 512 * 384 * 256
        self.kernel_key = "batched:gemm"

    def _gemm(self, dA, dB, dC):
        g = self.gpu
        g.check(g.raw.pb_gemm(g.ctx, 0, *self.args_gemm, p_(dA), p_(dB), p_(dC)), "gemm")

    def step(self):
        self._gemm(self.dA, self.dB, self.dC)

    def e2e_setup(self):
        self.hA = np.ascontiguousarray(self.Aloc)
        self.hB = np.ascontiguousarray(self.B)
        self.hC = np.empty((self.per, 16, 512, 384), np.float32)
        self.pinned = [self.hA, self.hB, self.hC]
        self.gpu.pin(self.pinned)

    e2e_how = ("; one pb_gemm_host call per step: host A and B in, host C out, uploads, "
               "products and downloads overlapped over the 8 outer batches")

    def e2e_step(self):
        g = self.gpu
        g.check(g.raw.pb_gemm_host(g.ctx, 0, *self.args_gemm, C.c_void_p(self.hA.ctypes.data),
                                   C.c_void_p(self.hB.ctypes.data), C.c_void_p(self.hC.ctypes.data), 0),
                "gemm_host")

    def e2e_bytes(self):
        return self.hA.nbytes + self.hB.nbytes, self.hC.nbytes

    def violations(self):
        C_ = np.empty((self.per, 16, 512, 384), np.float32)
        self.gpu.d2h(C_, self.dC)
        rows = np.random.default_rng(0).choice(512, size=64, replace=False)
        from oracle import numpy_backend, tolerance

        a = self.Aloc[..., rows, :]
        return tolerance.gemm_violations(C_[..., rows, :], numpy_backend.matmul(a, self.B), a, self.B)

    def cpu_prepare(self):
        if not hasattr(self, "A"):
            self.A, self.B = gen_batched()

    def cpu_step(self):
        from oracle import numpy_backend

        numpy_backend.matmul(self.A, self.B)
        return 2.0 * 8 * 16 * 512 * 384 * 256, "the full config-3 product (NumPy @ -> OpenBLAS sgemm per batch)"


class Gemm(Workload):
    """Config 1 (1024^3 f32, replicas) and config 5 (row blocks of A, B broadcast)."""

    unit, bound = "TFLOP/s", "tensor"

    def __init__(self, args, dist, which):
        super().__init__(args, dist)
        self.which = which
        if which == "gemm1024":
            self.seed, self.n, self.np_dtype, self.sharded = 0, args.n or 1024, np.float32, False
            self.name = "config1_gemm_f32_1024"
        elif which == "gemm_f32":
            self.seed, self.n, self.np_dtype, self.sharded = 4, args.n or 16384, np.float32, True
            self.name = "config5_gemm_f32_16384"
        else:
            self.seed, self.n, self.np_dtype, self.sharded = 4, args.n or 8192, np.float64, True
            self.name = "config5_gemm_f64_8192"
        self.scaling = "strong" if self.sharded else "weak"
        self.dtype = "f32 (3xTF32)" if self.np_dtype == np.float32 else "f64 (DMMA)"
        self.e2e_steps_cap = 5 if self.n >= 8192 else 20

    def metric(self):
        return f"{np.dtype(self.np_dtype).name} GEMM {self.n}^3 TFLOP/s"

    def config(self):
        cfg = {"workload": (f"BASELINE config {'1' if self.which == 'gemm1024' else '5'}: "
                            f"{np.dtype(self.np_dtype).name} {self.n}^3, N(0,1), default_rng({self.seed})"),
               "parallelism": (f"row blocks of A x{self.world} (B broadcast from rank 0 by NCCL)"
                               if self.sharded else f"replicas x{self.world}")}
        op_bytes = 3 * self.n * self.n * np.dtype(self.np_dtype).itemsize
        cfg["l2"] = (f"operands and output {op_bytes / 1e6:.0f} MB > 126 MB L2" if op_bytes > L2_BYTES
                     else f"operands and output {op_bytes / 1e6:.1f} MB fit the 126 MB L2; the step "
                          "is a single small product by definition (no flush)")
        return cfg

    def setup(self, gpu, comm):
        self.gpu, self.comm = gpu, comm
        A, self.B = gen_gemm(self.seed, self.n, self.np_dtype)
        n = self.n
        lo, hi = shard(n, self.world, self.rank) if self.sharded else (0, n)
        self.rows = hi - lo
        self.Aloc = np.ascontiguousarray(A[lo:hi])
        del A
        self.dA = gpu.upload(self.Aloc)
        if self.sharded and comm.active:
            self.dB = gpu.upload(self.B) if self.rank == 0 else gpu.empty(self.B.shape, self.np_dtype)
            t0 = time.perf_counter()
            comm.broadcast(self.dB, self.B.nbytes)
            gpu.sync()
            self.extra = {"b_broadcast_ms_once": (time.perf_counter() - t0) * 1e3}
        else:
            self.dB = gpu.upload(self.B)
        self.dC = gpu.empty((self.rows, n), self.np_dtype)
        self.code = gpu.lib.dtype_code(self.np_dtype)
        self.ns = gpu.lib.i64_array([])
        self.units = self.kernel_units = 2.0 * self.rows * n * n
        self.kernel_key = f"{self.which}:gemm"

    def step(self):
        g, n = self.gpu, self.n
        g.check(g.raw.pb_gemm(g.ctx, 0, self.code, 0, self.ns, self.ns, self.ns, self.rows, n, n,
                              p_(self.dA), p_(self.dB), p_(self.dC)), "gemm")

    def e2e_setup(self):
        self.hC = np.empty((self.rows, self.n), self.np_dtype)
        self.pinned = [self.Aloc, self.B, self.hC]
        self.gpu.pin(self.pinned)

    @property
    def e2e_how(self):
        if self.sharded and self.comm.active:
            return ", B broadcast by NCCL from rank 0"
        return ("; one pb_gemm_host call per step: host A and B in, host C out, uploads, products "
                "and downloads overlapped over row blocks of A")

    def e2e_step(self):
        g = self.gpu
        if self.sharded and self.comm.active:
            g.h2d(self.dA, self.Aloc)
            if self.rank == 0:
                g.h2d(self.dB, self.B)
            self.comm.broadcast(self.dB, self.B.nbytes)
            self.step()
            g.d2h_async(self.hC, self.dC)
            return
        n = self.n
        g.check(g.raw.pb_gemm_host(g.ctx, 0, self.code, 0, self.ns, self.ns, self.ns, self.rows, n, n,
                                   C.c_void_p(self.Aloc.ctypes.data), C.c_void_p(self.B.ctypes.data),
                                   C.c_void_p(self.hC.ctypes.data), 0), "gemm_host")

    def e2e_bytes(self):
        own_b = (not (self.sharded and self.comm.active)) or self.rank == 0
        return self.Aloc.nbytes + (self.B.nbytes if own_b else 0), self.hC.nbytes

    def violations(self):
        from oracle import numpy_backend, tolerance

        Cl = np.empty((self.rows, self.n), self.np_dtype)
        self.gpu.d2h(Cl, self.dC)
        if self.n <= 2048:
            return tolerance.gemm_violations(Cl, numpy_backend.matmul(self.Aloc, self.B), self.Aloc, self.B)
        rows = np.random.default_rng(0).choice(self.rows, size=min(64, self.rows), replace=False)
        a = self.Aloc[rows]
        return tolerance.gemm_violations(Cl[rows], numpy_backend.matmul(a, self.B), a, self.B)

    def cpu_prepare(self):
        # Config 1 whole; config 5 a block of rows (OpenBLAS runs such a block
        # at its full rate; the whole product takes seconds to minutes on CPU).
        self.sample_rows = self.n if self.n <= 2048 else 256
        if getattr(self, "Aloc", None) is not None and self.Aloc.shape[0] >= self.sample_rows:
            A = self.Aloc
        else:
            A, self.B = gen_gemm(self.seed, self.n, self.np_dtype)
        self.Asample = np.ascontiguousarray(A[: self.sample_rows])

    def cpu_step(self):
        from oracle import numpy_backend

        numpy_backend.matmul(self.Asample, self.B)
        what = ("the full product" if self.sample_rows == self.n
                else f"{self.sample_rows} rows of A times the full B")
        return 2.0 * self.sample_rows * self.n * self.n, f"{what} (NumPy @ -> OpenBLAS)"


class GemvDot(Workload):
    """GEMV 16384^2 + DOT 2^26, one replica per rank."""

    name = "config2_gemv_dot_f32"

    def metric(self):
        return "GEMV 16384x16384 + DOT 2^26 float32 HBM throughput"

    def config(self):
        return {"workload": "BASELINE config 2: y = A@x (A 16384x16384 f32) + DOT of two 2^26 f32 "
                            "vectors, U[-1,1], default_rng(1)",
                "parallelism": f"replicas x{self.world}",
                "l2": "inputs (1.6 GB) larger than the 126 MB L2; no flush needed"}

    def setup(self, gpu, comm):
        self.gpu = gpu
        self.A, self.x, self.u, self.v = gen_gemv_dot()
        self.M, self.K = self.A.shape
        self.n = self.u.size
        self.bytes_gemv = 4 * (self.M * self.K + self.K + self.M)
        self.bytes_dot = 2 * 4 * self.n
        self.dA, self.dx, self.du, self.dv = (gpu.upload(t) for t in (self.A, self.x, self.u, self.v))
        self.dy, self.dd = gpu.empty((self.M,), np.float32), gpu.empty((1,), np.float32)
        self.units = self.bytes_gemv + self.bytes_dot
        self.kernel_units = self.bytes_gemv
        self.kernel_key = "gemv_dot:gemv"

    def gemv(self):
        g = self.gpu
        g.check(g.raw.pb_gemv(g.ctx, 0, g.lib.PB_F32, self.M, self.K, p_(self.dA), p_(self.dx),
                              p_(self.dy)), "gemv")

    def dot(self):
        g = self.gpu
        g.check(g.raw.pb_dot(g.ctx, 0, g.lib.PB_F32, self.n, p_(self.du), p_(self.dv), p_(self.dd)),
                "dot")

    def step(self):
        self.gemv()
        self.dot()

    def kernel_step(self):
        self.gemv()

    def more_kernels(self, graph=False):
        t, _ = self.gpu.kernel_seconds(self.dot, self.args.steps, graph=graph)
        return {"gemv_gbs": None, "dot_ms": t * 1e3, "dot_gbs": self.bytes_dot / t / 1e9}

    def e2e_setup(self):
        self.hy = np.empty(self.M, np.float32)
        self.hd = np.empty(1, np.float32)
        self.pinned = [self.A, self.x, self.u, self.v, self.hy, self.hd]
        self.gpu.pin(self.pinned)

    def e2e_step(self):
        g = self.gpu
        for h, dbuf in ((self.A, self.dA), (self.x, self.dx), (self.u, self.du), (self.v, self.dv)):
            g.h2d(dbuf, h)
        self.step()
        g.d2h_async(self.hy, self.dy)
        g.d2h_async(self.hd, self.dd)

    def e2e_bytes(self):
        return sum(t.nbytes for t in (self.A, self.x, self.u, self.v)), self.hy.nbytes + 4

    def violations(self):
        from oracle import numpy_backend, tolerance

        y = np.empty(self.M, np.float32)
        d = np.empty(1, np.float32)
        self.gpu.d2h(y, self.dy)
        self.gpu.d2h(d, self.dd)
        bad = tolerance.gemm_violations(y, numpy_backend.matmul(self.A, self.x), self.A, self.x)
        bad += tolerance.gemm_violations(d.reshape(()), numpy_backend.dot(self.u, self.v), self.u, self.v)
        return bad

    def cpu_prepare(self):
        if not hasattr(self, "A"):
            self.A, self.x, self.u, self.v = gen_gemv_dot()

    def cpu_step(self):
        from oracle import numpy_backend

        numpy_backend.matmul(self.A, self.x)
        numpy_backend.dot(self.u, self.v)
        return (4.0 * (self.A.size + self.x.size + self.A.shape[0]) + 8.0 * self.u.size,
                "the full step (NumPy @ -> OpenBLAS sgemv + sdot)")


class Norm(Workload):
    """BASELINE config 4a (full norm, slices + peer-mailbox merge) and 4b
    (axis=1 row norms, row blocks)."""

    scaling = "strong"

    def __init__(self, args, dist, rows: bool, np_dtype):
        super().__init__(args, dist)
        self.rows_mode, self.np_dtype = rows, np.dtype(np_dtype)
        tag = "f64" if self.np_dtype == np.float64 else "f32"
        self.dtype = tag
        self.name = f"config4b_rows_{tag}" if rows else f"config4a_norm_{tag}"

    def metric(self):
        what = "rows (65536,4096)" if self.rows_mode else "full 2^28"
        return f"scaled norm {what} {self.np_dtype.name} GB/s"

    def config(self):
        span = 300 if self.np_dtype == np.float64 else 35
        cfg = {"workload": (f"BASELINE config 4{'b' if self.rows_mode else 'a'}: "
                            f"{'axis=1 norms of (65536,4096)' if self.rows_mode else 'norm of 2^28 values'} "
                            f"{self.np_dtype.name}, N(0,1)*10^U(-{span},{span}), default_rng(3)"),
               "l2": f"input {2 ** 28 * self.np_dtype.itemsize / 1e9:.2f} GB > 126 MB L2"}
        if self.rows_mode:
            cfg["parallelism"] = f"row blocks x{self.world}"
        else:
            cfg["parallelism"] = f"slices x{self.world}" + (
                f", (scale, ssq) pairs merged through {self.exchange}" if self.world > 1 else "")
        return cfg

    exchange = None

    def setup(self, gpu, comm):
        self.gpu, self.comm = gpu, comm
        self.x = norm_input(self.np_dtype)
        self.code = gpu.lib.dtype_code(self.np_dtype)
        if self.rows_mode:
            shape = (65536, 4096)
            lo, hi = shard(shape[0], self.world, self.rank)
            self.nrows = hi - lo
            self.xl = np.ascontiguousarray(self.x.reshape(shape)[lo:hi])
            self.out = gpu.empty((self.nrows,), self.np_dtype)
            self.kernel_key = f"norm_rows_{self.dtype}:norm"
        else:
            lo, hi = shard(self.x.size, self.world, self.rank)
            self.xl = self.x[lo:hi]
            self.out = gpu.empty((1,), self.np_dtype)
            self.exchange = comm.exchange
            self.kernel_key = f"norm_{self.dtype}:norm"
        self.dx = gpu.upload(self.xl)
        self.units = self.kernel_units = float(self.xl.nbytes)

    def graphable(self):
        # The sharded full norm exchanges through the peer mailboxes (or NCCL),
        # whose sequence numbers advance with every call.
        return self.rows_mode or not self.comm.active

    def step(self):
        g = self.gpu
        if self.rows_mode:
            g.check(g.raw.pb_norm(g.ctx, 0, self.code, self.nrows, 4096, 1, p_(self.dx), p_(self.out)),
                    "norm")
        elif self.comm.active:
            g.check(g.raw.pb_norm_sharded(g.ctx, 0, self.code, self.xl.size, p_(self.dx), p_(self.out)),
                    "norm")
        else:
            g.check(g.raw.pb_norm(g.ctx, 0, self.code, 1, self.xl.size, 1, p_(self.dx), p_(self.out)),
                    "norm")

    def e2e_setup(self):
        self.hx = np.ascontiguousarray(self.xl)
        self.hout = np.empty(self.nrows if self.rows_mode else 1, self.np_dtype)
        self.pinned = [self.hx, self.hout]
        self.gpu.pin(self.pinned)

    def e2e_step(self):
        self.gpu.h2d(self.dx, self.hx)
        self.step()
        self.gpu.d2h_async(self.hout, self.out)

    def e2e_bytes(self):
        return self.hx.nbytes, self.hout.nbytes

    def violations(self):
        from oracle import numpy_backend, tolerance

        out = np.empty(self.nrows if self.rows_mode else 1, self.np_dtype)
        self.gpu.d2h(out, self.out)
        if self.rows_mode:
            sel = np.arange(0, self.xl.shape[0], max(1, self.xl.shape[0] // 256))
            return tolerance.norm_violations(out[sel], numpy_backend.norm(self.xl[sel], axis=1))
        if self.rank != 0:
            return 0  # the merged norm is the same on every rank; rank 0 checks it
        return tolerance.norm_violations(out.reshape(()), numpy_backend.norm(self.x),
                                         exact=exact_norm(self.x))

    def cpu_prepare(self):
        self.x = norm_input(self.np_dtype)

    def cpu_step(self):
        from oracle import numpy_backend

        if self.rows_mode:
            sample = self.x.reshape(65536, 4096)[:4096]
            numpy_backend.norm(sample, axis=1)
            return float(sample.nbytes), "4096 of the 65536 rows through the NumPy-backend norm"
        sample = self.x[: 1 << 24]
        numpy_backend.norm(sample)
        return float(sample.nbytes), "2^24 of the 2^28 values through the NumPy-backend norm"


class Vecmat(Workload):
    """x @ A (vector @ matrix), float32 16384^2: the skinny kernel, replicas."""

    name = "vecmat_f32_16384"

    def metric(self):
        return f"vector @ matrix ({self.n} @ {self.n}x{self.n}) float32 HBM throughput"

    def config(self):
        return {"workload": f"x @ A, A {self.n}x{self.n} f32, U[-1,1], default_rng(5) (around the "
                            "path: the survey's vector edge shapes)",
                "parallelism": f"replicas x{self.world}",
                "l2": "A (1.07 GB) larger than the 126 MB L2; no flush needed"}

    def __init__(self, args, dist):
        super().__init__(args, dist)
        self.n = args.n or 16384

    def setup(self, gpu, comm):
        self.gpu = gpu
        rng = np.random.default_rng(5)
        n = self.n
        self.A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
        self.x = rng.uniform(-1, 1, n).astype(np.float32)
        self.dx, self.dA = gpu.upload(self.x), gpu.upload(self.A)
        self.dy = gpu.empty((n,), np.float32)
        self.ns = gpu.lib.i64_array([])
        self.units = self.kernel_units = 4.0 * (n * n + 2 * n)
        self.kernel_key = "vecmat:skinny"

    def step(self):
        g, n = self.gpu, self.n
        g.check(g.raw.pb_gemm(g.ctx, 0, g.lib.PB_F32, 0, self.ns, self.ns, self.ns, 1, n, n,
                              p_(self.dx), p_(self.dA), p_(self.dy)), "gemm")

    def e2e_setup(self):
        self.hy = np.empty(self.n, np.float32)
        self.pinned = [self.A, self.x, self.hy]
        self.gpu.pin(self.pinned)

    def e2e_step(self):
        self.gpu.h2d(self.dx, self.x)
        self.gpu.h2d(self.dA, self.A)
        self.step()
        self.gpu.d2h_async(self.hy, self.dy)

    def e2e_bytes(self):
        return self.A.nbytes + self.x.nbytes, self.hy.nbytes

    def violations(self):
        from oracle import numpy_backend, tolerance

        y = np.empty(self.n, np.float32)
        self.gpu.d2h(y, self.dy)
        x2 = self.x.reshape(1, -1)
        return tolerance.gemm_violations(y.reshape(1, -1), numpy_backend.matmul(x2, self.A), x2, self.A)

    def cpu_prepare(self):
        if not hasattr(self, "A"):
            rng = np.random.default_rng(5)
            self.A = rng.uniform(-1, 1, (self.n, self.n)).astype(np.float32)
            self.x = rng.uniform(-1, 1, self.n).astype(np.float32)

    def cpu_step(self):
        from oracle import numpy_backend

        numpy_backend.matmul(self.x, self.A)
        return 4.0 * (self.n * self.n + 2 * self.n), "the full product (NumPy @ -> OpenBLAS sgemv)"


class Around(Workload):
    """Operations around the path on 2^28 float32 values: elementwise add of
    two arrays (pb_elementwise) or their sum (pb_reduce)."""

    def __init__(self, args, dist, which):
        super().__init__(args, dist)
        self.which = which
        self.n = args.n or (1 << 28)
        self.name = f"{which}_f32_2p28"

    def metric(self):
        what = "elementwise add of two float32 arrays" if self.which == "elementwise" else "sum of float32 values"
        return f"{what} (n = {self.n}) HBM throughput"

    def config(self):
        return {"workload": f"{self.which}, n = {self.n} float32, N(0,1), default_rng(6)",
                "parallelism": f"replicas x{self.world}",
                "l2": "operands (1 GB each) larger than the 126 MB L2; no flush needed"}

    def _inputs(self):
        rng = np.random.default_rng(6)
        self.x = rng.standard_normal(self.n, dtype=np.float32)
        self.y = rng.standard_normal(self.n, dtype=np.float32) if self.which == "elementwise" else None

    def setup(self, gpu, comm):
        self.gpu = gpu
        self._inputs()
        L = gpu.lib
        self.dx = gpu.upload(self.x)
        if self.which == "elementwise":
            self.dy, self.dz = gpu.upload(self.y), gpu.empty((self.n,), np.float32)
            self.ptrs = (C.c_void_p * 2)(self.dx.ptr, self.dy.ptr)
            self.codes = (C.c_int * 2)(L.PB_F32, L.PB_F32)
            self.strides, self.shape = L.i64_array([1, 1]), L.i64_array([self.n])
            self.units = self.kernel_units = 12.0 * self.n
        else:
            self.dz = gpu.empty((1,), np.float32)
            self.shape = L.i64_array([self.n])
            self.units = self.kernel_units = 4.0 * self.n + 4
        self.kernel_key = f"{self.which}:{self.which}"

    def step(self):
        g, L = self.gpu, self.gpu.lib
        if self.which == "elementwise":
            g.check(g.raw.pb_elementwise(g.ctx, 0, L.EW_OPS["add"], 2, self.ptrs, self.codes, self.strides,
                                         1, self.shape, L.PB_F32, p_(self.dz)), "elementwise")
        else:
            g.check(g.raw.pb_reduce(g.ctx, 0, L.PB_REDUCE_SUM, L.PB_F32, p_(self.dx), 1, self.shape, 1,
                                    L.PB_F32, p_(self.dz)), "reduce")

    def e2e_setup(self):
        self.hz = np.empty(self.n if self.which == "elementwise" else 1, np.float32)
        self.pinned = [self.x, self.hz] + ([self.y] if self.y is not None else [])
        self.gpu.pin(self.pinned)

    def e2e_step(self):
        self.gpu.h2d(self.dx, self.x)
        if self.y is not None:
            self.gpu.h2d(self.dy, self.y)
        self.step()
        self.gpu.d2h_async(self.hz, self.dz)

    def e2e_bytes(self):
        return self.x.nbytes + (self.y.nbytes if self.y is not None else 0), self.hz.nbytes

    def violations(self):
        from oracle import numpy_backend, tolerance

        z = np.empty(self.n if self.which == "elementwise" else 1, np.float32)
        self.gpu.d2h(z, self.dz)
        if self.which == "elementwise":
            want = numpy_backend.elementwise("add", (self.x, self.y), np.float32)
            return int(np.sum(want.view(np.uint32) != z.view(np.uint32)))
        want = numpy_backend.reduce(self.x, (0,), False, np.float32)
        bound = 4 * self.x.size * tolerance.unit_roundoff(np.float32) * float(
            np.sum(np.abs(self.x), dtype=np.float64))
        return int(abs(float(z[0]) - float(want)) > bound)

    def cpu_prepare(self):
        if not hasattr(self, "x"):
            self._inputs()

    def cpu_step(self):
        from oracle import numpy_backend

        m = 1 << 25
        if self.which == "elementwise":
            numpy_backend.elementwise("add", (self.x[:m], self.y[:m]), np.float32)
            return 12.0 * m, "2^25 of the 2^28 elements (NumPy add)"
        numpy_backend.reduce(self.x[:m], (0,), False, np.float32)
        return 4.0 * m, "2^25 of the 2^28 values (NumPy sum)"


# ------------------------------------------------------ measurement --

def measure(w: Workload, gpu: Gpu, comm: Comm, args, dist: Dist, pk: dict) -> dict:
    """Everything the JSON line reports for one workload on this rank;
    collective steps (barriers, max) are taken identically on every rank."""
    w.setup(gpu, comm)
    for _ in range(args.warmup):
        w.step()
    gpu.sync()
    # One step captured into a CUDA graph and replayed (after the eager
    # warm-up has sized every internal buffer), unless it cannot be captured.
    # Every rank decides the same way: the steps may hold collectives.
    # With --launch auto the faster of the two is chosen on a short
    # calibration (max over ranks) before the timed region: a graph replay
    # saves the host's per-launch cost, eager launches keep the overlap of one
    # step's first kernel with the previous step's last (programmatic
    # dependent launch), which the boundary between two replays does not.
    use_graph = args.launch != "eager" and dist.max(0.0 if w.graphable() else 1.0) == 0.0
    graph = gpu.backend.capture(w.step) if use_graph else None
    alt = None
    try:
        if graph:
            calib = max(3, min(args.steps, 20))
            for _ in range(2):
                graph.launch()
            t_graph = dist.max(gpu.timer(graph.launch, calib))
            t_eager = dist.max(gpu.timer(w.step, calib))
            replay = not (args.launch == "auto" and t_eager < t_graph)
            alt = (("eager launches through the C ABI", w.step) if replay else
                   ("one step captured as a CUDA graph, replayed each step", graph.launch))
        else:
            replay = False
        step = graph.launch if replay else w.step
        gpu.sync()
        dist.barrier()
        with Clocks(gpu.backend.ordinal) as clocks:
            gpu.busy(step, dist)
            dist.barrier()
            l0 = gpu.launches()
            seconds = gpu.timer(step, args.steps)
            launches = graph.launches * args.steps if replay else gpu.launches() - l0
        if alt:
            dist.barrier()
            alt = (alt[0], dist.max(gpu.timer(alt[1], args.steps)))
    finally:
        if graph:
            graph.close()
    seconds = dist.max(seconds)
    total_units = dist.sum(w.units)

    # Main kernel alone (events around each launch), max over ranks.
    kt, kl = gpu.kernel_seconds(w.kernel_step, args.steps, graph=use_graph)
    kt = dist.max(kt or 0.0)
    more = w.more_kernels(use_graph) if hasattr(w, "more_kernels") else {}

    # End to end through the C ABI with pinned host buffers.
    w.e2e_setup()
    try:
        w.e2e_step()
        gpu.sync()
        dist.barrier()
        e2e_steps = max(1, min(args.steps, w.e2e_steps_cap))
        e2e_seconds = dist.max(gpu.timer(w.e2e_step, e2e_steps))
    finally:
        gpu.unpin(w.pinned)
    h2d, d2h = w.e2e_bytes()
    h2d, d2h = dist.sum(h2d), dist.sum(d2h)

    bad = int(dist.sum(float(w.violations())))

    scale = w.scale()
    rec = {
        "metric": w.metric(), "value": total_units * args.steps / seconds / scale, "unit": w.unit,
        "ms_per_step": seconds / args.steps * 1e3, "scaling": w.scaling, "dtype": w.dtype,
        "config": w.config(), "clocks": clocks.summary(), "gpu_launches": launches,
    }
    rec["config"]["launch"] = ("one step captured as a CUDA graph, replayed each step" if replay
                               else "eager launches through the C ABI")
    if graph:
        rec["config"]["launch_choice"] = args.launch
    if alt:
        rec["other_launch_mode"] = {"launch": alt[0], "value": total_units * args.steps / alt[1] / scale,
                                    "ms_per_step": alt[1] / args.steps * 1e3}
    rec["roofline"] = roofline(w, kt, pk)
    rec["kernel_ms"] = kt * 1e3
    if more:
        more["gemv_gbs"] = w.kernel_units / kt / 1e9 if kt else None
        rec["kernels"] = more
    rec["e2e"] = {"value": total_units * e2e_steps / e2e_seconds / scale, "unit": w.unit,
                  "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                  "ms_per_step": e2e_seconds / e2e_steps * 1e3,
                  "note": "whole job: every rank's pinned host inputs copied in and results read "
                          "back each step" + getattr(w, "e2e_how", "")}
    rec["parity_violations"] = bad
    if w.extra:
        rec.update(w.extra)
    return rec


def roofline(w: Workload, kt: float, pk: dict) -> dict:
    if not kt:
        return {"bound": w.bound, "achieved": None, "peak": None, "frac": None, "traffic": None}
    traffic, how = traffic_per_launch(w.kernel_key, w.kernel_units)
    if w.bound == "hbm":
        achieved = w.kernel_units / kt / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "peak_source": f"{pk['source']} copy bandwidth"}
    else:
        achieved = w.kernel_units / kt / 1e12
        if "f64" in w.dtype:
            peak, src = SPEC_FP64_TFLOPS, "B200 specification FP64 tensor 40 TFLOP/s (nominal)"
            alt = {"cublas_dgemm_measured": CUBLAS_DGEMM_TFLOPS,
                   "frac_of_cublas_dgemm": achieved / CUBLAS_DGEMM_TFLOPS}
        else:
            # 3xTF32: three TF32 products per logical product; TF32 runs at
            # half the bf16 rate.  A step of seconds runs at the sustained
            # (power-capped) clock, a short one at the burst clock.
            sustained = w.units >= 1e12
            bf16 = pk["bf16_tflops_sustained"] if sustained else pk["bf16_tflops"]
            peak = bf16 / 2 / 3
            src = (f"{pk['source']} bf16 {'sustained' if sustained else 'burst'} {bf16:.1f} / 2 (TF32) / 3 "
                   "(3xTF32)")
            alt = {"cublas_tf32_over_3": CUBLAS_TF32_TFLOPS / 3,
                   "frac_of_cublas_tf32_over_3": achieved / (CUBLAS_TF32_TFLOPS / 3)}
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": src, **alt}
    roof.update({"traffic": traffic, "traffic_source": how, "kernel": w.kernel_key,
                 "algorithmic_units_per_launch": w.kernel_units,
                 "kernel_ms_avg": kt * 1e3})
    return roof


def cpu_time(w: Workload, budget_s: float, max_steps: int, warmup: int = 1):
    """The reference's CPU path on w's bounded sample: (units/s, steps, sample)."""
    w.cpu_prepare()
    for _ in range(max(1, warmup)):
        w.cpu_step()
    done, steps, t0 = 0.0, 0, time.perf_counter()
    what = ""
    while True:
        units, what = w.cpu_step()
        done += units
        steps += 1
        if steps >= max_steps or time.perf_counter() - t0 > budget_s:
            break
    seconds = time.perf_counter() - t0
    return done / seconds / w.scale(), steps, what, seconds / steps


def make_workloads(args, dist):
    """Workloads in run order, each built when its turn comes (so only one
    config's inputs are held at a time)."""
    wl = args.workload
    if wl == "suite":
        yield Batched(args, dist)
        yield Gemm(args, dist, "gemm1024")
        yield GemvDot(args, dist)
        yield Norm(args, dist, False, np.float32)
        yield Norm(args, dist, True, np.float32)
        yield Norm(args, dist, False, np.float64)
        yield Norm(args, dist, True, np.float64)
        yield Gemm(args, dist, "gemm_f32")
        yield Gemm(args, dist, "gemm_f64")
        yield Vecmat(args, dist)
        yield Residual(args, dist)
        return
    dt = np.float64 if args.dtype == "f64" else np.float32
    yield {"batched": lambda: Batched(args, dist), "gemm1024": lambda: Gemm(args, dist, "gemm1024"),
           "gemm_f32": lambda: Gemm(args, dist, "gemm_f32"), "gemm_f64": lambda: Gemm(args, dist, "gemm_f64"),
           "gemv_dot": lambda: GemvDot(args, dist), "norm": lambda: Norm(args, dist, False, dt),
           "norm_rows": lambda: Norm(args, dist, True, dt), "vecmat": lambda: Vecmat(args, dist),
           "elementwise": lambda: Around(args, dist, "elementwise"),
           "reduce": lambda: Around(args, dist, "reduce"),
           "residual": lambda: Residual(args, dist)}[wl]()


class Residual(Workload):
    """b - A @ x with the subtraction fused into the GEMV epilogue (the
    compiled-plan residual, src/openpacho/_compiler.py:157-176), float32
    16384^2, against the unfused GEMV + elementwise subtract pair."""

    name = "residual_f32_16384"

    def metric(self):
        return "residual b - A @ x (A 16384x16384 float32, fused GEMV epilogue) HBM throughput"

    def config(self):
        return {"workload": "b - A @ x, A 16384x16384 f32, x and b 16384, U[-1,1], default_rng(7)",
                "parallelism": f"replicas x{self.world}",
                "l2": "A (1.07 GB) larger than the 126 MB L2; no flush needed"}

    def _inputs(self):
        rng = np.random.default_rng(7)
        self.A = rng.uniform(-1, 1, (16384, 16384)).astype(np.float32)
        self.x = rng.uniform(-1, 1, 16384).astype(np.float32)
        self.b = rng.uniform(-1, 1, 16384).astype(np.float32)

    def setup(self, gpu, comm):
        self.gpu = gpu
        self._inputs()
        self.dA, self.dx, self.db = (gpu.upload(t) for t in (self.A, self.x, self.b))
        self.dr = gpu.empty((16384,), np.float32)
        self.dy = gpu.empty((16384,), np.float32)
        self.units = self.kernel_units = 4.0 * (16384 * 16384 + 3 * 16384)
        self.kernel_key = "residual:gemv"

    def step(self):
        g = self.gpu
        g.check(g.raw.pb_gemv_residual(g.ctx, 0, g.lib.PB_F32, 16384, 16384, p_(self.dA), p_(self.dx),
                                       p_(self.db), p_(self.dr)), "gemv_residual")

    def unfused(self):
        g, L = self.gpu, self.gpu.lib
        g.check(g.raw.pb_gemv(g.ctx, 0, L.PB_F32, 16384, 16384, p_(self.dA), p_(self.dx), p_(self.dy)),
                "gemv")
        ptrs = (C.c_void_p * 2)(self.db.ptr, self.dy.ptr)
        codes = (C.c_int * 2)(L.PB_F32, L.PB_F32)
        g.check(g.raw.pb_elementwise(g.ctx, 0, L.EW_OPS["subtract"], 2, ptrs, codes, L.i64_array([1, 1]), 1,
                                     L.i64_array([16384]), L.PB_F32, p_(self.dy)), "subtract")

    def more_kernels(self, graph=False):
        if graph:
            self.unfused()
            with self.gpu.backend.capture(self.unfused) as g:
                t = self.gpu.timer(g.launch, self.args.steps) / self.args.steps
        else:
            t = self.gpu.timer(self.unfused, self.args.steps) / self.args.steps
        return {"unfused_gemv_then_subtract_ms": t * 1e3,
                "unfused_bytes": 4.0 * (16384 * 16384 + 2 * 16384 + 16384) + 12.0 * 16384,
                "fused_bytes": self.units}

    def e2e_setup(self):
        self.hr = np.empty(16384, np.float32)
        self.pinned = [self.A, self.x, self.b, self.hr]
        self.gpu.pin(self.pinned)

    def e2e_step(self):
        for h, dbuf in ((self.A, self.dA), (self.x, self.dx), (self.b, self.db)):
            self.gpu.h2d(dbuf, h)
        self.step()
        self.gpu.d2h_async(self.hr, self.dr)

    def e2e_bytes(self):
        return self.A.nbytes + self.x.nbytes + self.b.nbytes, self.hr.nbytes

    def violations(self):
        from oracle import numpy_backend, tolerance

        r = np.empty(16384, np.float32)
        self.gpu.d2h(r, self.dr)
        # The product is rounded to float32 before the subtraction
        # (src/openpacho/_gemv.py:1-6), so the bound is the GEMV's plus the
        # rounding of the difference.
        y = numpy_backend.matmul(self.A, self.x)
        want = numpy_backend.elementwise("subtract", (self.b, y), np.float32)
        bound = tolerance.gemm_bound(self.A, self.x) + tolerance.unit_roundoff(np.float32) * (
            np.abs(self.b.astype(np.float64)) + np.abs(y.astype(np.float64)))
        return int(np.sum(~(np.abs(r.astype(np.float64) - want.astype(np.float64)) <= 2 * bound)))

    def cpu_prepare(self):
        if not hasattr(self, "A"):
            self._inputs()

    def cpu_step(self):
        from oracle import numpy_backend

        y = numpy_backend.matmul(self.A, self.x)
        numpy_backend.elementwise("subtract", (self.b, y), np.float32)
        return 4.0 * (16384 * 16384 + 3 * 16384), "the full residual (NumPy @ -> OpenBLAS sgemv, then subtract)"


# ----------------------------------------------------- reference arm --

def reference_arm(args, dist: Dist):
    """The reference's CPU implementation of the path (the NumPy-backend
    restatement in oracle/, src/openpacho/backends.py:139-142 and
    src/openpacho/_norm.py:44-52) on the host cores, same workloads, configs
    and units as the b200 arm.  Under torchrun rank 0 alone runs."""
    if dist.rank != 0:
        return 0
    limiter, threads = blas_threads_all()
    records = {}
    headline = None
    for w in make_workloads(args, dist):
        budget = 20.0 if headline is None else 4.0
        value, steps, what, sec = cpu_time(w, budget, max_steps=args.steps, warmup=min(args.warmup, 2))
        # Configs are built as on the b200 arm for this world size.
        if isinstance(w, Norm) and not w.rows_mode and dist.world > 1:
            w.exchange = "NVLink peer mailboxes"
        rec = {"metric": w.metric(), "value": value, "unit": w.unit, "ms_per_step": sec * 1e3,
               "steps": steps, "scaling": w.scaling, "dtype": w.dtype, "config": w.config(),
               "cpu_baseline": {"value": value, "unit": w.unit, "cores": threads, "kind": "port",
                                "sample": f"{steps} steps of {what}; OpenBLAS threads {threads} of "
                                          f"{cpu_cores()} host cores"},
               "e2e": {"value": value, "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if headline is None:
            headline = rec
        else:
            records[w.name] = rec
    line = {
        "impl": "reference", "metric": headline["metric"], "value": headline["value"],
        "unit": headline["unit"], "n_gpus": args.gpus, "steps": headline["steps"], "warmup": args.warmup,
        "ms_per_step": headline["ms_per_step"], "higher_is_better": True, "scaling": headline["scaling"],
        "vs_baseline": None, "dtype": headline["dtype"], "data": DATA, "config": headline["config"],
        "cpu_baseline": headline["cpu_baseline"], "e2e": headline["e2e"],
    }
    if records:
        line["configs"] = records
    print(json.dumps(line))
    del limiter
    return 0


DATA = "synthetic (seeded numpy default_rng, BASELINE distributions)"


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


def b200_arm(args, dist: Dist) -> int:
    gpu = Gpu(dist.local)
    comm = Comm(gpu, dist)
    pk = peaks()
    limiter, threads = blas_threads_all() if dist.rank == 0 else (None, 0)
    records = {}
    try:
        for w in make_workloads(args, dist):
            rec = measure(w, gpu, comm, args, dist, pk)
            if dist.world == 1 and dist.rank == 0 and not args.no_cpu_baseline:
                budget = 15.0 if not records else 3.0
                value, steps, what, _ = cpu_time(w, budget, max_steps=200)
                rec["cpu_baseline"] = {"value": value, "unit": w.unit, "cores": threads, "kind": "port",
                                       "sample": f"{steps} steps of {what}; OpenBLAS threads {threads} "
                                                 f"of {cpu_cores()} host cores"}
            records[w.name] = rec
            del w
            gpu.backend.release_cached_memory()
    finally:
        comm.close()
    if dist.rank != 0:
        return 0
    names = list(records)
    head = records.pop(names[0])
    line = {
        "metric": head.pop("metric"), "value": head.pop("value"), "unit": head.pop("unit"),
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head.pop("ms_per_step"), "higher_is_better": True,
        "scaling": head.pop("scaling"), "vs_baseline": None, "dtype": head.pop("dtype"),
        "data": DATA, "config": head.pop("config"),
    }
    line.update(head)
    if records:
        line["configs"] = records
        line["parity_violations_all"] = int(line["parity_violations"] + sum(
            r["parity_violations"] for r in records.values()))
        line["gpu_launches_all"] = int(line["gpu_launches"] + sum(r["gpu_launches"] for r in records.values()))
    print(json.dumps(line))
    del limiter
    return 0


def pool_arm(args) -> int:
    """BASELINE config 5 through one backend object that holds N GPUs in one
    process (``B200Backend("0-<N-1>")``): A and B live on the primary, the
    product is split into row blocks by the backend itself, and the timed
    step includes the NVLink transfers (A blocks and B out, C blocks back).
    Run as one process, not under torchrun; the single-GPU product of the
    same inputs is timed beside it."""
    from pacho_b200 import B200Backend, DeviceArray

    f64 = args.workload == "pool_f64"
    n = args.n or (8192 if f64 else 16384)
    dtype = np.float64 if f64 else np.float32
    be = B200Backend(f"0-{args.gpus - 1}") if args.gpus > 1 else B200Backend(0)
    A, B = gen_gemm(4, n, dtype)
    dA = DeviceArray(be, be.upload(A), A.shape, dtype)
    dB = DeviceArray(be, be.upload(B), B.shape, dtype)
    lib, ctx = be._lib, be._ctx

    def step():
        return be.matmul(dA, dB, (n, n), dtype)

    def timed(fn, reps):
        be.synchronize()
        _lib_check(lib.pb_timer_start(ctx, 0), "timer")
        for _ in range(reps):
            out = fn()
            del out
        ms = C.c_float()
        _lib_check(lib.pb_timer_stop(ctx, 0, C.byref(ms)), "timer")
        return ms.value / 1e3

    for _ in range(args.warmup):
        step()
    splits0 = be._pool.splits if be._pool else 0
    with Clocks(be.ordinal) as clocks:
        seconds = timed(step, args.steps)
    split = (be._pool.splits - splits0) == args.steps if be._pool else False
    out = step()
    host = np.empty((n, n), dtype)
    _lib_check(lib.pb_d2h(ctx, 0, C.c_void_p(host.ctypes.data), C.c_void_p(out.ptr), host.nbytes), "d2h")
    from oracle import numpy_backend, tolerance  # the checker, outside the timed step

    rows = np.random.default_rng(0).choice(n, size=64, replace=False)
    bad = tolerance.gemm_violations(host[rows], numpy_backend.matmul(A[rows], B), A[rows], B)
    one = None
    if be._pool:
        gain = be.split_min_gain
        be.split_min_gain = 0.0  # never split: the primary alone
        for _ in range(2):
            step()
        one = timed(step, max(1, min(args.steps, 5))) / max(1, min(args.steps, 5))
        be.split_min_gain = gain
    flops = 2.0 * n ** 3
    value = flops * args.steps / seconds / 1e12
    line = {
        "metric": f"{np.dtype(dtype).name} GEMM {n}^3 TFLOP/s, one process over {args.gpus} GPUs",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": seconds / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64 (DMMA)" if f64 else "f32 (3xTF32)",
        "data": DATA,
        "config": {"workload": f"BASELINE config 5: {np.dtype(dtype).name} {n}^3, N(0,1), default_rng(4)",
                   "parallelism": (f"one backend over {args.gpus} GPUs: row blocks of A and the whole B "
                                   "sent from the primary over NVLink, C blocks copied back, all inside "
                                   "the timed step" if args.gpus > 1 else "one GPU"),
                   "l2": "operands and output far above the 126 MB L2"},
        "split_every_step": split, "clocks": clocks.summary(), "parity_violations": int(bad),
        "peer_access_all_pairs": bool(be._pool.all_peer) if be._pool else None,
    }
    if one:
        line["one_gpu"] = {"ms_per_step": one * 1e3, "value": flops / one / 1e12,
                           "speedup": one / (seconds / args.steps)}
    print(json.dumps(line))
    be.close()
    return 0


def _lib_check(status, what):
    from pacho_b200 import _lib

    _lib.check(status, what)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--workload", default="suite",
                        choices=("suite", "batched", "gemm1024", "gemv_dot", "norm", "norm_rows", "gemm_f32",
                                 "gemm_f64", "vecmat", "elementwise", "reduce", "residual", "pool_f32",
                                 "pool_f64"),
                        help="pool_f32 / pool_f64: config 5 through one backend over --gpus GPUs in one "
                             "process (not under torchrun)")
    parser.add_argument("--dtype", choices=("f32", "f64"), default="f32", help="norm workloads")
    parser.add_argument("--n", type=int, default=0,
                        help="GEMM / vecmat / around-path size override (profiling captures); 0 = BASELINE")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--launch", choices=("auto", "graph", "eager"), default="auto",
                        help="replay each step as a captured CUDA graph, launch it eagerly, or "
                             "take the faster of the two on a calibration run (auto)")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    if args.steps < 1:
        parser.error("--steps must be >= 1")
    if args.workload.startswith("pool"):
        if args.impl == "reference":
            parser.error("the pool workloads have no reference arm; the reference drives one device")
        return pool_arm(args)
    dist = Dist()
    try:
        if args.impl == "reference":
            return reference_arm(args, dist)
        return b200_arm(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    sys.exit(main())
