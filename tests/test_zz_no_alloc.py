"""pb_dot_noalloc: the DOT entry point for callers that cannot call cudaMalloc.

Some callers own every byte of device memory through their own allocator, or
run code that must never enter the driver's allocator (it can block, or fail
once memory is fully reserved); they cannot let the library grow its scratch
buffer.  pb_dot_noalloc keeps its partial sums in a fixed device array inside
the library instead.  These tests drive it through the C ABI:

* two calls in a row give exactly pb_dot's bits (same kernel, same plan, same
  fixed merge order) and stay within the DOT bound 4*K*u*sum|x*y| of the
  NumPy-backend oracle;
* in a fresh process, calls made before any pb_dot change neither the
  context's memory pool (reserved and used bytes), nor its scratch buffer
  (still 0 bytes), nor the device's free memory.

They live in a file of their own that pytest collects last, and pass alone in
a fresh process or after the other tests.
"""

from __future__ import annotations

import ctypes as C
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import numpy_backend, tolerance
from pacho_b200 import _lib

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _dot(backend, fn, code, n, dx, dy, dtype):
    out = backend.empty((1,), dtype)
    _lib.check(fn(backend._ctx, 0, code, n, C.c_void_p(dx.ptr), C.c_void_p(dy.ptr),
                  C.c_void_p(out.ptr)), fn.__name__)
    host = np.empty(1, dtype)
    _lib.check(backend._lib.pb_d2h(backend._ctx, 0, C.c_void_p(host.ctypes.data),
                                   C.c_void_p(out.ptr), host.nbytes), "pb_d2h")
    return host.reshape(())


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("n", [0, 1, 63, 4097, (1 << 20) + 3, 1 << 26])
def test_noalloc_dot_matches_pb_dot_on_two_calls(b200, dtype, n):
    rng = np.random.default_rng(9200 + n)
    x = rng.uniform(-1, 1, n).astype(dtype)
    y = rng.uniform(-1, 1, n).astype(dtype)
    dx, dy = b200.upload(x), b200.upload(y)
    code = _lib.dtype_code(dtype)
    lib = b200._lib
    reference = _dot(b200, lib.pb_dot, code, n, dx, dy, dtype)
    want = numpy_backend.dot(x, y)
    for _ in range(2):
        got = _dot(b200, lib.pb_dot_noalloc, code, n, dx, dy, dtype)
        assert got.tobytes() == reference.tobytes()
        assert tolerance.gemm_violations(got, want, x, y) == 0


_FRESH = r"""
import ctypes as C, json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from pacho_b200 import _lib
lib = _lib.load()
ctx = C.c_void_p()
_lib.check(lib.pb_init(1, (C.c_int * 1)(0), C.byref(ctx)), "pb_init")
n = 1 << 26
rng = np.random.default_rng(7)
x = rng.uniform(-1, 1, n).astype(np.float32)
y = rng.uniform(-1, 1, n).astype(np.float32)
ptrs = []
for host in (x, y, np.zeros(2, np.float32)):
    p = C.c_void_p()
    _lib.check(lib.pb_alloc(ctx, 0, host.nbytes, C.byref(p)), "pb_alloc")
    _lib.check(lib.pb_h2d(ctx, 0, p, C.c_void_p(host.ctypes.data), host.nbytes, 1), "pb_h2d")
    ptrs.append(p)
dx, dy, dout = ptrs
out2 = C.c_void_p(dout.value + 4)
# One kernel launch first (a fill, from the same module as the DOT kernel),
# so that what the driver sets up at a context's first launch is not counted.
_lib.check(lib.pb_fill(ctx, 0, _lib.PB_F32, dout, 2, 0.0), "pb_fill")
_lib.check(lib.pb_sync(ctx, 0), "pb_sync")

def stats():
    v = [C.c_size_t() for _ in range(4)]
    _lib.check(lib.pb_memory_stats(ctx, 0, *(C.byref(s) for s in v)), "pb_memory_stats")
    return [s.value for s in v]

def read(ptr):
    h = np.empty(1, np.float32)
    _lib.check(lib.pb_d2h(ctx, 0, C.c_void_p(h.ctypes.data), ptr, 4), "pb_d2h")
    return h

before = stats()
values = []
for _ in range(2):
    _lib.check(lib.pb_dot_noalloc(ctx, 0, _lib.PB_F32, n, dx, dy, dout), "pb_dot_noalloc")
    _lib.check(lib.pb_sync(ctx, 0), "pb_sync")
    values.append(read(dout))
after = stats()
_lib.check(lib.pb_dot(ctx, 0, _lib.PB_F32, n, dx, dy, out2), "pb_dot")
with_pb_dot = stats()
ref = read(out2)
print(json.dumps({"before": before, "after": after, "after_pb_dot": with_pb_dot,
                  "bits": [v.tobytes().hex() for v in values], "pb_dot_bits": ref.tobytes().hex()}))
lib.pb_destroy(ctx)
"""


def test_noalloc_dot_allocates_nothing_in_a_fresh_process(b200):
    """pool_reserved, pool_used, scratch_bytes, device_free: unchanged by two
    pb_dot_noalloc calls made before any other library call needing scratch;
    the first pb_dot afterwards grows the scratch (the check can see it)."""
    proc = subprocess.run([sys.executable, "-c", _FRESH, str(ROOT / "open-pacho_b200")],
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-3000:]
    r = json.loads(proc.stdout.strip().splitlines()[-1])
    assert r["after"] == r["before"], r
    assert r["before"][2] == 0  # no scratch buffer at all
    assert r["after_pb_dot"][2] > 0  # pb_dot did grow one: the probe is live
    assert r["bits"][0] == r["bits"][1] == r["pb_dot_bits"]
