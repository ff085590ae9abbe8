"""pb_dot_noalloc: the DOT entry point for callers that cannot call cudaMalloc.

Some callers own every byte of device memory through their own allocator, or
run code that must never enter the driver's allocator; they cannot let the
library grow its scratch buffer.  pb_dot_noalloc keeps its partial sums in a
fixed device array inside the library instead.  This test drives it through
the C ABI and checks that two calls in a row give what pb_dot gives, within
the DOT tolerance used everywhere else (4*K*u*sum|x*y|).  It runs alone in a
fresh process or after the other tests; it lives in a file of its own that
pytest collects last.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import tolerance
from pacho_b200 import _lib

pytestmark = pytest.mark.gpu


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
    for _ in range(2):
        got = _dot(b200, lib.pb_dot_noalloc, code, n, dx, dy, dtype)
        assert tolerance.gemm_violations(got, reference, x, y) == 0
