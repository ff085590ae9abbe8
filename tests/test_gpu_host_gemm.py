"""pb_gemm_host: products of host arrays with the uploads, the GEMM pieces and
the downloads overlapped (B200Backend.matmul_host).

Every piece runs the same kernels as pb_gemm on device buffers, so the
result meets the GEMM bound of the NumPy-backend oracle, and it carries the
bits of the device product wherever the pieces keep the kernel's
configuration (full waves of tiles, no K split).
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import front as pb
from oracle import numpy_backend, tolerance
from pacho_b200 import _lib

pytestmark = pytest.mark.gpu


def _check(got, a, b):
    want = numpy_backend.matmul(a, b)
    assert got.shape == want.shape and got.dtype == want.dtype
    assert tolerance.gemm_violations(got, want, a, b) == 0


@pytest.mark.parametrize("shapes", [
    ((8, 16, 512, 256), (1, 16, 256, 384)),    # config 3: pieces along the 8 outer batches
    ((1, 16, 512, 256), (1, 16, 256, 384)),    # pieces along the 16 inner ones, B sliced too
    ((4, 300, 64), (4, 64, 200)),              # B batched with A
    ((2048, 1024), (1024, 768)),               # rows of A
    ((3000, 96), (96, 4100)),                  # rows, wide output
    ((512, 256), (4, 256, 384)),               # A broadcast: one piece
    ((2, 3, 64, 32), (3, 32, 16)),             # small: one piece
    ((5, 7), (7, 3)),
])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_host_product_meets_the_gemm_bound(b200, shapes, dtype):
    rng = np.random.default_rng(sum(map(sum, shapes)))
    a = rng.standard_normal(shapes[0]).astype(dtype)
    b = rng.standard_normal(shapes[1]).astype(dtype)
    _check(b200.matmul_host(a, b), a, b)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_host_product_equals_the_device_product(b200, dtype):
    """Config 3's pieces (one outer batch each, 128 tiles) and the whole
    product both run without a K split: the same bits."""
    rng = np.random.default_rng(2)
    a = rng.standard_normal((8, 16, 512, 256)).astype(dtype)
    b = rng.standard_normal((1, 16, 256, 384)).astype(dtype)
    host = b200.matmul_host(a, b)
    dev = (pb.asarray(a, backend=b200) @ pb.asarray(b, backend=b200)).numpy()
    assert host.tobytes() == dev.tobytes()
    assert b200.matmul_host(a, b, chunks=1).tobytes() == host.tobytes()
    assert b200.matmul_host(a, b, chunks=3).tobytes() == host.tobytes()


def test_pinned_operands_and_repeated_calls(b200):
    rng = np.random.default_rng(5)
    a = rng.standard_normal((4096, 512)).astype(np.float32)
    b = rng.standard_normal((512, 2048)).astype(np.float32)
    lib = b200._lib
    for arr in (a, b):
        assert lib.pb_host_register(C.c_void_p(arr.ctypes.data), arr.nbytes) == _lib.PB_OK
    try:
        first = b200.matmul_host(a, b)
        for _ in range(3):
            assert b200.matmul_host(a, b).tobytes() == first.tobytes()
        _check(first, a, b)
    finally:
        for arr in (a, b):
            lib.pb_host_unregister(C.c_void_p(arr.ctypes.data))


def test_empty_and_k0_products(b200):
    a = np.ones((3, 0), np.float32)
    b = np.ones((0, 5), np.float32)
    assert np.array_equal(b200.matmul_host(a, b), np.zeros((3, 5), np.float32))
    assert b200.matmul_host(np.ones((0, 4)), np.ones((4, 6))).shape == (0, 6)
    with pytest.raises(ValueError):
        b200.matmul_host(np.ones((3, 4)), np.ones((5, 6)))


def test_special_values_through_the_host_path(b200):
    rng = np.random.default_rng(21)
    a = rng.standard_normal((1024, 512)).astype(np.float32)
    b = rng.standard_normal((512, 1024)).astype(np.float32)
    a[0, 5], b[5, 7] = np.inf, 0.0
    a[700, 3] = np.nan
    with np.errstate(all="ignore"):
        want = numpy_backend.matmul(a, b)
    got = b200.matmul_host(a, b)
    assert tolerance.gemm_violations(got, want, a, b) == 0
