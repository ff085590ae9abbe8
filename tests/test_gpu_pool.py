"""Several GPUs behind one backend in one process (``device="0-1"``, ...).

A product the pool splits must equal the single-GPU product: bit for bit
where each block runs the same kernel configuration as the whole (every
block still has a full wave of tiles, so no split-K), and within the GEMM
bound of the NumPy-backend oracle everywhere.  Memory-bound operations stay
on the primary.  Needs two or more GPUs.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import front as pb
from oracle import numpy_backend, tolerance
from pacho_b200 import B200Backend, _lib

pytestmark = pytest.mark.gpu


def _gpus():
    n = C.c_int(0)
    return n.value if _lib.load().pb_device_count(C.byref(n)) == 0 else 0


needs_two = pytest.mark.skipif(_gpus() < 2, reason="needs two or more GPUs")


@pytest.fixture(scope="module")
def pair():
    be = B200Backend("0-1")
    be.split_min_gain = 1e9  # split every product that has a cut
    yield be
    be.close()


@pytest.fixture(scope="module")
def single():
    be = B200Backend(0)
    yield be
    be.close()


def _check(got, a, b):
    want = numpy_backend.matmul(a, b)
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= 2 * tolerance.gemm_bound(a, b) + 1e-300)


@needs_two
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_row_split_equals_one_gpu_bit_for_bit(pair, single, dtype):
    rng = np.random.default_rng(11)
    a = rng.standard_normal((4096, 512)).astype(dtype)
    b = rng.standard_normal((512, 4096)).astype(dtype)
    before = pair._pool.splits
    got = (pb.asarray(a, backend=pair) @ pb.asarray(b, backend=pair)).numpy()
    assert pair._pool.splits == before + 1
    one = (pb.asarray(a, backend=single) @ pb.asarray(b, backend=single)).numpy()
    assert got.tobytes() == one.tobytes()
    _check(got, a, b)


@needs_two
@pytest.mark.parametrize("shapes", [((1000, 300), (300, 200)), ((129, 64), (64, 65)),
                                    ((4, 512, 256), (256, 384)), ((6, 2, 128, 96), (6, 2, 96, 160)),
                                    ((3, 257, 33), (3, 33, 129))])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_split_shapes_meet_the_gemm_bound(pair, shapes, dtype):
    rng = np.random.default_rng(sum(map(sum, shapes)))
    a = rng.uniform(-1, 1, shapes[0]).astype(dtype)
    b = rng.uniform(-1, 1, shapes[1]).astype(dtype)
    before = pair._pool.splits
    got = (pb.asarray(a, backend=pair) @ pb.asarray(b, backend=pair)).numpy()
    assert pair._pool.splits == before + 1
    _check(got, a, b)


@needs_two
def test_uncut_layouts_and_vectors_stay_on_the_primary(pair):
    rng = np.random.default_rng(3)
    cases = [((512, 256), (4, 256, 384)),          # A broadcast along the batch
             ((2, 3, 64, 32), (3, 32, 16)),        # B batched along an inner dim only
             ((1000, 300), (300,)),                # GEMV
             ((300,), (300,))]                     # DOT
    for sa, sb in cases:
        a = rng.standard_normal(sa).astype(np.float32)
        b = rng.standard_normal(sb).astype(np.float32)
        before = pair._pool.splits
        got = (pb.asarray(a, backend=pair) @ pb.asarray(b, backend=pair)).numpy()
        assert pair._pool.splits == before
        _check(np.asarray(got), a, b)


@needs_two
def test_small_products_are_not_split_by_default():
    be = B200Backend("0-1")
    try:
        a = np.ones((1024, 1024), np.float32)
        got = (pb.asarray(a, backend=be) @ pb.asarray(a, backend=be)).numpy()
        assert be._pool.splits == 0
        assert np.all(got == 1024)
    finally:
        be.close()


@needs_two
def test_every_gpu_of_the_box(single):
    n = _gpus()
    be = B200Backend(f"0-{n - 1}")
    be.split_min_gain = 1e9
    try:
        rng = np.random.default_rng(n)
        a = rng.standard_normal((128 * n * 3 + 17, 640)).astype(np.float32)
        b = rng.standard_normal((640, 768)).astype(np.float32)
        got = (pb.asarray(a, backend=be) @ pb.asarray(b, backend=be)).numpy()
        assert be._pool.splits == 1
        _check(got, a, b)
    finally:
        be.close()
