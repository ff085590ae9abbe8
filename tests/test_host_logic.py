"""Host-side routing of B200Backend, checked on CPU with a recording library.

The fake records the C calls (it computes nothing); the assertions pin the
shapes, strides and kernel entry points the backend chooses, mirroring the
reference's matmul/norm routing (src/openpacho/_cuda.py:493-517,
src/openpacho/_norm.py:12-25).
"""

from __future__ import annotations

import ctypes as C
import threading
import weakref

import numpy as np
import pytest

from pacho_b200 import _lib
from pacho_b200.backend import B200Backend, _matrix_strides


class RecordingLib:
    def __init__(self):
        self.calls = []
        self.next_ptr = 0x1000

    def pb_alloc(self, ctx, dev, nbytes, out):
        C.cast(out, C.POINTER(C.c_void_p))[0] = self.next_ptr
        self.next_ptr += ((nbytes + 255) // 256) * 256
        return 0

    def pb_free(self, ctx, dev, ptr):
        return 0

    def __getattr__(self, name):
        def call(*args):
            self.calls.append((name, args))
            return 0

        return call


class Operand:
    def __init__(self, shape, dtype, ptr):
        self.shape, self.dtype, self._data = tuple(shape), np.dtype(dtype), type("D", (), {"ptr": ptr})()

    ndim = property(lambda self: len(self.shape))


@pytest.fixture
def backend():
    b = object.__new__(B200Backend)
    b._lib = RecordingLib()
    b._ctx = C.c_void_p(1)
    b._lock = threading.RLock()
    b._closed = False
    b._buffers = weakref.WeakSet()
    yield b
    b._closed = True


def _ints(arr, n):
    return [arr[i] for i in range(n)]


def test_matrix_strides_follow_numpy_broadcasting():
    assert _matrix_strides((8, 16), (8, 16)) == [16, 1]
    assert _matrix_strides((8, 16), (1, 16)) == [0, 1]
    assert _matrix_strides((2, 3), (2, 1)) == [1, 0]
    assert _matrix_strides((2, 3), ()) == [0, 0]
    assert _matrix_strides((4, 2, 3), (3,)) == [0, 0, 1]


@pytest.mark.parametrize(
    "ashape,bshape,entry",
    [((7,), (7,), "pb_dot"), ((3, 5), (5,), "pb_gemv"), ((2, 3, 257), (257,), "pb_gemv"),
     ((5,), (5, 4), "pb_gemm"), ((3, 33, 17), (3, 17, 65), "pb_gemm")],
)
def test_matmul_routes_like_the_reference(backend, ashape, bshape, entry):
    a, b = Operand(ashape, np.float32, 0x10), Operand(bshape, np.float32, 0x20)
    shape = np.matmul(np.zeros(ashape), np.zeros(bshape)).shape
    backend.matmul(a, b, shape, np.float32)
    (name, args), = backend._lib.calls
    assert name == entry
    if entry == "pb_gemv":
        assert args[3] == int(np.prod(ashape[:-1])) and args[4] == ashape[-1]


def test_broadcast_batch_is_one_gemm_call(backend):
    # (8,16,512,256) @ (1,16,256,384).
    a, b = Operand((8, 16, 512, 256), np.float32, 0x10), Operand((1, 16, 256, 384), np.float32, 0x20)
    backend.matmul(a, b, (8, 16, 512, 384), np.float32)
    (name, args), = backend._lib.calls
    assert name == "pb_gemm"
    _, dev, dtype, ndim, shape, astr, bstr, M, N, K = args[:10]
    assert (dtype, ndim, M, N, K) == (_lib.PB_F32, 2, 512, 384, 256)
    assert _ints(shape, 2) == [8, 16] and _ints(astr, 2) == [16, 1] and _ints(bstr, 2) == [0, 1]


def test_vector_matrix_broadcasts_the_vector(backend):
    a, b = Operand((7,), np.float64, 0x10), Operand((2, 7, 3), np.float64, 0x20)
    backend.matmul(a, b, (2, 3), np.float64)
    (name, args), = backend._lib.calls
    assert name == "pb_gemm" and args[2] == _lib.PB_F64
    assert _ints(args[5], 1) == [0] and _ints(args[6], 1) == [1] and args[7:10] == (1, 3, 7)


def test_empty_output_launches_nothing(backend):
    a, b = Operand((0, 5, 7), np.float32, 0x10), Operand((1, 7, 3), np.float32, 0x20)
    backend.matmul(a, b, (0, 5, 3), np.float32)
    assert backend._lib.calls == []


@pytest.mark.parametrize(
    "shape,axes,expect",
    [((65536, 4096), (1,), ("pb_norm", 65536, 4096, 1)),
     ((1 << 28,), (0,), ("pb_norm", 1, 1 << 28, 1)),
     ((64, 1024), (0,), ("pb_norm", 1, 64, 1024)),
     ((2, 3, 4, 5), (1, 2), ("pb_norm", 2, 12, 5)),
     ((3, 5, 7), (0, 1, 2), ("pb_norm", 1, 105, 1)),
     ((), (), ("pb_norm", 1, 1, 1))],
)
def test_norm_contiguous_axes_use_the_3d_view(backend, shape, axes, expect):
    backend.norm(Operand(shape, np.float32, 0x10), axes, False, np.float32)
    (name, args), = backend._lib.calls
    assert (name, args[3], args[4], args[5]) == expect


def test_norm_general_axes_use_strides(backend):
    # tests/test_stable_norm.py uses shape (3,5,7) with axis=(2,0).
    backend.norm(Operand((3, 5, 7), np.float64, 0x10), (0, 2), True, np.float64)
    (name, args), = backend._lib.calls
    assert name == "pb_norm_strided"
    assert args[3] == 1 and _ints(args[4], 1) == [5] and _ints(args[5], 1) == [7]
    assert args[6] == 2 and _ints(args[7], 2) == [3, 7] and _ints(args[8], 2) == [35, 1]


def test_validate_dtype(backend):
    from pacho_b200.exceptions import UnsupportedDtypeError

    assert backend.validate_dtype("float32") == np.float32
    assert backend.validate_dtype("bool") == np.bool_
    for bad in ("int32", "float16", "complex64", ">f4"):
        with pytest.raises(UnsupportedDtypeError):
            backend.validate_dtype(bad)


def test_padding_hint_is_declined(backend):
    assert backend.prepare_padded_matmul((33, 17), (17, 65), (33, 65), np.float32) is None


def test_elementwise_broadcast_strides_and_codes(backend):
    a = Operand((4, 1, 3), np.float32, 0x100)
    b = Operand((5, 1), np.float64, 0x200)
    backend.elementwise("add", [a, b], (4, 5, 3), np.float64)
    (name, args), = [c for c in backend._lib.calls if c[0] == "pb_elementwise"]
    assert args[2] == _lib.EW_OPS["add"] and args[3] == 2
    assert [args[5][i] for i in range(2)] == [_lib.PB_F32, _lib.PB_F64]
    # a: (4,1,3) -> strides (3, 0, 1); b: (5,1) padded (1,5,1) -> (0, 1, 0)
    assert [args[6][i] for i in range(6)] == [3, 0, 1, 0, 1, 0]
    assert args[7] == 3 and [args[8][i] for i in range(3)] == [4, 5, 3]
    assert args[9] == _lib.PB_F64


def test_elementwise_names_and_limits(backend):
    assert _lib.EW_OPS["divide"] == _lib.EW_OPS["true_divide"]
    assert len(set(_lib.EW_OPS.values())) == 23
    with pytest.raises(NotImplementedError):
        backend.elementwise("arctan2", [], (1,), np.float32)
    with pytest.raises(NotImplementedError):
        backend.elementwise("add", [], (1,) * 9, np.float32)
    assert backend.elementwise("add", [], (0, 3), np.float32) is not None  # empty: no launch
    assert not [c for c in backend._lib.calls if c[0] == "pb_elementwise"]


def test_reduce_mask_gather_and_float_only_paths(backend):
    x = Operand((2, 3, 4), np.bool_, 0x300)
    backend.reduce(x, (0, 2), False, np.float32)
    (name, args), = [c for c in backend._lib.calls if c[0] == "pb_reduce"]
    assert args[2] == _lib.PB_REDUCE_SUM and args[3] == _lib.PB_BOOL and args[7] == 0b101
    assert args[8] == _lib.PB_F32
    with pytest.raises(NotImplementedError):
        backend.reduce(x, (0,), False, np.bool_)  # boolean sums, as in the reference
    with pytest.raises(ValueError):
        backend.reduce(x, (0,), False, np.float32, operation="prod")
    backend.gather(Operand((5, 5), np.float32, 0x400), (5,), 0, (6,))
    (name, args), = [c for c in backend._lib.calls if c[0] == "pb_gather"]
    assert args[4] == 1 and args[6] == 0 and args[7][0] == 6
    m = Operand((4, 4), np.bool_, 0x500)
    with pytest.raises(NotImplementedError):
        backend.matmul(m, m, (4, 4), np.bool_)
    with pytest.raises(NotImplementedError):
        backend.norm(m, (0, 1), False, np.bool_)

