"""Drop-in check against the real OpenPacho front end (CPU, skipped without it).

``pacho_b200.register()`` installs "b200" into OpenPacho's hard-coded backend
dispatch (src/openpacho/backends.py:178-214).  With a recording fake in place
of the CUDA library, OpenPacho's own ``asarray``/``matmul``/``compile``/
``linalg.norm`` must reach the b200 entry points with the right shapes --
the same calls the compiled plans make (src/openpacho/_compiler.py:298-305).
"""

from __future__ import annotations

import ctypes as C
import threading
import weakref

import numpy as np
import pytest

openpacho = pytest.importorskip("openpacho", reason="OpenPacho not importable (set OPENPACHO_SRC)")

import pacho_b200  # noqa: E402
from pacho_b200 import _lib  # noqa: E402
from pacho_b200.backend import B200Backend  # noqa: E402


class RecordingLib:
    def __init__(self):
        self.calls = []
        self.next_ptr = 0x10000

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


@pytest.fixture
def fake_b200():
    b = object.__new__(B200Backend)
    b._lib = RecordingLib()
    b._ctx = C.c_void_p(1)
    b._lock = threading.RLock()
    b._closed = False
    b._buffers = weakref.WeakSet()
    b.device = "fake B200"
    b.ordinal = 0
    pacho_b200.register(openpacho)
    yield b
    b._closed = True
    pacho_b200.unregister(openpacho)


def _entries(b, name):
    return [args for n, args in b._lib.calls if n == name]


def test_register_accepts_b200_objects_and_delegates_other_names(fake_b200):
    assert openpacho.get_backend(fake_b200) is fake_b200
    assert openpacho.backends.get_backend("numpy").name == "numpy"
    with openpacho.use_backend(fake_b200) as selected:
        assert selected is fake_b200
        assert openpacho.asarray(np.ones(3, np.float32))._backend is fake_b200
    with pytest.raises(ValueError):
        openpacho.get_backend("b200", blas="cublas")


def test_register_is_idempotent_and_reversible():
    original = openpacho.backends.get_backend
    pacho_b200.register(openpacho)
    wrapped = openpacho.backends.get_backend
    pacho_b200.register(openpacho)
    assert openpacho.backends.get_backend is wrapped
    assert openpacho._array.get_backend is wrapped
    pacho_b200.unregister(openpacho)
    assert openpacho.backends.get_backend is original
    assert openpacho._array.get_backend is original


def test_b200_string_without_gpu_raises_openpachos_error():
    pacho_b200.register(openpacho)
    try:
        count = C.c_int(0)
        if _lib.load().pb_device_count(C.byref(count)) == 0 and count.value > 0:
            pytest.skip("a GPU is visible")
        pacho_b200.register.__globals__["_get_b200"].cache_clear()
        with pytest.raises(openpacho.BackendUnavailableError):
            openpacho.set_backend("b200")
    finally:
        pacho_b200.unregister(openpacho)


def test_openpacho_matmul_and_compiled_plan_reach_pb_gemm(fake_b200):
    a = openpacho.asarray(np.ones((8, 16, 512, 256), np.float32), backend=fake_b200)
    b = openpacho.asarray(np.ones((1, 16, 256, 384), np.float32), backend=fake_b200)
    c = openpacho.matmul(a, b, padding=True)  # b200 declines the padding hint
    assert c.shape == (8, 16, 512, 384) and c._backend is fake_b200
    compiled = openpacho.compile(lambda x, y: x @ y)
    c2 = compiled(a, b)
    assert c2.shape == c.shape
    gemms = _entries(fake_b200, "pb_gemm")
    assert len(gemms) == 2
    for args in gemms:
        assert args[3] == 2 and args[7:10] == (512, 384, 256)
        assert [args[5][i] for i in range(2)] == [16, 1] and [args[6][i] for i in range(2)] == [0, 1]


def test_openpacho_dot_gemv_and_norm_reach_their_entry_points(fake_b200):
    u = openpacho.asarray(np.ones(1000, np.float64), backend=fake_b200)
    A = openpacho.asarray(np.ones((30, 1000), np.float64), backend=fake_b200)
    openpacho.dot(u, u)
    A @ u
    openpacho.linalg.norm(A, axis=1)
    openpacho.linalg.norm(A)
    assert _entries(fake_b200, "pb_dot")[0][2] == _lib.PB_F64
    assert _entries(fake_b200, "pb_gemv")[0][3:5] == (30, 1000)
    norms = _entries(fake_b200, "pb_norm")
    assert [n[3:6] for n in norms] == [(30, 1000, 1), (1, 30000, 1)]


def test_openpacho_elementwise_reductions_and_views_reach_their_entry_points(fake_b200):
    """OpenPacho's own operators on b200 arrays (src/openpacho/_array.py:241-281,
    389-503): the backend sees pb_elementwise / pb_reduce / pb_gather calls with
    the reference's operation names and dtypes."""
    a = openpacho.asarray(np.ones((4, 3), np.float32), backend=fake_b200)
    b = openpacho.asarray(np.ones(3, np.float32), backend=fake_b200)
    c = a + b
    assert c.shape == (4, 3) and c._backend is fake_b200
    d = a * 2.0  # host scalar: uploaded as a 0-d array on b200
    assert d.dtype == np.float32
    mask = openpacho.isfinite(a)
    assert mask.dtype == np.bool_
    openpacho.where(mask, a, 0.0)
    a.astype(np.float64)
    openpacho.sum(a, axis=0)
    openpacho.mean(a)
    openpacho.amin(a, axis=1)
    openpacho.transpose(a)
    openpacho.diag(a)
    ops = [args[2] for name, args in fake_b200._lib.calls if name == "pb_elementwise"]
    names = {v: k for k, v in _lib.EW_OPS.items() if k != "divide"}
    assert [names[o] for o in ops] == ["add", "multiply", "isfinite", "where", "cast",
                                       "true_divide"]
    reduces = [args for name, args in fake_b200._lib.calls if name == "pb_reduce"]
    assert [(r[2], r[7]) for r in reduces] == [(_lib.PB_REDUCE_SUM, 0b01), (_lib.PB_REDUCE_SUM, 0b11),
                                               (_lib.PB_REDUCE_MIN, 0b10)]
    gathers = [args for name, args in fake_b200._lib.calls if name == "pb_gather"]
    assert [tuple(g[5][i] for i in range(g[4])) for g in gathers] == [(3, 4), (3,)]


def test_openpacho_compiled_residual_plan_on_b200(fake_b200):
    """A compiled solver step (b - A @ x, then its norm): the product has no
    other use, so the plan's residual step reaches the fused GEMV epilogue
    (src/openpacho/_compiler.py:157-176, 306-307, through create_lowering)."""
    A = openpacho.asarray(np.ones((64, 64), np.float64), backend=fake_b200)
    x = openpacho.asarray(np.ones(64, np.float64), backend=fake_b200)
    b = openpacho.asarray(np.ones(64, np.float64), backend=fake_b200)
    step = openpacho.compile(lambda A, x, b: openpacho.linalg.norm(b - A @ x))
    n = step(A, x, b)
    assert n.shape == ()
    called = [name for name, _ in fake_b200._lib.calls]
    assert "pb_gemv_residual" in called and "pb_norm" in called
    assert "pb_gemv" not in called
    (args,) = _entries(fake_b200, "pb_gemv_residual")
    assert args[2] == _lib.PB_F64 and args[3:5] == (64, 64)


def test_compiled_plans_with_the_b200_lowering_match_openpachos_numpy_backend():
    """OpenPacho's real compiler over the b200 lowering (host stand-in for the
    arithmetic): residual GEMV, elementwise groups with scalars and casts, and
    a reduction of an elementwise group give the NumPy backend's bits."""
    from host_b200 import HostB200

    host = HostB200()
    rng = np.random.default_rng(5)
    A = rng.standard_normal((48, 33)).astype(np.float32)
    x = rng.standard_normal(33).astype(np.float32)
    b = rng.standard_normal(48).astype(np.float32)
    programs = (
        lambda A, x, b: b - A @ x,
        lambda A, x, b: ((b * 2.0 - 1) / 3.0).astype(np.float64) + b,
        lambda A, x, b: openpacho.sum(b * b + 1.5, axis=0),
        lambda A, x, b: openpacho.where(b > 0, b, 0.0) - openpacho.sqrt(openpacho.absolute(b)),
        lambda A, x, b: (openpacho.linalg.norm(b - A @ x), openpacho.amax(A * 2.0, axis=1)),
    )
    pacho_b200.register(openpacho)
    try:
        for fn in programs:
            host.calls.clear()
            got = openpacho.compile(fn)(*(openpacho.asarray(v, backend=host) for v in (A, x, b)))
            want = openpacho.compile(fn)(*(openpacho.asarray(v, backend="numpy") for v in (A, x, b)))
            got = got if isinstance(got, tuple) else (got,)
            want = want if isinstance(want, tuple) else (want,)
            for g, w in zip(got, want):
                g, w = openpacho.asnumpy(g), openpacho.asnumpy(w)
                assert g.dtype == w.dtype and g.shape == w.shape
                np.testing.assert_array_equal(g, w)
        assert any(c[0] == "residual_matvec" for c in host.calls)
    finally:
        pacho_b200.unregister(openpacho)
