"""CUDA graphs of hot-path calls (pb_capture_begin/end, pb_graph_launch).

A replayed graph must give the bits an eager call gives on the same buffer
contents, read the buffers afresh each replay, refuse what cannot be captured
(allocation, synchronisation) without losing the context, keep a buffer that
grew after the capture alive until the graph is destroyed, and let the kernel
timer's events live inside the graph.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from pacho_b200 import _lib

pytestmark = pytest.mark.gpu

NONE = (C.c_int64 * 1)()


class Raw:
    def __init__(self, backend):
        self.b, self.lib, self.ctx = backend, backend._lib, backend._ctx

    def ok(self, status, what):
        assert status == _lib.PB_OK, f"{what}: {_lib.last_error()}"

    def put(self, host):
        buf = self.b.upload(np.ascontiguousarray(host))
        return buf

    def get(self, buf, shape, dtype):
        out = np.empty(shape, dtype)
        self.ok(self.lib.pb_d2h(self.ctx, 0, C.c_void_p(out.ctypes.data), C.c_void_p(buf.ptr),
                                out.nbytes), "d2h")
        return out

    def h2d(self, buf, host):
        host = np.ascontiguousarray(host)
        self.ok(self.lib.pb_h2d(self.ctx, 0, C.c_void_p(buf.ptr), C.c_void_p(host.ctypes.data),
                                host.nbytes, 1), "h2d")

    def gemm(self, code, M, N, K, A, B, Cbuf):
        self.ok(self.lib.pb_gemm(self.ctx, 0, code, 0, NONE, NONE, NONE, M, N, K, C.c_void_p(A.ptr),
                                 C.c_void_p(B.ptr), C.c_void_p(Cbuf.ptr)), "gemm")

    def dot(self, code, n, x, y, out):
        self.ok(self.lib.pb_dot(self.ctx, 0, code, n, C.c_void_p(x.ptr), C.c_void_p(y.ptr),
                                C.c_void_p(out.ptr)), "dot")

    def norm_rows(self, code, rows, cols, x, out):
        self.ok(self.lib.pb_norm(self.ctx, 0, code, rows, cols, 1, C.c_void_p(x.ptr),
                                 C.c_void_p(out.ptr)), "norm")


def _step_buffers(raw, rng, M, N, K, n):
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    A64 = rng.standard_normal((M, K))
    B64 = rng.standard_normal((K, N))
    x = rng.standard_normal(n).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    return [A, B, A64, B64, x, y]


def _step(raw, M, N, K, n, dev):
    dA, dB, dA64, dB64, dx, dy, dC, dC64, dd, dnr = dev
    raw.gemm(_lib.PB_F32, M, N, K, dA, dB, dC)
    raw.gemm(_lib.PB_F64, M, N, K, dA64, dB64, dC64)
    raw.dot(_lib.PB_F32, n, dx, dy, dd)
    raw.norm_rows(_lib.PB_F32, M, K, dA, dnr)


def _results(raw, M, N, dev):
    dC, dC64, dd, dnr = dev[6:]
    return (raw.get(dC, (M, N), np.float32), raw.get(dC64, (M, N), np.float64),
            raw.get(dd, (), np.float32), raw.get(dnr, (M,), np.float32))


@pytest.mark.parametrize("M,N,K,n", [(512, 384, 256, 1 << 20), (1000, 333, 77, 4097)])
def test_replay_matches_eager_and_reads_fresh_inputs(b200, M, N, K, n):
    raw = Raw(b200)
    rng = np.random.default_rng(M + N + K)
    hosts = _step_buffers(raw, rng, M, N, K, n)
    dev = [raw.put(h) for h in hosts]
    dev += [b200.empty((M, N), np.float32), b200.empty((M, N), np.float64),
            b200.empty((), np.float32), b200.empty((M,), np.float32)]
    _step(raw, M, N, K, n, dev)  # sizes the internal buffers
    first = _results(raw, M, N, dev)
    graph = b200.capture(lambda: _step(raw, M, N, K, n, dev))
    try:
        assert graph.launches >= 4
        graph.launch()
        again = _results(raw, M, N, dev)
        for a, b in zip(first, again):
            assert a.tobytes() == b.tobytes()
        # New contents in the same buffers: the replay must use them.
        for _ in range(2):
            new = _step_buffers(raw, rng, M, N, K, n)
            for d, h in zip(dev, new):
                raw.h2d(d, h)
            graph.launch()
            replayed = _results(raw, M, N, dev)
            _step(raw, M, N, K, n, dev)
            eager = _results(raw, M, N, dev)
            for a, b in zip(replayed, eager):
                assert a.tobytes() == b.tobytes()
            assert abs(float(eager[2]) - float(np.dot(new[4].astype(np.float64), new[5]))) < 1e-3 * n ** 0.5
    finally:
        graph.close()


def test_capture_refuses_allocation_and_sync_and_stays_usable(b200):
    raw = Raw(b200)
    lib, ctx = raw.lib, raw.ctx
    ptr = C.c_void_p()
    raw.ok(lib.pb_capture_begin(ctx, 0), "begin")
    assert lib.pb_capture_begin(ctx, 0) == _lib.PB_ERR_INVALID
    assert lib.pb_alloc(ctx, 0, 1024, C.byref(ptr)) == _lib.PB_ERR_UNSUPPORTED
    assert lib.pb_sync(ctx, 0) == _lib.PB_ERR_UNSUPPORTED
    assert lib.pb_ktimer_enable(ctx, 0, 1) == _lib.PB_ERR_UNSUPPORTED
    handle = C.c_void_p()
    raw.ok(lib.pb_capture_end(ctx, 0, C.byref(handle)), "end")
    raw.ok(lib.pb_graph_launch(ctx, 0, handle), "launch empty graph")
    raw.ok(lib.pb_graph_destroy(ctx, 0, handle), "destroy")
    assert lib.pb_capture_end(ctx, 0, C.byref(handle)) == _lib.PB_ERR_INVALID
    # The context still computes.
    x = raw.put(np.arange(1000, dtype=np.float32))
    out = b200.empty((), np.float32)
    raw.dot(_lib.PB_F32, 1000, x, x, out)
    exact = float(np.dot(np.arange(1000.0), np.arange(1000.0)))
    assert abs(float(raw.get(out, (), np.float32)) - exact) <= 1e-6 * exact


def test_a_call_that_would_grow_a_buffer_is_refused_during_capture(b200):
    raw = Raw(b200)
    M = N = K = 2048  # pre-split operands far above any earlier scratch
    A = raw.put(np.ones((M, K), np.float32))
    B = raw.put(np.ones((K, N), np.float32))
    Cb = b200.empty((M, N), np.float32)
    b200.release_cached_memory()  # drops the scratch buffer: the GEMM must grow it
    with pytest.raises(Exception, match="grow"):
        b200.capture(lambda: raw.gemm(_lib.PB_F32, M, N, K, A, B, Cb))
    raw.gemm(_lib.PB_F32, M, N, K, A, B, Cb)
    assert np.all(raw.get(Cb, (M, N), np.float32) == K)


def test_grown_buffers_live_until_the_last_graph_is_destroyed(b200):
    raw = Raw(b200)
    rng = np.random.default_rng(5)
    small = [rng.standard_normal((128, 64)).astype(np.float32),
             rng.standard_normal((64, 256)).astype(np.float32)]
    dA, dB = (raw.put(h) for h in small)
    dC = b200.empty((128, 256), np.float32)
    b200.release_cached_memory()
    raw.gemm(_lib.PB_F32, 128, 256, 64, dA, dB, dC)
    want = raw.get(dC, (128, 256), np.float32)
    graph = b200.capture(lambda: raw.gemm(_lib.PB_F32, 128, 256, 64, dA, dB, dC))
    # A large eager GEMM grows the scratch buffer; the small graph's one is kept.
    n = 3072
    bigA, bigB = raw.put(np.ones((n, n), np.float32)), raw.put(np.ones((n, n), np.float32))
    bigC = b200.empty((n, n), np.float32)
    raw.gemm(_lib.PB_F32, n, n, n, bigA, bigB, bigC)
    raw.h2d(dC, np.zeros((128, 256), np.float32))
    graph.launch()
    assert raw.get(dC, (128, 256), np.float32).tobytes() == want.tobytes()
    assert np.all(raw.get(bigC, (n, n), np.float32) == n)

    def used():
        r, u, s, f = (C.c_size_t() for _ in range(4))
        raw.ok(raw.lib.pb_memory_stats(raw.ctx, 0, C.byref(r), C.byref(u), C.byref(s), C.byref(f)),
               "stats")
        return u.value

    before = used()
    with pytest.raises(Exception, match="graphs"):
        b200.release_cached_memory()  # pb_trim is refused while a graph lives
    graph.close()
    b200.synchronize()
    assert used() < before
    b200.release_cached_memory()


def test_kernel_timer_events_inside_a_graph(b200):
    raw = Raw(b200)
    lib, ctx = raw.lib, raw.ctx
    M = N = K = 1024
    A = raw.put(np.ones((M, K), np.float32))
    B = raw.put(np.ones((K, N), np.float32))
    Cb = b200.empty((M, N), np.float32)
    raw.gemm(_lib.PB_F32, M, N, K, A, B, Cb)
    raw.ok(lib.pb_ktimer_enable(ctx, 0, 2), "ktimer")
    try:
        graph = b200.capture(lambda: raw.gemm(_lib.PB_F32, M, N, K, A, B, Cb))
        total, count = C.c_double(), C.c_uint64()
        with graph:
            for _ in range(3):
                graph.launch()
                raw.ok(lib.pb_ktimer_read(ctx, 0, C.byref(total), C.byref(count)), "read")
                assert count.value == 1
                assert 0.0 < total.value < 100.0
    finally:
        raw.ok(lib.pb_ktimer_enable(ctx, 0, 0), "ktimer off")
    assert np.all(raw.get(Cb, (M, N), np.float32) == K)
