"""Record the backend calls OpenPacho's real front end makes on b200.

Run once in the build container, where the reference is importable:

    OPENPACHO_SRC=/path/to/open-pacho/src python tests/golden/make_frontend_trace.py

It registers b200 with OpenPacho (``pacho_b200.register``) and runs a set of
programs through OpenPacho's own public API -- ``asarray``, ``@``/``matmul``
(with ``padding=``), ``dot``, ``linalg.norm``, ``compile`` (which takes this
package's lowering: fused residual GEMVs, elementwise groups), ``astype``,
``where``, ``mean``/``sum``/``amax``, ``transpose``/``diag`` and the
reference's example conjugate-gradient solver (examples/solvers.py) -- on a
recording stand-in for the backend (tests/host_b200.py) whose arithmetic is
the NumPy-backend oracle.  For every protocol call it stores the method, its
arguments (operand buffers by id with shape and dtype, host scalars, axes,
strides ...) and the value of every buffer, into ``frontend_trace.json`` and
``frontend_trace.npz`` next to this file.  Each program is also run on
OpenPacho's own NumPy backend, whose results are stored beside the trace's.

The GPU machines do not have OpenPacho; tests/test_gpu_frontend_replay.py
replays every recorded call on the real B200 backend and checks its output,
and tests/test_frontend_trace.py checks on CPU that the recorded calls
reproduce the NumPy backend's results.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path[:0] = [str(ROOT / "open-pacho_b200"), str(ROOT), str(ROOT / "tests")]

from host_b200 import HostB200, HostBuffer  # noqa: E402


class TraceBuffer(HostBuffer):
    __slots__ = ("id",)


class TraceB200(HostB200):
    """The host stand-in, recording every protocol call and buffer value."""

    def __init__(self):
        super().__init__("trace")
        self.log = []
        self.values = {}
        self._next = 0
        self.program = None

    def _buffer(self, array):
        buf = TraceBuffer(array, self)
        buf.id = self._next
        self._next += 1
        self.values[buf.id] = buf.array.copy()
        return buf

    @staticmethod
    def _ref(a):
        if getattr(a, "_host_scalar", False):
            return {"scalar": np.asarray(a._data).item(), "dtype": np.dtype(a.dtype).name}
        return {"buf": a._data.id, "shape": list(a.shape), "dtype": np.dtype(a.dtype).name}

    def _record(self, method, out, **fields):
        entry = {"program": self.program, "method": method, **fields}
        if out is not None:
            entry["out"] = out.id
        self.log.append(entry)
        return out

    def upload(self, a):
        out = super().upload(a)
        return self._record("upload", out, shape=list(np.shape(a)), dtype=np.asarray(a).dtype.name)

    def full(self, shape, value, dtype):
        out = super().full(shape, value, dtype)
        return self._record("full", out, shape=list(shape), value=float(value), dtype=np.dtype(dtype).name)

    def empty(self, shape, dtype):
        out = super().empty(shape, dtype)
        return self._record("empty", out, shape=list(shape), dtype=np.dtype(dtype).name)

    def download(self, a):
        self._record("download", None, arg=self._ref(a))
        return super().download(a)

    def matmul(self, a, b, shape, dtype):
        out = super().matmul(a, b, shape, dtype)
        return self._record("matmul", out, args=[self._ref(a), self._ref(b)], shape=list(shape),
                            dtype=np.dtype(dtype).name)

    def norm(self, a, axes, keepdims, dtype):
        out = super().norm(a, axes, keepdims, dtype)
        return self._record("norm", out, args=[self._ref(a)], axes=[int(i) for i in axes],
                            keepdims=bool(keepdims), dtype=np.dtype(dtype).name)

    def elementwise(self, name, args, shape, dtype):
        out = super().elementwise(name, args, shape, dtype)
        return self._record("elementwise", out, name=name, args=[self._ref(a) for a in args],
                            shape=list(shape), dtype=np.dtype(dtype).name)

    def gather(self, a, shape, offset, strides):
        out = super().gather(a, shape, offset, strides)
        return self._record("gather", out, args=[self._ref(a)], shape=list(shape), offset=int(offset),
                            strides=[int(s) for s in strides])

    def reduce(self, a, axes, keepdims, dtype, *, operation="sum"):
        out = super().reduce(a, axes, keepdims, dtype, operation=operation)
        return self._record("reduce", out, args=[self._ref(a)], axes=[int(i) for i in axes],
                            keepdims=bool(keepdims), dtype=np.dtype(dtype).name, operation=operation)

    def residual_matvec(self, a, x, b):
        out = super().residual_matvec(a, x, b)
        return self._record("residual_matvec", out, args=[self._ref(a), self._ref(x), self._ref(b)])


def programs(p, solvers):
    """(name, inputs, function of the front-end module and the arrays)."""
    rng = np.random.default_rng(2024)
    f32, f64 = np.float32, np.float64
    n = 96
    q = rng.standard_normal((n, n))
    spd = q @ q.T / n + np.eye(n)
    yield ("batched_broadcast", (rng.standard_normal((2, 3, 64, 48)).astype(f32),
                                 rng.standard_normal((1, 3, 48, 40)).astype(f32)),
           lambda a, b: (p.matmul(a, b), p.matmul(a, b, padding=True)))
    yield ("gemv_dot_vecmat", (rng.uniform(-1, 1, (70, 130)).astype(f32), rng.uniform(-1, 1, 130).astype(f32),
                               rng.uniform(-1, 1, 70).astype(f32)),
           lambda A, x, y: (A @ x, p.dot(x, x), y @ A, p.dot(A, x)))
    yield ("mixed_dtype_matmul", (rng.standard_normal((33, 17)).astype(f32), rng.standard_normal((17, 9))),
           lambda a, b: (a @ b,))
    ext = (rng.standard_normal((6, 50, 7)) * 10.0 ** rng.uniform(-300, 300, (6, 50, 7)))
    yield ("norms", (ext.astype(f64), (ext * 1e-280).astype(f32)),
           lambda x, y: (p.linalg.norm(x), p.linalg.norm(x, axis=1), p.linalg.norm(x, axis=(0, 2), keepdims=True),
                         p.linalg.norm(x[0], ord="fro"), p.linalg.norm(y, axis=-1), p.linalg.norm(y)))
    yield ("compiled_residual", (spd, rng.standard_normal(n), rng.standard_normal(n)),
           lambda A, x, b: p.compile(lambda A, x, b: (b - A @ x, p.linalg.norm(b - A @ x)))(A, x, b))
    yield ("compiled_groups", (rng.standard_normal((40, 30)).astype(f32), rng.standard_normal(30).astype(f32)),
           lambda A, v: p.compile(lambda A, v: (p.sum(A * 2.0 - v, axis=1), (v / 3.0).astype(np.float64) + 1,
                                                p.amax(p.where(A > 0, A, 0.0), axis=0)))(A, v))
    yield ("views_casts_reductions", (rng.standard_normal((5, 8)).astype(f32),),
           lambda a: (p.transpose(a), p.diag(a), p.diag(a, 2), a.astype(np.float64), p.mean(a, axis=0),
                      p.sum(p.isfinite(a), dtype=np.float32), a.T @ a))
    A = spd.astype(f64)
    b = rng.standard_normal(n)
    yield ("conjugate_gradient", (A, b),
           lambda A, b: (solvers.conjugate_gradient(A, b, rtol=1e-10, maxiter=200).x,))


def main() -> int:
    src = os.environ.get("OPENPACHO_SRC")
    if src:
        sys.path.append(src)
    import openpacho as p

    import pacho_b200

    sys.path.append(str(Path(p.__file__).resolve().parents[2] / "examples"))
    import solvers

    pacho_b200.register(p)
    trace = TraceB200()
    finals, meta = {}, []
    try:
        for name, inputs, fn in programs(p, solvers):
            trace.program = name
            b200_in = [p.asarray(v, backend=trace) for v in inputs]
            got = fn(*b200_in)
            got = got if isinstance(got, tuple) else (got,)
            trace.program = None
            want = fn(*(p.asarray(v, backend="numpy") for v in inputs))
            want = want if isinstance(want, tuple) else (want,)
            outs = []
            for k, (g, w) in enumerate(zip(got, want)):
                w = p.asnumpy(w)
                finals[f"final/{name}/{k}"] = w
                outs.append({"buf": g._data.id, "shape": list(g.shape), "dtype": g.dtype.name})
            meta.append({"program": name, "outputs": outs})
    finally:
        pacho_b200.unregister(p)
    arrays = {f"b{k}": v for k, v in trace.values.items()}
    arrays.update(finals)
    np.savez_compressed(HERE / "frontend_trace.npz", **arrays)
    (HERE / "frontend_trace.json").write_text(json.dumps({"programs": meta, "calls": trace.log}, indent=0) + "\n")
    print(f"{len(trace.log)} calls in {len(meta)} programs, {len(arrays)} arrays")
    return 0


if __name__ == "__main__":
    sys.exit(main())
