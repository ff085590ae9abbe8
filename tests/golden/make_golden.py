"""Generate the golden fixtures by running the REFERENCE itself.

Run once in the build container, where the reference is importable:

    PYTHONPATH=/path/to/open-pacho/src python tests/golden/make_golden.py

It imports ``openpacho`` (the reference, NumPy backend -- its parity oracle,
src/openpacho/backends.py:82-150) and evaluates the reference's own hot-path
test cases from ``cases.py`` through the public API
(``openpacho.matmul``/``openpacho.linalg.norm``, asarray/asnumpy), and the
elementwise, cast, reduction and gather cases around that path through the
matching public functions.  For every
case it stores the SHA-256 of the inputs and the reference's outputs in
``golden.npz`` next to this file.  The GPU box never runs this script.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import cases  # noqa: E402


def main() -> int:
    import openpacho as p

    if p.get_backend().name != "numpy":
        raise SystemExit("expected the reference's default NumPy backend")
    out, meta = {}, {}

    def record_matmul(name, a, b):
        c = p.asnumpy(p.matmul(p.asarray(a), p.asarray(b)))
        out[f"{name}"] = c
        meta[name] = {"kind": "matmul", "inputs": cases.digest(a, b)}

    for gen in (cases.matmul_cases, cases.empty_cases, cases.batched_cases, cases.gemv_cases,
                cases.dot_cases, cases.signed_cases, cases.special_value_cases):
        for name, a, b in gen():
            record_matmul(name, a, b)
    name, a, b = cases.cancellation_case()
    record_matmul(name, a, b)

    for gen in (cases.norm_extreme_cases, cases.norm_special_cases, cases.norm_chunk_cases,
                cases.norm_distribution_cases):
        for name, x, axis, keepdims in gen():
            r = p.asnumpy(p.linalg.norm(p.asarray(x), axis=axis, keepdims=keepdims))
            out[name] = r
            meta[name] = {"kind": "norm", "inputs": cases.digest(x), "axis": axis,
                          "keepdims": keepdims}

    for name, kind, op, inputs, params in cases.around_cases():
        args = [p.asarray(a) for a in inputs]
        if kind == "ew":
            r = getattr(p, op)(*args)
        elif kind == "cast":
            r = args[0].astype(np.dtype(params["dtype"]))
        elif kind == "reduce":
            r = getattr(p, op)(args[0], axis=params["axis"])
        elif op == "transpose":
            r = p.transpose(args[0], params["axes"])
        else:
            r = p.diag(args[0], params["k"])
        out[name] = p.asnumpy(r)
        meta[name] = {"kind": kind, "op": op, "inputs": cases.digest(*inputs)}

    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden.json").write_text(json.dumps(
        {"reference": "openpacho " + getattr(p, "__version__", "?") + " (NumPy backend)",
         "numpy": np.__version__, "cases": meta}, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(out)} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
