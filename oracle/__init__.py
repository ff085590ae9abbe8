"""CPU oracle for the b200 linear-algebra path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and its ``--impl reference`` arm) may import this package, and only as
the checker or the timed reference; the product (``pacho_b200``) never does.

What it restates (the reference's NumPy backend, the parity oracle):
* ``numpy_backend.matmul`` -- ``NumpyBackend.matmul``
  (src/openpacho/backends.py:139-142): NumPy ``@`` through OpenBLAS
  (NumPy >=2.0,<3 per the reference's pyproject.toml; 2.3.5 with OpenBLAS
  0.3.30 here), NumPy's loop over broadcast batches;
* ``numpy_backend.norm`` -- the NumPy branch of ``norm_data``
  (src/openpacho/_norm.py:39-52): s = max|x|, sum((x/s)^2) in the input dtype
  (NumPy pairwise summation), s*sqrt(sum), Inf scale passed through, empty -> 0;
* ``exact`` -- independent exact references in the spirit of the reference's
  benchmarks/gemm_precision_oracle.py:27-93 (exact dyadic dot products),
  benchmarks/fp64_contraction_oracle.py:109-125 (Fraction binary64) and
  benchmarks/accuracy.py:61-66 (Decimal sqrt(sum x^2)).

Parity pin: ``tests/golden/make_golden.py`` imports the reference itself
(``openpacho`` on its NumPy backend) in the build container and stores its
inputs and outputs for the reference's own hot-path test cases in
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this oracle
against them bit for bit.
"""

from . import exact, numpy_backend, tolerance

__all__ = ["exact", "numpy_backend", "tolerance"]
