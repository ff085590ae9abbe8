"""Compiled-plan lowering for the b200 backend.

OpenPacho's compiler asks a backend once, when it prepares a plan, for a
lowering object (``create_lowering``, src/openpacho/_lowering.py:224-231) and
then hands it three kinds of step (src/openpacho/_compiler.py:157-220,
277-307):

* **residual GEMV** -- ``b - A @ x`` where the product has no other use: if
  :meth:`B200Lowering.can_residual_matvec` accepts it, the plan calls
  ``backend.residual_matvec(A, x, b)``, which here is one GEMV launch with the
  subtraction in its epilogue (``pb_gemv_residual``): the product never goes
  to HBM, and the result is bit-identical to the eager product followed by
  the elementwise subtract (the product is rounded to the dtype first,
  src/openpacho/_gemv.py:1-6).
* **elementwise groups** (``prepare_fused``/``run_fused``) and
* **reductions of an elementwise group** (``prepare_map_reduce``/
  ``run_map_reduce``): evaluated operation by operation on the b200
  elementwise and reduction kernels, each operation rounding to its own
  dtype with its inputs cast to the resolved dtypes first -- exactly the
  steps an unlowered plan takes (src/openpacho/_compiler.py:282-296).

Prepared payloads hold only the group's structure (operation names, input
positions, dtypes, shapes), never arrays or bound scalar values, as the
lowering seam requires (src/openpacho/_lowering.py:1-7).
"""

from __future__ import annotations

import numpy as np

from .backend import DeviceArray


class _Scalar:
    """A host scalar operand for ``B200Backend.elementwise`` (uploaded by the
    backend as a one-element array): the attributes the protocol reads."""

    _host_scalar = True
    shape = ()
    ndim = 0

    def __init__(self, value, dtype):
        self.dtype = np.dtype(dtype)
        self._data = np.asarray(value, dtype=self.dtype)[()]


class _Program:
    """An elementwise group in evaluation order.

    ``steps[i] = (op, refs, resolved, shape, dtype)``: ``refs`` name each input
    as ``("leaf", j)`` (the j-th plan argument) or ``("step", k)`` (an earlier
    step's result)."""

    def __init__(self, group, leaves):
        position = {id(leaf): ("leaf", j) for j, leaf in enumerate(leaves)}
        self.steps = []
        for k, node in enumerate(group):
            refs = tuple(position[id(child)] for child in node.inputs)
            self.steps.append((node.op, refs, tuple(np.dtype(t) for t in node.resolved),
                               tuple(node.shape), np.dtype(node.dtype)))
            position[id(node)] = ("step", k)

    def run(self, backend, operands):
        """The last step's value as a device array (operands in leaf order)."""
        results = []
        for op, refs, resolved, shape, dtype in self.steps:
            args = []
            for (kind, index), want in zip(refs, resolved):
                value = operands[index] if kind == "leaf" else results[index]
                args.append(_convert(backend, value, want))
            data = backend.elementwise(op, args, shape, dtype)
            results.append(DeviceArray(backend, data, shape, dtype))
        return results[-1]


def _convert(backend, value, dtype):
    """``value`` in ``dtype``: host scalars re-typed, arrays cast on the GPU."""
    if getattr(value, "_host_scalar", False):
        return value if value.dtype == dtype else _Scalar(value._data, dtype)
    if np.dtype(value.dtype) == dtype:
        return value
    data = backend.elementwise("cast", [value], value.shape, dtype)
    return DeviceArray(backend, data, value.shape, dtype)


class B200Lowering:
    """The object ``B200Backend.create_lowering()`` returns."""

    def __init__(self, backend):
        self.backend = backend

    # -- residual GEMV -------------------------------------------------------
    def can_residual_matvec(self, matrix, vector, rhs, node):
        """A 2-D matrix, two vectors and one float dtype throughout (the
        conditions of src/openpacho/_lowering.py:20-30)."""
        product = node.inputs[1]
        dtype = np.dtype(node.dtype)
        return (
            matrix.ndim == 2
            and vector.ndim == 1
            and rhs.ndim == 1
            and tuple(rhs.shape) == tuple(product.shape) == tuple(node.shape)
            and dtype.kind == "f"
            and dtype == matrix.dtype == vector.dtype == rhs.dtype == product.dtype
        )

    # -- reductions ------------------------------------------------------------
    def can_reduce_materialized(self, node):
        """Reductions of stored arrays stay plain ``backend.reduce`` steps."""
        return False

    # -- elementwise groups --------------------------------------------------
    def prepare_fused(self, node, group, leaves):
        return tuple(leaves), _Program(group, leaves)

    def run_fused(self, node, payload, arguments, operands):
        return payload.run(self.backend, operands)._data

    def prepare_map_reduce(self, node, group, leaves):
        return tuple(leaves), _Program(group, leaves)

    def run_map_reduce(self, node, payload, arguments, operands):
        mapped = payload.run(self.backend, operands)
        options = {"operation": node.attrs["operation"]} if "operation" in node.attrs else {}
        return self.backend.reduce(mapped, node.attrs["axes"], node.attrs["keepdims"], node.dtype,
                                   **options)
