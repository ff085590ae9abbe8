"""pacho_b200: B200 (sm_100a) backend for OpenPacho's linear-algebra hot path.

* :class:`B200Backend` -- OpenPacho's backend protocol (``matmul``, ``norm``,
  ``upload``/``download``/``empty``/``full``, ``synchronize``) over the C-ABI
  library ``libpacho_b200.so`` (hand-written CUDA for sm_100a).
* :func:`register` -- adds ``"b200"`` to an installed OpenPacho's dispatch.
* ``asarray``/``asnumpy``/``matmul``/``dot``/``linalg.norm``/``set_backend``/
  ``use_backend``, the elementwise ufuncs, ``where``, ``sum``/``mean``/
  ``amin``/``amax``, ``transpose``/``diag`` -- the same public API for
  environments without OpenPacho.
* :mod:`pacho_b200.distributed` -- sharded GEMM and norm across GPUs (NCCL).
* ``devices()`` and ``python -m pacho_b200 devices|benchmark`` -- discovery and
  the synchronized benchmark of OpenPacho's ``pacho`` command.
"""

from . import linalg
from .api import (
    absolute,
    add,
    amax,
    amin,
    array,
    asarray,
    asnumpy,
    cos,
    diag,
    divide,
    dot,
    empty,
    equal,
    exp,
    full,
    get_backend,
    greater,
    greater_equal,
    isfinite,
    less,
    less_equal,
    log,
    matmul,
    mean,
    multiply,
    ndarray,
    negative,
    not_equal,
    ones,
    ones_like,
    positive,
    power,
    reshape,
    set_backend,
    sin,
    sqrt,
    subtract,
    sum,
    synchronize,
    tanh,
    to_backend,
    transpose,
    true_divide,
    use_backend,
    where,
    zeros,
    zeros_like,
)
from .backend import B200Backend, DeviceBuffer
from .discovery import DeviceInfo, devices
from .exceptions import BackendMismatchError, BackendUnavailableError, UnsupportedDtypeError
from .register import register, unregister

__version__ = "0.1.0"

__all__ = [
    "B200Backend",
    "BackendMismatchError",
    "BackendUnavailableError",
    "DeviceBuffer",
    "DeviceInfo",
    "UnsupportedDtypeError",
    "array",
    "asarray",
    "asnumpy",
    "devices",
    "dot",
    "empty",
    "full",
    "get_backend",
    "linalg",
    "matmul",
    "ndarray",
    "ones",
    "register",
    "reshape",
    "set_backend",
    "synchronize",
    "to_backend",
    "unregister",
    "use_backend",
    "zeros",
]
