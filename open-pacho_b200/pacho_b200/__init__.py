"""pacho_b200: B200 (sm_100a) backend for OpenPacho's linear-algebra hot path.

* :class:`B200Backend` -- OpenPacho's backend protocol (``matmul``, ``norm``,
  ``upload``/``download``/``empty``/``full``, ``synchronize``; ``elementwise``,
  ``gather``, ``reduce`` around the path; ``residual_matvec`` and
  ``create_lowering`` for compiled plans) over the C-ABI library
  ``libpacho_b200.so`` (hand-written CUDA for sm_100a).
* :func:`register` -- adds ``"b200"`` to an installed OpenPacho's dispatch, so
  ``openpacho.set_backend("b200")``, ``openpacho.asarray(x, backend="b200")``,
  ``@``, ``openpacho.linalg.norm``, ``openpacho.compile`` and the ``pacho``
  command (``python -m pacho_b200``) run on the B200.
* :mod:`pacho_b200.distributed` -- the sharded forms (batch split, row blocks
  with B broadcast, norm and DOT partials over NVLink) for one process per GPU.
* :func:`devices` -- the visible B200s as OpenPacho-style ``DeviceInfo``.
* :class:`DeviceArray` -- a typed view of a device buffer, returned by this
  package's own functions when they are not handed OpenPacho arrays.
"""

from .backend import B200Backend, DeviceArray, DeviceBuffer
from .discovery import DeviceInfo, devices
from .exceptions import BackendMismatchError, BackendUnavailableError, UnsupportedDtypeError
from .register import register, unregister

__version__ = "0.2.0"

__all__ = [
    "B200Backend",
    "BackendMismatchError",
    "BackendUnavailableError",
    "DeviceArray",
    "DeviceBuffer",
    "DeviceInfo",
    "UnsupportedDtypeError",
    "devices",
    "register",
    "unregister",
]
