"""Install ``"b200"`` into an installed OpenPacho's backend dispatch.

OpenPacho hard-codes its backend names: ``get_backend`` accepts backend
objects only if they are a ``NumpyBackend`` or are named opencl/vulkan/cuda,
and strings only from that set (src/openpacho/backends.py:198-214).
``_array`` binds ``get_backend`` at import (src/openpacho/_array.py:11), as
do ``random`` (src/openpacho/random.py:18) and ``cli`` (src/openpacho/cli.py:15),
while ``set_backend`` and
``use_backend`` look the module global up at call time (backends.py:219,226).
So :func:`register` wraps ``get_backend`` and rebinds the wrapper in each of
those places.  The wrapper resolves ``"b200"`` (optionally ``device=``) and
``B200Backend`` objects and delegates everything else unchanged.
"""

from __future__ import annotations

from functools import lru_cache

from .backend import B200Backend

_MARK = "_pacho_b200_wrapped"
# Modules that bind get_backend by name at import: the array front end
# (src/openpacho/_array.py:11), random (src/openpacho/random.py:18) and the
# command line (src/openpacho/cli.py:15).
_BINDERS = ("_array", "random", "cli")


@lru_cache(maxsize=8)
def _get_b200(device):
    return B200Backend(device)


def _adopt_exceptions(theirs):
    """Make the errors this backend raises catchable as OpenPacho's own classes
    (``except openpacho.BackendUnavailableError`` and the dtype/mismatch
    errors), whatever the import order was: each class is replaced by one that
    derives from both this package's and OpenPacho's, and the raise sites look
    the class up at raise time."""
    import pacho_b200

    from . import exceptions as ours

    for name in ("BackendUnavailableError", "UnsupportedDtypeError", "BackendMismatchError"):
        mine, other = getattr(ours, name), getattr(theirs, name)
        if issubclass(mine, other):
            continue
        merged = type(name, (mine, other), {"__module__": ours.__name__, "__doc__": mine.__doc__})
        setattr(ours, name, merged)
        setattr(pacho_b200, name, merged)


def register(openpacho=None):
    """Make ``openpacho.set_backend("b200", device=...)`` and friends work.

    Idempotent.  Returns the OpenPacho module it patched."""
    if openpacho is None:
        import openpacho  # type: ignore[import-not-found]
    import importlib

    backends = importlib.import_module(openpacho.__name__ + ".backends")
    _adopt_exceptions(importlib.import_module(openpacho.__name__ + ".exceptions"))
    original = backends.get_backend
    if getattr(original, _MARK, False):
        return openpacho

    def get_backend(backend=None, *, device=None, blas=None, clblast_library=None):
        if isinstance(backend, B200Backend):
            if device is not None or blas is not None or clblast_library is not None:
                raise ValueError("device cannot accompany an existing backend")
            return backend
        if isinstance(backend, str) and backend == "b200":
            if blas is not None:
                raise ValueError("BLAS configuration requires backend='opencl' or 'cuda'")
            if clblast_library is not None:
                raise ValueError("clblast_library requires backend='opencl'")
            return _get_b200(None if device is None else str(device))
        return original(backend, device=device, blas=blas, clblast_library=clblast_library)

    setattr(get_backend, _MARK, True)
    get_backend.__wrapped__ = original
    get_backend.__doc__ = original.__doc__
    backends.get_backend = get_backend
    _wrap_devices(openpacho, backends)
    for name in _BINDERS:
        try:
            module = importlib.import_module(f"{openpacho.__name__}.{name}")
        except ImportError:
            continue
        if getattr(module, "get_backend", None) is original:
            module.get_backend = get_backend
    if getattr(openpacho, "get_backend", None) is original:
        openpacho.get_backend = get_backend
    return openpacho


def _wrap_devices(openpacho, backends):
    """``devices("b200")`` (src/openpacho/backends.py:50-60, bound by name in
    the package and its CLI) lists b200 devices as OpenPacho's DeviceInfo."""
    import importlib

    from .discovery import devices as b200_devices

    original = backends.devices

    def devices(backend="opencl"):
        if backend == "b200":
            return [backends.DeviceInfo(**vars(d)) for d in b200_devices("b200")]
        return original(backend)

    setattr(devices, _MARK, True)
    devices.__wrapped__ = original
    devices.__doc__ = original.__doc__
    backends.devices = devices
    for module in (openpacho, importlib.import_module(openpacho.__name__ + ".cli")):
        if getattr(module, "devices", None) is original:
            module.devices = devices


def _unwrap_devices(openpacho, backends):
    import importlib

    wrapped = backends.devices
    if not getattr(wrapped, _MARK, False):
        return
    backends.devices = wrapped.__wrapped__
    for module in (openpacho, importlib.import_module(openpacho.__name__ + ".cli")):
        if getattr(module, "devices", None) is wrapped:
            module.devices = wrapped.__wrapped__


def unregister(openpacho=None):
    """Undo :func:`register` (used by tests)."""
    if openpacho is None:
        import openpacho  # type: ignore[import-not-found]
    import importlib

    backends = importlib.import_module(openpacho.__name__ + ".backends")
    wrapped = backends.get_backend
    if not getattr(wrapped, _MARK, False):
        return
    original = wrapped.__wrapped__
    backends.get_backend = original
    for name in _BINDERS:
        try:
            module = importlib.import_module(f"{openpacho.__name__}.{name}")
        except ImportError:
            continue
        if getattr(module, "get_backend", None) is wrapped:
            module.get_backend = original
    if getattr(openpacho, "get_backend", None) is wrapped:
        openpacho.get_backend = original
    _unwrap_devices(openpacho, backends)
