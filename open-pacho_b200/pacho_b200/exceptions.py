"""Error types of the b200 backend.

They are OpenPacho's own classes (src/openpacho/exceptions.py:4-13) when
OpenPacho is importable, so ``except openpacho.UnsupportedDtypeError`` keeps
working after the backend is registered; otherwise classes with the same
names, bases and meaning.
"""

try:  # pragma: no cover - depends on the environment
    from openpacho.exceptions import (  # type: ignore[import-not-found]
        BackendMismatchError,
        BackendUnavailableError,
        UnsupportedDtypeError,
    )
except ImportError:

    class BackendUnavailableError(RuntimeError):
        """The requested runtime or device cannot be used."""

    class UnsupportedDtypeError(TypeError):
        """A dtype is outside the supported set or the device's capabilities."""

    class BackendMismatchError(ValueError):
        """An operation combines arrays from different backends/contexts."""


__all__ = ["BackendMismatchError", "BackendUnavailableError", "UnsupportedDtypeError"]
