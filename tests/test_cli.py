"""The ``python -m pacho_b200`` command and ``devices("b200")`` (CPU parts).

Mirrors src/openpacho/cli.py:100-147: argument choices, exit status 2 with a
message when discovery fails, and OpenPacho's own ``devices`` learning the
``"b200"`` name through :func:`pacho_b200.register`.
"""

from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np
import pytest

import pacho_b200 as pb
from pacho_b200 import _lib, cli


def _gpu_visible() -> bool:
    n = C.c_int(0)
    return _lib.load().pb_device_count(C.byref(n)) == 0 and n.value > 0


def test_backend_choice_is_b200_only():
    with pytest.raises(SystemExit):
        cli.main(["benchmark", "--backend", "cuda"])
    with pytest.raises(SystemExit):
        cli.main(["devices", "--backend", "opencl"])
    with pytest.raises(ValueError):
        pb.devices("cuda")


def test_discovery_failure_exits_2_with_a_message(capsys):
    if _gpu_visible():
        pytest.skip("a GPU is visible")
    assert cli.main(["devices"]) == 2
    assert "b200 device discovery failed" in capsys.readouterr().err
    assert cli.main(["benchmark", "--size", "8"]) == 2


def test_benchmark_rejects_bad_arguments():
    with pytest.raises(ValueError):
        cli.benchmark(size=0)
    with pytest.raises(ValueError):
        cli.benchmark(dtype="float16")


def test_register_teaches_openpacho_devices_b200():
    reference_src = Path("/root/reference/src")
    if reference_src.exists() and str(reference_src) not in sys.path:
        sys.path.append(str(reference_src))
    openpacho = pytest.importorskip("openpacho")
    import openpacho.cli as ocli

    original = openpacho.backends.devices
    pb.register(openpacho)
    try:
        assert openpacho.backends.devices is not original
        assert ocli.devices is openpacho.backends.devices
        if not _gpu_visible():
            with pytest.raises(openpacho.BackendUnavailableError):
                openpacho.backends.devices("b200")
    finally:
        pb.unregister(openpacho)
    assert openpacho.backends.devices is original and ocli.devices is original


def test_ndarray_methods_route_to_the_backend():
    class Fake(pb.B200Backend):
        device = "fake"

        def __init__(self):  # no library, no device
            self.calls = []

        def validate_dtype(self, dtype):
            return np.dtype(dtype)

        def reduce(self, a, axes, keepdims, dtype, *, operation="sum"):
            self.calls.append(("reduce", axes, operation, np.dtype(dtype)))
            return object()

        def gather(self, a, shape, offset, strides):
            self.calls.append(("gather", tuple(shape), offset, tuple(strides)))
            return object()

        def elementwise(self, name, args, shape, dtype):
            self.calls.append(("elementwise", name))
            return object()

        def upload(self, host):
            return object()

    f = Fake()
    a = pb.ndarray._wrap(object(), (2, 3), np.float32, f)
    assert a.T.shape == (3, 2)
    a.transpose(1, 0)
    a.sum(axis=1)
    a.min()
    a.max(axis=0)
    a.mean()
    assert f.calls[:2] == [("gather", (3, 2), 0, (1, 3)), ("gather", (3, 2), 0, (1, 3))]
    assert [c[1:3] for c in f.calls if c[0] == "reduce"] == [((1,), "sum"), ((0, 1), "min"),
                                                             ((0,), "max"), ((0, 1), "sum")]
    assert f.calls[-1] == ("elementwise", np.true_divide.__name__)  # "divide" in NumPy 2
