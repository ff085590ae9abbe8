"""``python -m pacho_b200`` runs OpenPacho's own ``pacho`` command with b200.

The command is OpenPacho's (src/openpacho/cli.py:99-147); this package only
registers b200 and lets the two ``--backend`` options accept it.  These CPU
tests run the real command (skipped without OpenPacho) with the host stand-in
in place of the GPU backend, so the benchmark's own validation and report
come out of OpenPacho's code.
"""

from __future__ import annotations

import argparse
import ctypes as C
import importlib
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import pacho_b200 as pb
from host_b200 import HostB200
from pacho_b200 import _lib, command

register_module = importlib.import_module("pacho_b200.register")

ROOT = Path(__file__).resolve().parent.parent


def _gpu_visible() -> bool:
    n = C.c_int(0)
    return _lib.load().pb_device_count(C.byref(n)) == 0 and n.value > 0


def test_command_without_openpacho_exits_2():
    env = {k: v for k, v in os.environ.items() if k not in ("OPENPACHO_SRC", "PYTHONPATH")}
    env["PYTHONPATH"] = str(ROOT / "open-pacho_b200")
    proc = subprocess.run([sys.executable, "-c", "import sys; sys.modules['openpacho'] = None; "
                           "from pacho_b200.command import main; raise SystemExit(main(['devices']))"],
                          capture_output=True, text=True, env=env, timeout=120)
    assert proc.returncode == 2
    assert "OpenPacho is not installed" in proc.stderr


def test_backend_option_accepts_b200_only_while_the_command_runs(openpacho):
    parser = argparse.ArgumentParser()
    with command._backend_choice_b200():
        parser.add_argument("--backend", choices=("opencl", "cuda"))
        parser.add_argument("--other", choices=("x",))
    assert parser.parse_args(["--backend", "b200"]).backend == "b200"
    with pytest.raises(SystemExit):
        parser.parse_args(["--other", "b200"])
    later = argparse.ArgumentParser()
    later.add_argument("--backend", choices=("opencl",))
    with pytest.raises(SystemExit):
        later.parse_args(["--backend", "b200"])


def test_pacho_benchmark_on_b200_is_openpachos_benchmark(openpacho, monkeypatch, capsys):
    host = HostB200()
    monkeypatch.setattr(register_module, "_get_b200", lambda device: host)
    try:
        rc = command.main(["benchmark", "--backend", "b200", "--size", "16", "--repeat", "2"], openpacho)
        report = json.loads(capsys.readouterr().out)
    finally:
        pb.unregister(openpacho)
    assert rc == 0
    assert report["backend"] == "b200" and report["device"] == "host stand-in"
    assert [c["operation"] for c in report["cases"]] == ["add", "matmul", "sum"]
    assert report["all_valid"]
    methods = {c[0] for c in host.calls}
    assert {"upload", "elementwise", "matmul", "reduce", "download"} <= methods


def test_pacho_devices_b200_without_a_gpu_exits_2(openpacho, capsys):
    if _gpu_visible():
        pytest.skip("a GPU is visible")
    try:
        assert command.main(["devices", "--backend", "b200"], openpacho) == 2
    finally:
        pb.unregister(openpacho)
    assert capsys.readouterr().err.startswith("pacho: ")


def test_register_teaches_openpacho_devices_b200(openpacho):
    import openpacho.cli as ocli

    original = openpacho.backends.devices
    pb.register(openpacho)
    try:
        assert openpacho.backends.devices is not original
        assert ocli.devices is openpacho.backends.devices
        assert ocli.get_backend is openpacho.backends.get_backend
        if not _gpu_visible():
            with pytest.raises(openpacho.BackendUnavailableError):
                openpacho.backends.devices("b200")
    finally:
        pb.unregister(openpacho)
    assert openpacho.backends.devices is original and ocli.devices is original
    assert ocli.get_backend is openpacho.backends.get_backend


def test_openpacho_array_methods_route_to_the_backend(openpacho):
    """OpenPacho's ndarray methods on a b200 array reach gather/reduce/
    elementwise (src/openpacho/_array.py:88-160, 389-456)."""
    host = HostB200()
    pb.register(openpacho)
    try:
        a = openpacho.asarray(np.arange(6, dtype=np.float32).reshape(2, 3), backend=host)
        assert a.T.shape == (3, 2)
        np.testing.assert_array_equal(openpacho.asnumpy(a.transpose(1, 0)), np.arange(6).reshape(2, 3).T)
        np.testing.assert_array_equal(openpacho.asnumpy(a.sum(axis=1)), [3, 12])
        assert openpacho.asnumpy(a.min()) == 0 and openpacho.asnumpy(a.mean()) == 2.5
    finally:
        pb.unregister(openpacho)
    kinds = [c[0] for c in host.calls]
    assert kinds.count("gather") == 2 and kinds.count("reduce") == 3
