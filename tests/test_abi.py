"""The C-ABI library loads on a CPU machine and exports what the header declares."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "pacho_b200.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(pb_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from pacho_b200 import _lib

    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_prototypes_cover_the_header():
    from pacho_b200 import _lib

    assert set(_declared()) == set(_lib.PROTOTYPES) | {"pb_last_error"}


def test_header_compiles_as_c(tmp_path):
    import subprocess

    src = tmp_path / "t.c"
    src.write_text('#include "pacho_b200.h"\nint main(void){return pb_abi_version()==0;}\n')
    proc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only",
                           "-I", str(HEADER.parent), str(src)], capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr


def test_abi_version_and_argument_errors_without_a_gpu(lib):
    from pacho_b200 import _lib

    assert lib.pb_abi_version() == 1
    # Null context is rejected before any CUDA call.
    assert lib.pb_gemm(None, 0, 0, 0, None, None, None, 1, 1, 1, None, None, None) == _lib.PB_ERR_INVALID
    assert b"null context" in lib.pb_last_error()
    assert lib.pb_norm(None, 0, 0, 1, 1, 1, None, None) == _lib.PB_ERR_INVALID
    assert lib.pb_dot(None, 0, 0, 4, None, None, None) == _lib.PB_ERR_INVALID
    assert lib.pb_comm_unique_id(None) == _lib.PB_ERR_INVALID


def test_error_mapping_is_loud():
    from pacho_b200 import _lib
    from pacho_b200.exceptions import BackendUnavailableError, UnsupportedDtypeError

    with pytest.raises(BackendUnavailableError):
        _lib.check(_lib.PB_ERR_UNAVAILABLE)
    with pytest.raises(ValueError):
        _lib.check(_lib.PB_ERR_INVALID)
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.PB_ERR_UNSUPPORTED)
    with pytest.raises(_lib.B200Error):
        _lib.check(_lib.PB_ERR_DEVICE)
    with pytest.raises(UnsupportedDtypeError):
        _lib.dtype_code("int32")


def test_missing_library_raises_instead_of_falling_back(monkeypatch, tmp_path):
    from pacho_b200 import _lib
    from pacho_b200.exceptions import BackendUnavailableError

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("PACHO_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(BackendUnavailableError):
        _lib.load()


def test_no_device_is_reported(lib):
    """In a container without a GPU the backend refuses to start."""
    from pacho_b200 import _lib

    count = C.c_int(-1)
    status = lib.pb_device_count(C.byref(count))
    if status == _lib.PB_OK and count.value > 0:
        pytest.skip("a GPU is visible")
    assert status == _lib.PB_ERR_UNAVAILABLE and count.value == 0
    ctx = C.c_void_p()
    assert lib.pb_init(1, (C.c_int * 1)(0), C.byref(ctx)) == _lib.PB_ERR_UNAVAILABLE
