"""Device discovery for the ``"b200"`` backend (``devices("b200")``).

Same record as OpenPacho's ``DeviceInfo`` (src/openpacho/backends.py:24-32)
and the same fields ``cuda_devices`` fills (src/openpacho/_cuda.py:68-94):
id, name, vendor, kind, fp64, memory_bytes, driver.  Only sm_100 devices
(B200-class) are listed; other GPUs are not b200 devices.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib
from . import exceptions as _exc


@dataclass(frozen=True)
class DeviceInfo:
    id: str
    name: str
    vendor: str
    kind: str
    fp64: bool
    memory_bytes: int
    driver: str


def devices(backend="b200"):
    """List the B200-class devices; ``backend`` must be ``"b200"``."""
    if backend != "b200":
        raise ValueError(f"pacho_b200 lists b200 devices only, not {backend!r}")
    lib = _lib.load()
    count = C.c_int(0)
    if lib.pb_device_count(C.byref(count)) != _lib.PB_OK:
        raise _exc.BackendUnavailableError(f"b200 device discovery failed: {_lib.last_error()}")
    version = C.c_int(0)
    _lib.check(lib.pb_driver_version(C.byref(version)), "pb_driver_version")
    found = []
    for i in range(count.value):
        name = C.create_string_buffer(256)
        total = C.c_size_t(0)
        sms, major, minor = C.c_int(), C.c_int(), C.c_int()
        _lib.check(lib.pb_device_info(i, name, 256, C.byref(total), C.byref(sms), C.byref(major),
                                      C.byref(minor)), "pb_device_info")
        if major.value != 10:
            continue
        found.append(DeviceInfo(str(i), name.value.decode(), "NVIDIA", "GPU", True, int(total.value),
                                str(version.value)))
    return found
