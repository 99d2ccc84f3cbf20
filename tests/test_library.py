"""The C-ABI library loads and exports every entry point include/dsv4moe.h declares;
its host-only loader functions work without a GPU."""

import ctypes
import os
import re
import tempfile

import pytest

from conftest import REPO

HEADER = REPO / "include" / "dsv4moe.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"DSV4_API\s+[\w\s\*]+?\b(dsv4_\w+)\s*\(", text)))


def test_header_declares_api():
    names = _declared()
    assert "dsv4_moe_forward" in names and "dsv4_materialize" in names and len(names) >= 15


def test_library_exports_every_declared_symbol():
    from spark_b200 import _lib

    lib = _lib.load()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib.EXPORTED) == set(_declared())
    assert lib.dsv4_version() == 1
    assert lib.dsv4_status_string(-5) == b"short packed expert read"


def test_read_into_short_and_errors():
    from spark_b200 import _lib

    lib = _lib.load()
    data = bytes(range(256)) * 4
    with tempfile.NamedTemporaryFile() as f:
        f.write(data)
        f.flush()
        fd = os.open(f.name, os.O_RDONLY)
        try:
            buf = ctypes.create_string_buffer(2048)
            got = ctypes.c_longlong(0)
            err = ctypes.c_int(0)
            assert lib.dsv4_read_into(fd, buf, 2048, 100, 10, ctypes.byref(got), ctypes.byref(err)) == 0
            assert got.value == 100 and buf.raw[:100] == data[10:110]
            # short count at EOF, not an error
            assert lib.dsv4_read_into(fd, buf, 2048, 2000, 1000, ctypes.byref(got), ctypes.byref(err)) == 0
            assert got.value == 24
            # negative offset / too small destination
            assert lib.dsv4_read_into(fd, buf, 2048, 10, -1, ctypes.byref(got), ctypes.byref(err)) == _lib.ERR_ARG
            assert lib.dsv4_read_into(fd, buf, 5, 10, 0, ctypes.byref(got), ctypes.byref(err)) == _lib.ERR_ARG
        finally:
            os.close(fd)
    # bad fd -> pread errno
    buf = ctypes.create_string_buffer(16)
    got = ctypes.c_longlong(0)
    err = ctypes.c_int(0)
    assert lib.dsv4_read_into(987654, buf, 16, 16, 0, ctypes.byref(got), ctypes.byref(err)) == _lib.ERR_IO
    assert err.value != 0


def test_check_maps_codes_to_reference_messages():
    from spark_b200 import _lib

    with pytest.raises(RuntimeError, match="short packed expert read"):
        _lib.check(_lib.ERR_SHORT_READ)
    with pytest.raises(RuntimeError, match="source slice exceeds storage tensor"):
        _lib.check(_lib.ERR_BOUNDS)
    _lib.check(_lib.OK)
