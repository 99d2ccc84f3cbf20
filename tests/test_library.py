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


def test_peer_exchange_sizes_and_argument_checks():
    """Host-side checks of the peer-memory expert-parallel entry points (no GPU:
    every case returns before a CUDA call)."""
    from spark_b200 import _lib

    lib = _lib.load()
    H, k = 4096, 6
    rb = lib.dsv4_ep_row_bytes(H, k)
    for W, cap in ((2, 64), (8, 64), (8, 4096)):
        n = lib.dsv4_ep_exchange_bytes(H, k, W, cap)
        recv = (W * cap * rb + 255) // 256 * 256
        ret = (cap * k * H * 2 + 255) // 256 * 256
        assert n == 1024 + recv + ret
    # unsupported shapes / capacities
    assert lib.dsv4_ep_exchange_bytes(H, k, 9, 64) == -1          # more than 8 ranks
    assert lib.dsv4_ep_exchange_bytes(1000, k, 2, 64) == -1       # hidden not a multiple of 512
    assert lib.dsv4_ep_exchange_bytes(H, k, 2, 0) == -1           # no capacity
    assert lib.dsv4_ep_exchange_bytes(H, k, 2, 1 << 22) == -1     # return rows beyond the 24-bit index
    assert lib.dsv4_ep_p2p_dispatch_workspace_bytes(-1, 2) == -1
    assert lib.dsv4_ep_p2p_dispatch_workspace_bytes(64, 2) > 0
    p = ctypes.c_void_p()
    assert lib.dsv4_ep_exchange_alloc(0, 0, ctypes.byref(p)) == _lib.ERR_ARG
    assert lib.dsv4_ep_exchange_alloc(-1, 1024, ctypes.byref(p)) == _lib.ERR_ARG
    assert lib.dsv4_ipc_handle(None, None) == _lib.ERR_ARG
    assert lib.dsv4_ipc_open(0, None, ctypes.byref(p)) == _lib.ERR_ARG
    assert lib.dsv4_ep_exchange_free(None) == _lib.OK and lib.dsv4_ipc_close(None) == _lib.OK
    fake = ctypes.c_void_p(0x1000)
    ws = ctypes.c_void_p(0x2000)
    args = dict(x=fake, idx=fake, w=fake, T=4, H=H, k=k, E=256, W=2, rank=0, bases=fake, cap=4, epoch=1,
                ret=fake, ws=ws, wsb=1 << 20, st=None)

    def dispatch(**kw):
        a = dict(args, **kw)
        return lib.dsv4_ep_dispatch_p2p(a["x"], a["idx"], a["w"], a["T"], a["H"], a["k"], a["E"], a["W"],
                                        a["rank"], a["bases"], a["cap"], a["epoch"], a["ret"], a["ws"],
                                        a["wsb"], a["st"])

    assert dispatch(rank=2) == _lib.ERR_ARG              # rank outside the world
    assert dispatch(W=9) == _lib.ERR_ARG                 # more than 8 ranks
    assert dispatch(T=5) == _lib.ERR_ARG                 # more tokens than the exchange holds
    assert dispatch(E=255) == _lib.ERR_ARG               # experts do not divide over the ranks
    assert dispatch(bases=None) == _lib.ERR_ARG          # no peer table
    assert dispatch(wsb=16) == _lib.ERR_WORKSPACE        # workspace too small
    assert dispatch(x=None) == _lib.ERR_ARG              # tokens but no input
