"""Drop-in for the reference's native packed-slab loader module.

Same functions, classes, argument meaning, return values and error messages as
the extension built by spark_runtime/native_packed_loader.py from
spark_runtime/native/native_packed_loader.cpp (pybind module at :325-359):

* ``read_into(fd, destination, size, offset) -> int`` (:26-68)
* ``copy_storage_to_tensors(storage, targets, offsets, non_blocking) -> int`` (:70-119,176-190)
* ``ExpertCopyPlan(offsets, sizes)`` with ``.count``, ``.copy_storage_to_tensors``,
  ``.copy_storage_to_tensors_cuda``, ``.read_into_and_copy``,
  ``.read_into_and_copy_cuda`` (:199-321)

A failed ``pread`` raises ``RuntimeError("pread failed: <strerror>")``, as the
reference's ``std::system_error`` does through pybind11.  The work is done by libdsv4moe.so (``dsv4_read_into``, ``dsv4_copy_slices``,
``dsv4_read_into_and_copy``); ctypes releases the GIL around every call, as
the reference's ``py::gil_scoped_release`` does.  Device targets get one
``cudaMemcpyAsync`` each on the current stream.  On B200 the bulk path is
``PackedExpertStore.upload_experts`` + ``ExpertArena.materialize`` (one H2D
copy of all blocks, then the device materializer); these per-tensor copies
are kept for compatibility.
"""

from __future__ import annotations

import ctypes
import errno
import os

import torch

from . import _lib
from ._lib import ERR_BOUNDS, ERR_IO, ERR_SHORT_READ, ERR_SIZE

_LL = ctypes.c_longlong


def load_native_packed_loader():
    """Counterpart of spark_runtime.native_packed_loader.load_native_packed_loader:
    returns the loader module (this one); the native library is prebuilt."""
    _lib.load()
    import sys

    return sys.modules[__name__]


def _check_cpu_u8(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cpu":
        raise RuntimeError(f"{name} must be a CPU tensor")
    if t.dtype != torch.uint8:
        raise RuntimeError(f"{name} must be uint8")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def read_into(fd: int, destination: torch.Tensor, size: int, offset: int) -> int:
    if fd < 0:
        raise RuntimeError("fd must be non-negative")
    if size < 0:
        raise RuntimeError("size must be non-negative")
    if offset < 0:
        raise RuntimeError("offset must be non-negative")
    _check_cpu_u8(destination, "destination")
    if destination.numel() < size:
        raise RuntimeError("destination tensor is too small")
    got = _LL(0)
    err = ctypes.c_int(0)
    rc = _lib.load().dsv4_read_into(int(fd), destination.data_ptr(), destination.numel(), int(size), int(offset),
                                    ctypes.byref(got), ctypes.byref(err))
    if rc == ERR_IO:
        raise RuntimeError(f"pread failed: {os.strerror(err.value or errno.EIO)}")
    _lib.check(rc, "read_into")
    return int(got.value)


def _copy(storage: torch.Tensor, targets, offsets, expected, cuda_required: bool, non_blocking: bool) -> int:
    _check_cpu_u8(storage, "storage")
    targets = list(targets)
    offsets = [int(o) for o in offsets]
    if len(targets) != len(offsets):
        raise RuntimeError("targets and offsets length mismatch")
    if expected is not None and len(targets) != len(expected):
        raise RuntimeError("targets and expected sizes length mismatch")
    if not targets:
        return 0
    to_device = bool(cuda_required or targets[0].is_cuda)
    for o, t in zip(offsets, targets):
        if o < 0:
            raise RuntimeError("offset must be non-negative")
        if cuda_required and not t.is_cuda:
            raise RuntimeError("CUDA memcpy target must be a CUDA tensor")
        if not t.is_contiguous():
            raise RuntimeError("target must be contiguous")
        if t.is_cuda != to_device:
            raise RuntimeError("targets must all be on the same kind of device")
    n = len(targets)
    ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in targets])
    nbytes = (_LL * n)(*[t.numel() * t.element_size() for t in targets])
    offs = (_LL * n)(*offsets)
    exp = (_LL * n)(*[int(e) for e in expected]) if expected is not None else None
    copied = _LL(0)
    stream = torch.cuda.current_stream(targets[0].device).cuda_stream if to_device else 0
    rc = _lib.load().dsv4_copy_slices(storage.data_ptr(), storage.numel(), ptrs, nbytes, offs, exp, n,
                                      1 if to_device else 0, stream, ctypes.byref(copied))
    _raise_copy(rc)
    if to_device and not non_blocking and not cuda_required:
        torch.cuda.current_stream(targets[0].device).synchronize()
    return int(copied.value)


def _raise_copy(rc: int) -> None:
    if rc == ERR_SIZE:
        raise RuntimeError("target size does not match expert copy plan")
    if rc == ERR_BOUNDS:
        raise RuntimeError("source slice exceeds storage tensor")
    _lib.check(rc, "copy_storage_to_tensors")


def copy_storage_to_tensors(storage: torch.Tensor, targets, offsets, non_blocking: bool) -> int:
    return _copy(storage, targets, offsets, None, False, non_blocking)


class ExpertCopyPlan:
    """Planned slice copies of one packed expert block (offsets and byte sizes of
    its tensors inside the block)."""

    def __init__(self, offsets, sizes):
        offsets = [int(o) for o in offsets]
        sizes = [int(s) for s in sizes]
        if len(offsets) != len(sizes):
            raise RuntimeError("offsets and sizes length mismatch")
        for o, s in zip(offsets, sizes):
            if o < 0:
                raise RuntimeError("copy-plan offset must be non-negative")
            if s < 0:
                raise RuntimeError("copy-plan size must be non-negative")
        self._offsets = offsets
        self._sizes = sizes

    @property
    def count(self) -> int:
        return len(self._offsets)

    def copy_storage_to_tensors(self, storage, targets, non_blocking: bool) -> int:
        return _copy(storage, targets, self._offsets, self._sizes, False, non_blocking)

    def copy_storage_to_tensors_cuda(self, storage, targets) -> int:
        return _copy(storage, targets, self._offsets, self._sizes, True, True)

    def _read_and_copy(self, fd, staging, size, offset, targets, cuda_required, non_blocking):
        if fd < 0:
            raise RuntimeError("fd must be non-negative")
        if size < 0:
            raise RuntimeError("size must be non-negative")
        if offset < 0:
            raise RuntimeError("offset must be non-negative")
        _check_cpu_u8(staging, "destination")
        if staging.numel() < size:
            raise RuntimeError("destination tensor is too small")
        targets = list(targets)
        if len(targets) != len(self._offsets):
            raise RuntimeError("targets and offsets length mismatch")
        to_device = bool(cuda_required or (targets and targets[0].is_cuda))
        for t in targets:
            if cuda_required and not t.is_cuda:
                raise RuntimeError("CUDA memcpy target must be a CUDA tensor")
            if not t.is_contiguous():
                raise RuntimeError("target must be contiguous")
        n = len(targets)
        ptrs = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in targets])
        nbytes = (_LL * max(n, 1))(*[t.numel() * t.element_size() for t in targets])
        offs = (_LL * max(n, 1))(*self._offsets)
        exp = (_LL * max(n, 1))(*self._sizes)
        rb, cb = _LL(0), _LL(0)
        rs, cs = ctypes.c_double(0.0), ctypes.c_double(0.0)
        err = ctypes.c_int(0)
        stream = torch.cuda.current_stream(targets[0].device).cuda_stream if (to_device and targets) else 0
        rc = _lib.load().dsv4_read_into_and_copy(int(fd), staging.data_ptr(), staging.numel(), int(size),
                                                 int(offset), ptrs, nbytes, offs, exp, n, 1 if to_device else 0,
                                                 stream, ctypes.byref(rb), ctypes.byref(cb), ctypes.byref(rs),
                                                 ctypes.byref(cs), ctypes.byref(err))
        if rc == ERR_IO:
            raise RuntimeError(f"pread failed: {os.strerror(err.value or errno.EIO)}")
        if rc == ERR_SHORT_READ:
            raise RuntimeError("short packed expert read")
        _raise_copy(rc)
        if to_device and not non_blocking and not cuda_required and targets:
            torch.cuda.current_stream(targets[0].device).synchronize()
        return int(rb.value), int(cb.value), float(rs.value), float(cs.value)

    def read_into_and_copy(self, fd, staging, size, offset, targets, non_blocking: bool):
        return self._read_and_copy(fd, staging, size, offset, targets, False, non_blocking)

    def read_into_and_copy_cuda(self, fd, staging, size, offset, targets):
        return self._read_and_copy(fd, staging, size, offset, targets, True, True)

