"""Device memory, streams, events and the current device of the ``cuda`` backend.

Everything here is a thin owner of handles returned by ``libmtorch_cuda.so``'s device runtime
(``mt_cuda_malloc`` / ``mt_cuda_library_stream`` / ``mt_cuda_event_*`` / ``mt_cuda_host_alloc``);
no other library provides device memory or streams to this package.

* ``DeviceBuffer`` is the device counterpart of the reference's ``Storage``
  (cpp/mtorch/core/tensor.h:60-63): a block of device bytes shared by every view of a tensor,
  returned to the library's caching allocator when the last view is collected.
* Each device has ONE library stream on which every kernel and copy of this package is issued,
  so buffers are reused in stream order without events.  ``current_stream()`` returns it.
* ``Event`` mirrors ``torch.cuda.Event(enable_timing=True)`` (record / synchronize /
  elapsed_time) for timing on that stream.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L

_current = [0]
_initialised: set = set()
_streams: dict = {}
capturing: set = set()  # devices with a graph capture open (graphs.Graphed)


def _ensure_device(idx: int) -> None:
    """Makes `idx` the current device of the calling thread (verifying it is an sm_100 part)."""
    if idx not in _initialised:
        lib = L.lib()
        if lib.mt_cuda_device_count() <= idx:
            raise RuntimeError(f"CUDA device {idx} requested but only {lib.mt_cuda_device_count()} visible")
        L.check(lib.mt_cuda_set_device(idx), "set_device")
        _initialised.add(idx)
        _current[0] = idx
    elif _current[0] != idx:
        L.check(L.lib().mt_cuda_set_device(idx), "set_device")
        _current[0] = idx


def set_device(idx) -> None:
    _ensure_device(int(getattr(idx, "index", idx) or 0))


def current_device() -> int:
    return _current[0]


class DeviceBuffer:
    """`nbytes` device bytes on device `device` from the library's caching allocator."""

    __slots__ = ("ptr", "nbytes", "device", "__weakref__")

    def __init__(self, nbytes: int, device: int):
        _ensure_device(device)
        p = C.c_void_p()
        nbytes = max(int(nbytes), 16)
        L.check(L.lib().mt_cuda_malloc(C.byref(p), nbytes), "device allocation")
        self.ptr, self.nbytes, self.device = p.value, nbytes, device

    def data_ptr(self) -> int:
        return self.ptr

    def numel(self) -> int:
        return self.nbytes

    def __del__(self):
        lib = L._LIB
        if lib is not None and self.ptr:
            lib.mt_cuda_free(self.ptr)
            self.ptr = None


def stream_ptr(idx: int):
    """The library stream of device `idx` (cudaStream_t as an integer)."""
    s = _streams.get(idx)
    if s is None:
        _ensure_device(idx)
        p = C.c_void_p()
        L.check(L.lib().mt_cuda_library_stream(idx, C.byref(p)), "library stream")
        s = _streams[idx] = p.value
    return s


class Stream:
    """Handle of a device's library stream (``cuda_stream`` is the raw cudaStream_t)."""

    def __init__(self, device: int = None):
        self.device = current_device() if device is None else int(device)
        self.cuda_stream = stream_ptr(self.device)

    def synchronize(self) -> None:
        L.check(L.lib().mt_cuda_synchronize(self.cuda_stream), "stream synchronize")


def current_stream(device=None) -> Stream:
    return Stream(device)


def synchronize(device=None) -> None:
    """Waits for all work on the device (every stream), then reports a device-side wait that
    expired inside a kernel since the last check."""
    L.check(L.lib().mt_cuda_synchronize(None), "synchronize")
    L.check(L.lib().mt_cuda_device_status(1), "device status")


class Event:
    """Timing event (the ``torch.cuda.Event(enable_timing=True)`` calls the benchmarks use)."""

    def __init__(self, enable_timing: bool = True):
        p = C.c_void_p()
        L.check(L.lib().mt_cuda_event_create(C.byref(p)), "event create")
        self.handle = p.value

    def record(self, stream=None) -> None:
        s = stream.cuda_stream if isinstance(stream, Stream) else (stream or stream_ptr(current_device()))
        L.check(L.lib().mt_cuda_event_record(self.handle, s), "event record")

    def synchronize(self) -> None:
        L.check(L.lib().mt_cuda_event_synchronize(self.handle), "event synchronize")

    def elapsed_time(self, end: "Event") -> float:
        ms = C.c_float()
        end.synchronize()
        L.check(L.lib().mt_cuda_event_elapsed_ms(self.handle, end.handle, C.byref(ms)), "event elapsed")
        return float(ms.value)

    def __del__(self):
        lib = L._LIB
        if lib is not None and getattr(self, "handle", None):
            lib.mt_cuda_event_destroy(self.handle)
            self.handle = None


class _PinnedOwner:
    __slots__ = ("ptr",)

    def __init__(self, ptr):
        self.ptr = ptr

    def __del__(self):
        lib = L._LIB
        if lib is not None and self.ptr:
            lib.mt_cuda_host_free(self.ptr)


def pinned_array(n: int, np_dtype) -> np.ndarray:
    """A numpy array of `n` elements over page-locked host memory (freed with the array)."""
    dt = np.dtype(np_dtype)
    p = C.c_void_p()
    L.check(L.lib().mt_cuda_host_alloc(C.byref(p), max(n, 1) * dt.itemsize), "pinned host allocation")
    raw = (C.c_uint8 * (max(n, 1) * dt.itemsize)).from_address(p.value)
    arr = np.frombuffer(raw, dtype=dt, count=max(n, 1))
    # keep the allocation alive exactly as long as the array: the ctypes buffer holds the owner
    raw._mt_owner = _PinnedOwner(p.value)
    return arr


def memory_stats(device: int = None) -> dict:
    d = current_device() if device is None else int(device)
    a, b = C.c_size_t(), C.c_size_t()
    L.check(L.lib().mt_cuda_memory_stats(d, C.byref(a), C.byref(b)), "memory stats")
    return {"allocated_bytes": a.value, "cached_bytes": b.value}


def empty_cache() -> None:
    L.check(L.lib().mt_cuda_empty_cache(), "empty_cache")
