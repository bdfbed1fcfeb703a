"""Device memory — replaces torchcl/runtime/memory.py (CLBufferPool) with the
native caching cudaMalloc pool of libojx (ojx_malloc / ojx_free).

`CLBuffer` keeps the reference's fields (memory.py:27-58); `buffer` is the CUDA
device address as an int.  Pool semantics follow memory.py:61-203: size bins
(512 B minimum, powers of two to 64 MiB, 2 MiB multiples above), free returns the
block to its bin, an OOM evicts the cache and retries once, then MemoryError.
"""
from __future__ import annotations

import ctypes
import threading
import weakref
from typing import Any

import numpy as np
import torch

from torchcl import _lib as L
from torchcl.runtime import context as _ctx
from torchcl.runtime.context import _ensure_initialized, check_not_capturing, get_queue


def _next_power_of_two(n: int) -> int:
    """Capacity of the pool bin serving an n-byte request (memory.py:20-24)."""
    cap = ctypes.c_size_t()
    L.check(L.lib().ojx_pool_bin_size(max(int(n), 0), ctypes.byref(cap)))
    return cap.value


class CLBuffer:
    """A pool block: device address + slab metadata (memory.py:27-58)."""

    __slots__ = ("buffer", "nbytes", "capacity", "dtype", "shape", "_id", "is_pinned", "_freed",
                 "__weakref__")
    _counter = 0
    _lock = threading.RLock()  # reentrant: see CLBufferPool

    def __init__(self, buffer: int, nbytes: int, capacity: int, dtype=None, shape=None,
                 is_pinned: bool = False):
        self.buffer = buffer
        self.nbytes = nbytes
        self.capacity = capacity
        self.dtype = dtype
        self.shape = shape
        self.is_pinned = is_pinned
        self._freed = False
        with CLBuffer._lock:
            CLBuffer._counter += 1
            self._id = CLBuffer._counter

    @property
    def ptr(self) -> int:
        return self.buffer

    def __repr__(self) -> str:
        return (f"CLBuffer(id={self._id}, ptr=0x{self.buffer:x}, nbytes={self.nbytes}, "
                f"capacity={self.capacity}, dtype={self.dtype}, shape={self.shape})")


def _host_view(arr) -> tuple[int, int, Any]:
    """(address, nbytes, keepalive) of a contiguous host numpy array or torch tensor."""
    if isinstance(arr, torch.Tensor):
        t = arr.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        t = t.contiguous()
        return t.data_ptr(), t.numel() * t.element_size(), t
    a = np.ascontiguousarray(arr)
    return a.ctypes.data, a.nbytes, a


# ── graph capture bookkeeping ─────────────────────────────────────────────
# A captured graph replays launches on fixed device addresses.  While a capture is
# active every buffer allocated or handed to a launch is recorded; when it ends the
# graph pins those addresses, and freeing a pinned buffer is deferred until the
# last graph that uses it is destroyed, so a replay never writes into memory the
# pool has handed out again.  Frees requested during the capture are deferred too.
_cap_lock = threading.RLock()
_capture_sink: dict[int, CLBuffer] | None = None
_pins: dict[int, int] = {}
_deferred: dict[int, "CLBuffer"] = {}


def note_use(buf) -> None:
    """Record `buf` as used by the graph being captured (no-op otherwise)."""
    if _capture_sink is not None and isinstance(buf, CLBuffer):
        with _cap_lock:
            if _capture_sink is not None:
                _capture_sink[buf.buffer] = buf


def begin_capture() -> None:
    global _capture_sink
    with _cap_lock:
        if _capture_sink is not None:
            raise RuntimeError("a graph capture is already active")
        _capture_sink = {}
        _ctx._capture_active = True


def end_capture(keep: bool) -> list[int]:
    """Close the capture; pin its buffers if `keep`.  Returns the pinned addresses."""
    global _capture_sink
    with _cap_lock:
        sink, _capture_sink = _capture_sink or {}, None
        _ctx._capture_active = False
        addrs = sorted(sink) if keep else []
        for a in addrs:
            _pins[a] = _pins.get(a, 0) + 1
        pending = [a for a in list(_deferred) if a not in _pins]
    for a in pending:
        _really_free(a)
    return addrs


def release_pins(addrs) -> None:
    """A graph using `addrs` was destroyed: finish the frees it deferred."""
    ready = []
    with _cap_lock:
        for a in addrs:
            n = _pins.get(a, 0) - 1
            if n > 0:
                _pins[a] = n
                continue
            _pins.pop(a, None)
            if a in _deferred and _capture_sink is None:
                ready.append(a)
    for a in ready:
        _really_free(a)


def _really_free(addr: int) -> None:
    with _cap_lock:
        buf = _deferred.pop(addr, None)
    if buf is not None:
        L.check(L.lib().ojx_free(addr), "free")


class CLBufferPool:
    """Caching device allocator facade (memory.py:61-203)."""

    def __init__(self) -> None:
        self._active: dict[int, CLBuffer] = weakref.WeakValueDictionary()
        # Reentrant on purpose.  Device-tensor handles return their buffers through
        # weakref finalizers (torchcl.api), and a finalizer runs wherever a garbage
        # collection happens to start: possibly on this thread inside one of the
        # locked sections below (an insertion into _active allocates).  With a plain
        # Lock, the finalizer's free() would then wait forever for a lock its own
        # thread holds, a host-side stall with the GPU idle.
        self._lock = threading.RLock()

    def allocate(self, nbytes: int, dtype=None, shape=None, pin_memory: bool = False) -> CLBuffer:
        _ensure_initialized()
        if nbytes <= 0:
            nbytes = 64
        p = ctypes.c_void_p()
        cap = ctypes.c_size_t()
        L.check(L.lib().ojx_malloc(int(nbytes), ctypes.byref(p), ctypes.byref(cap)), "allocate")
        buf = CLBuffer(p.value, int(nbytes), cap.value, dtype, shape, is_pinned=pin_memory)
        with self._lock:
            self._active[buf._id] = buf
        note_use(buf)
        return buf

    def free(self, cl_buf: CLBuffer) -> None:
        if cl_buf is None or cl_buf._freed:
            return
        cl_buf._freed = True
        with self._lock:
            self._active.pop(cl_buf._id, None)
        with _cap_lock:
            if _capture_sink is not None or cl_buf.buffer in _pins:
                _deferred[cl_buf.buffer] = cl_buf  # a graph may still use it
                return
        L.check(L.lib().ojx_free(cl_buf.buffer), "free")

    def empty_cache(self) -> None:
        L.check(L.lib().ojx_empty_cache(), "empty_cache")

    def host_to_device(self, host_array, cl_buf: CLBuffer | None = None,
                       non_blocking: bool = False) -> CLBuffer:
        """Copy a host numpy array (or CPU torch tensor) into a (new) device buffer."""
        check_not_capturing("host_to_device")
        addr, nbytes, keep = _host_view(host_array)
        if cl_buf is None:
            dtype = keep.dtype
            cl_buf = self.allocate(nbytes, dtype, tuple(keep.shape))
        q = get_queue()
        L.check(L.lib().ojx_memcpy_h2d(cl_buf.buffer, addr, nbytes, q), "host_to_device")
        if not non_blocking:
            L.check(L.lib().ojx_stream_synchronize(q), "host_to_device sync")
        return cl_buf

    def device_to_host(self, cl_buf: CLBuffer, dtype=np.float32, shape=None) -> np.ndarray:
        """Blocking copy of a buffer into a new numpy array (memory.py:162-177)."""
        if shape is not None:
            out = np.empty(shape, dtype=dtype)
        else:
            out = np.empty(cl_buf.nbytes // np.dtype(dtype).itemsize, dtype=dtype)
        self.copy_to_host(cl_buf, out.ctypes.data, out.nbytes)
        return out

    def copy_to_host(self, cl_buf: CLBuffer, host_addr: int, nbytes: int) -> None:
        check_not_capturing("device_to_host")
        q = get_queue()
        L.check(L.lib().ojx_memcpy_d2h(host_addr, cl_buf.buffer, nbytes, q), "device_to_host")
        L.check(L.lib().ojx_stream_synchronize(q), "device_to_host sync")
        L.check(L.lib().ojx_poll_device_error(), "device error")

    def device_to_device(self, src: CLBuffer, dst: CLBuffer | None = None) -> CLBuffer:
        if dst is None:
            dst = self.allocate(src.nbytes, src.dtype, src.shape)
        note_use(src)
        note_use(dst)
        L.check(L.lib().ojx_memcpy_d2d(dst.buffer, src.buffer, src.nbytes, get_queue()), "d2d")
        return dst

    def zero_fill(self, cl_buf: CLBuffer) -> None:
        note_use(cl_buf)
        L.check(L.lib().ojx_memset(cl_buf.buffer, 0, cl_buf.nbytes, get_queue()), "zero_fill")

    def get_stats(self) -> dict[str, Any]:
        st = L.PoolStats()
        L.check(L.lib().ojx_pool_stats_get(ctypes.byref(st)))
        out = {name: int(getattr(st, name)) for name, _ in L.PoolStats._fields_}
        return out

    def active_count(self) -> int:
        with self._lock:
            return len(self._active)


_global_pool: CLBufferPool | None = None


def get_buffer_pool() -> CLBufferPool:
    global _global_pool
    if _global_pool is None:
        _global_pool = CLBufferPool()
    return _global_pool
