"""Streams and events — replaces torchcl/runtime/stream.py (OpenCL queues and
markers) with CUDA streams/events through libojx.  Same classes and methods:
Stream(synchronize, wait_event, wait_stream), Event(record, wait, query,
synchronize, elapsed_time), the `stream` context manager, current_stream and
default_stream.
"""
from __future__ import annotations

import ctypes
from typing import Optional

from torchcl import _lib as L
from torchcl.runtime.context import _get_default_queue, _set_current_queue, get_queue, _ensure_initialized


class Event:
    """A marker in a stream (stream.py:32-71)."""

    def __init__(self, enable_timing: bool = True) -> None:
        _ensure_initialized()
        self.enable_timing = enable_timing
        e = ctypes.c_void_p()
        L.check(L.lib().ojx_event_create(ctypes.byref(e), int(enable_timing)), "Event")
        self._ev = e.value
        self._recorded = False

    def __del__(self):
        try:
            if getattr(self, "_ev", None):
                L.lib().ojx_event_destroy(self._ev)
        except Exception:
            pass

    def record(self, stream: Optional["Stream"] = None) -> None:
        q = stream.queue if stream is not None else get_queue()
        L.check(L.lib().ojx_event_record(self._ev, q), "Event.record")
        self._recorded = True

    def wait(self, stream: Optional["Stream"] = None) -> None:
        if not self._recorded:
            return
        q = stream.queue if stream is not None else get_queue()
        L.check(L.lib().ojx_stream_wait_event(q, self._ev), "Event.wait")

    def query(self) -> bool:
        if not self._recorded:
            return True
        done = ctypes.c_int()
        L.check(L.lib().ojx_event_query(self._ev, ctypes.byref(done)), "Event.query")
        return bool(done.value)

    def synchronize(self) -> None:
        if self._recorded:
            L.check(L.lib().ojx_event_synchronize(self._ev), "Event.synchronize")

    def elapsed_time(self, end_event: "Event") -> float:
        """Milliseconds between this event and end_event (both recorded)."""
        if not self._recorded or not end_event._recorded:
            return 0.0
        self.synchronize()
        end_event.synchronize()
        ms = ctypes.c_float()
        L.check(L.lib().ojx_event_elapsed_ms(self._ev, end_event._ev, ctypes.byref(ms)),
                "Event.elapsed_time")
        return float(ms.value)


class Stream:
    """An in-order CUDA stream (stream.py:74-99)."""

    def __init__(self, priority: int = 0, _handle: int | None = None, _owned: bool = True) -> None:
        _ensure_initialized()
        if _handle is None:
            s = ctypes.c_void_p()
            L.check(L.lib().ojx_stream_create(ctypes.byref(s)), "Stream")
            _handle = s.value
        self.queue = _handle
        self._owned = _owned and _handle is not None

    def __del__(self):
        try:
            if getattr(self, "_owned", False) and self.queue:
                L.lib().ojx_stream_destroy(self.queue)
        except Exception:
            pass

    def synchronize(self) -> None:
        L.check(L.lib().ojx_stream_synchronize(self.queue), "Stream.synchronize")

    def wait_event(self, event: Event) -> None:
        event.wait(self)

    def wait_stream(self, other_stream: "Stream") -> None:
        ev = Event(enable_timing=False)
        ev.record(other_stream)
        self.wait_event(ev)


class stream:
    """Context manager that makes `stream_obj` the current stream of this thread."""

    def __init__(self, stream_obj: Stream) -> None:
        self.stream_obj = stream_obj
        self.prev_queue = None

    def __enter__(self) -> Stream:
        self.prev_queue = get_queue()
        _set_current_queue(self.stream_obj.queue)
        return self.stream_obj

    def __exit__(self, exc_type, exc_val, exc_tb) -> None:
        _set_current_queue(self.prev_queue)


def current_stream() -> Stream:
    return Stream(_handle=get_queue(), _owned=False)


def default_stream() -> Stream:
    return Stream(_handle=_get_default_queue(), _owned=False)
