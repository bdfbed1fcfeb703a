"""CUDA runtime context — replaces torchcl/runtime/context.py (OpenCL platform,
device, context and queue singletons) with the libojx C-ABI.

One device per process (`init_opencl(device_index)`, default: the current CUDA
device, else 0) and one library-owned non-blocking stream as the default queue.
A thread-local "current stream" mirrors the reference's thread-local current
queue (context.py:104-124).
"""
from __future__ import annotations

import ctypes
import os
import threading

from torchcl import _lib as L

_initialized = False
_device = None
_device_info: dict | None = None
_default_stream = None
_init_lock = threading.Lock()
_thread_local = threading.local()


def init_opencl(platform_index: int | None = None, device_index: int | None = None,
                device_type=None) -> None:
    """Initialise the runtime on one CUDA device (idempotent).

    The name and the first two arguments are those of the reference
    (context.py:26-100); `platform_index` is accepted and ignored (one backend).
    Raises RuntimeError when no sm_100 device is present — there is no CPU mode.
    """
    global _initialized, _device, _device_info, _default_stream
    if _initialized:
        return
    with _init_lock:
        if _initialized:
            return
        lib = L.lib()
        if device_index is None:
            env = os.environ.get("OJX_DEVICE", os.environ.get("LOCAL_RANK"))
            device_index = int(env) if env is not None else 0
        info = L.DeviceInfo()
        L.check(lib.ojx_init(int(device_index), ctypes.byref(info)), "ojx_init")
        s = ctypes.c_void_p()
        L.check(lib.ojx_stream_create(ctypes.byref(s)), "default stream")
        _default_stream = s.value
        _device = int(device_index)
        _device_info = _query_device_info(info)
        _initialized = True


init = init_opencl


def _ensure_initialized() -> None:
    if not _initialized:
        init_opencl()


def _query_device_info(info: "L.DeviceInfo") -> dict:
    # Keys of the reference's _query_device_info (context.py:169-186), filled from CUDA.
    return {
        "name": info.name.decode(),
        "vendor": "NVIDIA",
        "version": f"CUDA sm_{info.cc_major}{info.cc_minor}",
        "driver_version": "",
        "device_type": "GPU",
        "max_compute_units": int(info.sm_count),
        "max_clock_frequency_mhz": int(info.clock_khz) // 1000,
        "max_work_group_size": 1024,
        "max_work_item_sizes": [1024, 1024, 64],
        "global_mem_size_mb": int(info.total_mem_bytes) // (1024 * 1024),
        "local_mem_size_kb": int(info.max_smem_per_block) // 1024,
        "max_mem_alloc_size_mb": int(info.total_mem_bytes) // (1024 * 1024),
        "preferred_vector_width_float": 4,
        "image_support": False,
        "l2_cache_mb": int(info.l2_bytes) // (1024 * 1024),
        "device_index": int(info.device),
    }


def get_device_info() -> dict:
    _ensure_initialized()
    return dict(_device_info)


def get_device() -> int:
    _ensure_initialized()
    return _device


def get_context() -> int:
    """The CUDA device index (the context is the device's primary context)."""
    return get_device()


def get_queue() -> int | None:
    """The current stream of this thread (a cudaStream_t as int)."""
    _ensure_initialized()
    q = getattr(_thread_local, "current_queue", None)
    return q if q is not None else _default_stream


def _set_current_queue(q) -> None:
    _thread_local.current_queue = q


def _get_default_queue() -> int:
    _ensure_initialized()
    return _default_stream


# True while torchcl.jit.graph_runner.capture_graph records launches: nothing
# executes then, so waiting for results (synchronize, downloads) is an error.
_capture_active = False


def check_not_capturing(what: str) -> None:
    if _capture_active:
        raise RuntimeError(f"{what} is not allowed while a graph is being captured: upload inputs "
                           "before capture_graph() and read results after its `with` block")


def synchronize() -> None:
    """Block until all work on the current stream (and the default queue) finished."""
    _ensure_initialized()
    check_not_capturing("synchronize")
    lib = L.lib()
    q = get_queue()
    L.check(lib.ojx_stream_synchronize(q), "synchronize")
    if q != _default_stream:
        L.check(lib.ojx_stream_synchronize(_default_stream), "synchronize")
    L.check(lib.ojx_poll_device_error(), "device error")


def is_available() -> bool:
    try:
        n = ctypes.c_int(0)
        return L.lib().ojx_device_count(ctypes.byref(n)) == 0 and n.value > 0
    except Exception:
        return False
