"""ctypes binding of libojx.so (include/ojx.h).

The shared library is built in-tree by ojasx-open-source-cuda-_b200/build.py into
torchcl/_lib/libojx.so.  There is no fallback: if the library is missing or no
sm_100 device is present, the first device call raises.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import threading

_LIB_DIR = pathlib.Path(__file__).resolve().parent / "_lib"
# OJX_DEBUG_BOUNDS=1 in the environment (read when the library is first loaded)
# selects the bounds-checking build: every TMA tile origin and epilogue store is
# checked on the device and reported through ojx_poll_device_error.
DEBUG_BOUNDS = os.environ.get("OJX_DEBUG_BOUNDS", "") not in ("", "0")
LIB_PATH = _LIB_DIR / ("libojx_debug.so" if DEBUG_BOUNDS else "libojx.so")

# status codes (include/ojx.h)
OJX_OK = 0
OJX_ERR_INVALID = 1
OJX_ERR_OOM = 2
OJX_ERR_CUDA = 3
OJX_ERR_TIMEOUT = 4
OJX_ERR_UNSUPPORTED = 5
OJX_ERR_NOT_INITIALIZED = 6
OJX_ERR_BOUNDS = 7

F32, BF16, F16 = 0, 1, 2
UNARY = {"relu": 1, "sigmoid": 2, "tanh": 3, "neg": 4, "abs": 5, "exp": 6, "log": 7,
         "sqrt": 8, "silu": 9, "gelu": 10, "square": 11}
BINARY = {"add": 1, "sub": 2, "mul": 3, "div": 4}
OPERAND_NONE, OPERAND_ROW, OPERAND_FULL = 0, 1, 2
FP32_AUTO, FP32_3XTF32, FP32_FFMA = 0, 1, 2
FLAG_FORCE_SIMT, FLAG_NO_SKINNY, FLAG_FORCE_SKINNY, FLAG_PAIR = 0x1, 0x2, 0x4, 0x8
FLAG_SKINNY_COUNTER = 0x10
ROUTES = {0: "none", 1: "tc_f16", 2: "tc_3xtf32", 3: "skinny", 4: "simt", 5: "flash_attn"}
ATTN_FLAG_COMPOSED = 0x1
ATTN_FLAG_ONE_QTILE, ATTN_FLAG_TWO_QTILE = 0x2, 0x4
MAX_UNARY = 8
MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class TimeoutError_(RuntimeError):
    """A bounded device-side wait expired (OJX_ERR_TIMEOUT)."""


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
        ("dtype_a", ctypes.c_int32), ("dtype_b", ctypes.c_int32),
        ("dtype_c", ctypes.c_int32), ("dtype_operand", ctypes.c_int32),
        ("trans_a", ctypes.c_int32), ("trans_b", ctypes.c_int32),
        ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64),
        ("ld_operand", ctypes.c_int64),
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p),
        ("operand", ctypes.c_void_p),
        ("operand_kind", ctypes.c_int32), ("binary_op", ctypes.c_int32),
        ("operand_is_lhs", ctypes.c_int32), ("n_unary", ctypes.c_int32),
        ("unary", ctypes.c_int32 * MAX_UNARY),
        ("fp32_mode", ctypes.c_int32), ("flags", ctypes.c_int32),
    ]


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256), ("device", ctypes.c_int32),
        ("cc_major", ctypes.c_int32), ("cc_minor", ctypes.c_int32),
        ("sm_count", ctypes.c_int32), ("total_mem_bytes", ctypes.c_int64),
        ("l2_bytes", ctypes.c_int64), ("max_smem_per_block", ctypes.c_int32),
        ("clock_khz", ctypes.c_int32),
    ]


class PoolStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "alloc_count", "reuse_count", "free_count", "active_bytes", "cached_bytes",
        "peak_bytes", "total_allocated_bytes", "active_buffers", "evictions")]


class GraphNode(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("grid", ctypes.c_int32 * 3),
                ("block", ctypes.c_int32 * 3), ("smem_bytes", ctypes.c_int32),
                ("name", ctypes.c_char * 128)]


NODE_TYPES = {0: "other", 1: "kernel", 2: "memset", 3: "memcpy"}

_P = ctypes.c_void_p
_SIGS = {
    "ojx_abi_version": ([], ctypes.c_int),
    "ojx_device_count": ([ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ojx_init": ([ctypes.c_int, ctypes.POINTER(DeviceInfo)], ctypes.c_int),
    "ojx_current_device": ([ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ojx_synchronize": ([], ctypes.c_int),
    "ojx_last_error": ([], ctypes.c_char_p),
    "ojx_poll_device_error": ([], ctypes.c_int),
    "ojx_debug_bounds_enabled": ([], ctypes.c_int),
    "ojx_set_wait_budget": ([ctypes.c_uint64], ctypes.c_int),
    "ojx_kernel_launch_count": ([], ctypes.c_uint64),
    "ojx_last_route": ([], ctypes.c_int),
    "ojx_malloc": ([ctypes.c_size_t, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "ojx_free": ([_P], ctypes.c_int),
    "ojx_empty_cache": ([], ctypes.c_int),
    "ojx_pool_stats_get": ([ctypes.POINTER(PoolStats)], ctypes.c_int),
    "ojx_pool_bin_size": ([ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "ojx_pool_debug_fail_next": ([ctypes.c_int64], ctypes.c_int),
    "ojx_memcpy_h2d": ([_P, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "ojx_memcpy_d2h": ([_P, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "ojx_memcpy_d2d": ([_P, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "ojx_memset": ([_P, ctypes.c_int, ctypes.c_size_t, _P], ctypes.c_int),
    "ojx_host_alloc": ([ctypes.c_size_t, ctypes.POINTER(_P)], ctypes.c_int),
    "ojx_host_free": ([_P], ctypes.c_int),
    "ojx_stream_create": ([ctypes.POINTER(_P)], ctypes.c_int),
    "ojx_stream_destroy": ([_P], ctypes.c_int),
    "ojx_stream_synchronize": ([_P], ctypes.c_int),
    "ojx_stream_wait_event": ([_P, _P], ctypes.c_int),
    "ojx_event_create": ([ctypes.POINTER(_P), ctypes.c_int], ctypes.c_int),
    "ojx_event_destroy": ([_P], ctypes.c_int),
    "ojx_event_record": ([_P, _P], ctypes.c_int),
    "ojx_event_query": ([_P, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ojx_event_synchronize": ([_P], ctypes.c_int),
    "ojx_event_elapsed_ms": ([_P, _P, ctypes.POINTER(ctypes.c_float)], ctypes.c_int),
    "ojx_gemm": ([ctypes.POINTER(GemmDesc), _P], ctypes.c_int),
    "ojx_elementwise": ([_P, ctypes.c_int32, _P, ctypes.c_int32, _P, ctypes.c_int32,
                         ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                         ctypes.c_int64, _P], ctypes.c_int),
    "ojx_transpose": ([_P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _P], ctypes.c_int),
    "ojx_fill": ([_P, ctypes.c_double, ctypes.c_int64, ctypes.c_int32, _P], ctypes.c_int),
    "ojx_cast": ([_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_int64, _P], ctypes.c_int),
    "ojx_gemm_batched": ([ctypes.POINTER(GemmDesc), ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                          ctypes.c_int64, ctypes.c_int64, _P], ctypes.c_int),
    "ojx_gemm_host_io": ([ctypes.POINTER(GemmDesc), _P, _P, ctypes.c_int64, _P], ctypes.c_int),
    "ojx_attention": ([_P, _P, _P, _P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_int32,
                       ctypes.c_int64, ctypes.c_int32, _P], ctypes.c_int),
    "ojx_sum_columns": ([_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                         ctypes.c_int64, _P], ctypes.c_int),
    "ojx_ipc_get_handle": ([_P, _P], ctypes.c_int),
    "ojx_ipc_open_handle": ([_P, ctypes.POINTER(_P)], ctypes.c_int),
    "ojx_ipc_close_handle": ([_P], ctypes.c_int),
    "ojx_gemm_allgather": ([ctypes.POINTER(GemmDesc), ctypes.POINTER(_P), ctypes.c_int32,
                            ctypes.c_int64, _P], ctypes.c_int),
    "ojx_gemm_skinny_noalloc": ([ctypes.POINTER(GemmDesc), _P], ctypes.c_int),
    "ojx_graph_capture_begin": ([_P], ctypes.c_int),
    "ojx_graph_capture_end": ([_P, ctypes.POINTER(_P)], ctypes.c_int),
    "ojx_graph_launch": ([_P, _P], ctypes.c_int),
    "ojx_graph_destroy": ([_P], ctypes.c_int),
    "ojx_graph_node_count": ([_P, ctypes.c_int, ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "ojx_graph_node_get": ([_P, ctypes.c_int32, ctypes.POINTER(GraphNode)], ctypes.c_int),
    "ojx_debug_silence_producer_once": ([], ctypes.c_int),
    "ojx_debug_silence_skinny_contributors_once": ([], ctypes.c_int),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libojx.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"libojx.so not found at {LIB_PATH}; build it with "
                        "`python ojasx-open-source-cuda-_b200/build.py`")
                L = ctypes.CDLL(str(LIB_PATH))
                for name, (args, res) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = L
    return _lib


def last_error() -> str:
    msg = lib().ojx_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str = "") -> None:
    """Map an ojx status to the reference's Python exception types."""
    if rc == OJX_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc == OJX_ERR_INVALID:
        raise ValueError(msg)
    if rc == OJX_ERR_OOM:
        raise MemoryError(msg)
    if rc == OJX_ERR_TIMEOUT:
        raise TimeoutError_(msg)
    raise RuntimeError(msg)


def exported_symbols() -> list[str]:
    return list(_SIGS)
