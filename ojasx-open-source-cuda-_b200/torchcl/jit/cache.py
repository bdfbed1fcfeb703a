"""Plan cache — the reference's KernelCache (torchcl/jit/cache.py:17-78).

The reference caches compiled OpenCL kernels per generated source.  libojx has no
runtime compiler (every kernel is built ahead of time for sm_100a), so what is
cached is the fusion *plan* — the op-code tuple a fused launch executes — under
the same keys, with the same LRU, hit/miss statistics and thread safety.
"""
from __future__ import annotations

import hashlib
import threading
from collections import OrderedDict
from typing import Any


class KernelCache:
    def __init__(self, max_size: int = 512) -> None:
        self._cache: OrderedDict[str, Any] = OrderedDict()
        self._max_size = max_size
        self._lock = threading.Lock()
        self._hits = 0
        self._misses = 0

    def get(self, key: str):
        with self._lock:
            if key in self._cache:
                self._cache.move_to_end(key)
                self._hits += 1
                return self._cache[key]
            self._misses += 1
            return None

    def put(self, key: str, plan) -> None:
        with self._lock:
            if key in self._cache:
                self._cache.move_to_end(key)
            elif len(self._cache) >= self._max_size:
                self._cache.popitem(last=False)
            self._cache[key] = plan

    def clear(self) -> None:
        with self._lock:
            self._cache.clear()
            self._hits = 0
            self._misses = 0

    def stats(self) -> dict:
        with self._lock:
            total = self._hits + self._misses
            return {"size": len(self._cache), "max_size": self._max_size, "hits": self._hits,
                    "misses": self._misses,
                    "hit_rate": f"{self._hits / total:.1%}" if total > 0 else "N/A"}

    @staticmethod
    def make_key(*parts) -> str:
        raw = ":".join(str(p) for p in parts)
        return hashlib.sha256(raw.encode()).hexdigest() if len(raw) > 128 else raw


_global_cache: KernelCache | None = None


def get_kernel_cache() -> KernelCache:
    global _global_cache
    if _global_cache is None:
        _global_cache = KernelCache()
    return _global_cache
