"""Fusion plans of the elementwise path, built once per op chain.

The reference compiles one OpenCL program per generated kernel source and keeps
the kernel objects (torchcl/jit/cache.py:17-78); its tests only read the hit
counter, `get_kernel_cache().stats()["hits"]` (tests/test_jit.py:81-95,
tests/test_jit_integration.py:28-47).

Nothing is compiled at run time here.  Every chain runs on the one ahead-of-time
ojx_elementwise kernel, which takes the chain as an array of op codes, so the
thing worth keeping between calls is that array (building it validates every op
name and allocates a ctypes array).  A plan depends only on the chain itself
(binary op and unary op names): not on the element count, the buffers or the
dtypes.  The cache is therefore keyed by the chain tuple, and it holds at most
one entry per distinct chain a program fuses, a small and bounded set (the op
alphabet is fixed and a chain holds at most eight unary ops), so it never evicts.
"""
from __future__ import annotations

import threading
from typing import Callable, Hashable


class PlanCache:
    """chain -> plan, built on first use by the caller's `build(chain)`."""

    def __init__(self) -> None:
        self._plans: dict[Hashable, object] = {}
        self._build_lock = threading.Lock()
        self._hits = 0
        self._builds = 0

    def plan_for(self, chain: Hashable, build: Callable[[Hashable], object]) -> object:
        plan = self._plans.get(chain)
        if plan is None:
            # Builds are serialised so two threads never build the same chain twice;
            # lookups of chains already present take no lock.
            with self._build_lock:
                plan = self._plans.get(chain)
                if plan is None:
                    plan = build(chain)  # raises on an unknown op: nothing is stored
                    self._plans[chain] = plan
                    self._builds += 1
                    return plan
        self._hits += 1
        return plan

    def __contains__(self, chain: Hashable) -> bool:
        return chain in self._plans

    def __len__(self) -> int:
        return len(self._plans)

    def stats(self) -> dict:
        """hits: lookups answered from the cache; misses: plans built; size: chains held."""
        return {"hits": self._hits, "misses": self._builds, "size": len(self._plans)}

    def clear(self) -> None:
        with self._build_lock:
            self._plans = {}
            self._hits = self._builds = 0


_plans = PlanCache()


def get_kernel_cache() -> PlanCache:
    """The process-wide plan cache (the reference's accessor name)."""
    return _plans
