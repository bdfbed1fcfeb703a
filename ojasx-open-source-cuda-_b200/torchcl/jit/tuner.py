"""Launch-parameter heuristics — the reference's AutoTuner (torchcl/jit/tuner.py:18-117).

libojx sizes its own grids (persistent GEMMs use one CTA per SM; elementwise
kernels use a grid-stride loop over up to 16 CTAs per SM), so only the queries
callers of the reference make are kept (tests/test_jit.py:72-78): the 1-D
work-group size and the tile size, under the reference's contract (powers of two,
tile sizes in {4, 8, 16}), plus the device limits.
"""
from __future__ import annotations

from torchcl.runtime.context import get_device_info


class AutoTuner:
    def __init__(self) -> None:
        self._info: dict | None = None

    @property
    def info(self) -> dict:
        if self._info is None:
            self._info = get_device_info()
        return self._info

    def optimal_workgroup_1d(self, n: int) -> int:
        """Largest power of two <= min(256, n) (tuner.py:26-53)."""
        wg = 1
        target = min(256, self.info["max_work_group_size"], max(int(n), 1))
        while wg * 2 <= target:
            wg *= 2
        return wg

    def optimal_tile_size(self, M: int, N: int, K: int) -> int:
        return 16 if min(M, N, K) >= 32 else (8 if min(M, N, K) >= 16 else 4)

    def max_alloc_elements(self, dtype_bytes: int = 4) -> int:
        return (self.info["max_mem_alloc_size_mb"] * 1024 * 1024) // dtype_bytes

    def summary(self) -> str:
        i = self.info
        return "\n".join([f"Device: {i['name']}", f"Compute Units: {i['max_compute_units']}",
                          f"Shared memory per block: {i['local_mem_size_kb']} KB",
                          f"Global Memory: {i['global_mem_size_mb']} MB"])


_global_tuner: AutoTuner | None = None


def get_auto_tuner() -> AutoTuner:
    global _global_tuner
    if _global_tuner is None:
        _global_tuner = AutoTuner()
    return _global_tuner
