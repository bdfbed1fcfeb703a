"""KernelConfig of the reference (torchcl/liquid/cost_model.py:34-46)."""
from __future__ import annotations


class KernelConfig:
    def __init__(self, workgroup_size: int, tile_size: int = 1, strategy: str = "default",
                 precision: str = "float"):
        self.workgroup_size = workgroup_size
        self.tile_size = tile_size
        self.strategy = strategy
        self.precision = precision

    def to_tuple(self) -> tuple:
        return (self.workgroup_size, self.tile_size, self.strategy, self.precision)

    def __repr__(self) -> str:
        return (f"KernelConfig(wg={self.workgroup_size}, tile={self.tile_size}, "
                f"strat={self.strategy}, prec={self.precision})")
