"""Foundation result types (``src/flextensor/types.py:14-59``)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class GPUMemoryUsage:
    """Device memory owned by the offload runtime: ring slots + permanently resident tensors."""

    blocks_bytes: int
    unmapped_tensors_bytes: int
    total_bytes: int

    @property
    def blocks_mb(self) -> float:
        return self.blocks_bytes / (1024 * 1024)

    @property
    def unmapped_tensors_mb(self) -> float:
        return self.unmapped_tensors_bytes / (1024 * 1024)

    @property
    def total_mb(self) -> float:
        return self.total_bytes / (1024 * 1024)
