"""Strategy protocol and result types (contract of ``src/flextensor/strategy/protocol.py:38-106``).

Pipeline model shared by every strategy:

* ``strategy_map[L]`` lists the tensors copied host->device *while trap L
  computes*; they all belong to one later trap ``transfer_to_compute_map[L]``.
* Each transferring label owns a GPU ring slot (``label_to_block_id``); a slot's
  size is the largest transfer assigned to it (``block_sizes``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol, runtime_checkable

from flextensor_b200.core.stats import LayerStatistics, TensorStatistics


class StrategyComputeError(Exception):
    """A strategy cannot produce a valid plan for these inputs (recoverable)."""


@dataclass
class BlockStrategyData:
    label_to_size_map: dict[str, int]
    """transfer label -> bytes it moves."""
    allocation_ordered: dict[int, list[str]]
    """block id -> transfer labels using that slot, in execution order."""
    block_sizes: dict[int, int] | list[int]
    """block id -> slot size in bytes (max over its labels)."""
    label_to_block_id: dict[str, int]
    transfer_to_compute_map: dict[str, str]


@dataclass
class StrategyResult:
    strategy_map: dict[str, list[TensorStatistics]]
    block_data: BlockStrategyData | None = None


@runtime_checkable
class Strategy(Protocol):
    """Anything with ``compute(layer_stats, memory_stats, max_gpu_mem_bytes)``."""

    def compute(
        self,
        layer_stats: list[LayerStatistics],
        memory_stats: dict[int, float] | None = None,
        max_gpu_mem_bytes: int | None = None,
    ) -> StrategyResult: ...
