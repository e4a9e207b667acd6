"""Shared planner helpers: transfer windows, maps, block data, scoring.

``transfer_to_compute_map`` and the evaluation formulas follow
``src/flextensor/strategy/utils.py:170-193`` and
``src/flextensor/strategy/evaluation.py:22-195``:

* peak GPU bytes = sum of slot sizes + (model bytes - offloaded bytes);
* overhead = sum over traps of max(0, transfer_ms - window_ms) / total compute ms,
  where the window of a transfer issued at trap i for trap j spans traps i..j-1;
* a violation is two adjacent transferring labels sharing a slot.
"""

from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass

from flextensor_b200.core.stats import LayerStatistics, TensorStatistics
from flextensor_b200.planner.blocks import (
    MemoryBlockPlanner,
    OptimizedRoundRobinAssignment,
    StrictRoundRobinAssignment,
    allocation_from_assignment,
)
from flextensor_b200.planner.interpolator import MemoryTransferInterpolator
from flextensor_b200.planner.protocol import BlockStrategyData, StrategyComputeError, StrategyResult

MB = 1024 * 1024


def validate_memory_params(scale: float) -> None:
    if not (isinstance(scale, (int, float)) and scale > 0 and math.isfinite(scale)):
        raise ValueError(f"scale must be a positive finite number, got {scale!r}")


def compute_label_to_size_map(
    layer_stats: list[LayerStatistics], strategy_map: dict[str, list[TensorStatistics]]
) -> OrderedDict[str, int]:
    out: OrderedDict[str, int] = OrderedDict()
    for layer in layer_stats:
        size = sum(t.size_bytes for t in strategy_map.get(layer.label, ()))
        if size > 0:
            out[layer.label] = size
    return out


def calculate_transfer_to_compute_map(
    layer_stats: list[LayerStatistics], strategy_map: dict[str, list[TensorStatistics]]
) -> dict[str, str]:
    owner = {t.tensor_id: layer.label for layer in layer_stats for t in layer.tensors}
    return {label: owner[ts[0].tensor_id] for label, ts in strategy_map.items() if ts}


def reverse_transfer_to_compute_map(t2c: dict[str, str]) -> dict[str, str]:
    out: dict[str, str] = {}
    for transfer, compute in t2c.items():
        if compute in out:
            raise ValueError(f"Compute label '{compute}' mapped from both '{out[compute]}' and '{transfer}'")
        out[compute] = transfer
    return out


def interpolator_for(
    layer_stats: list[LayerStatistics], memory_stats: dict[int, float] | None
) -> MemoryTransferInterpolator | None:
    if memory_stats:
        return MemoryTransferInterpolator(memory_stats)
    from flextensor_b200.core.stats import extract_memory_transfers_from_layer_stats

    pts = extract_memory_transfers_from_layer_stats(layer_stats)
    return MemoryTransferInterpolator(pts) if pts else None


def transfer_ms(interp: MemoryTransferInterpolator | None, tensors: list[TensorStatistics]) -> float:
    nbytes = sum(t.size_bytes for t in tensors)
    if nbytes <= 0:
        return 0.0
    if interp is not None:
        return interp.bytes_to_duration(nbytes)
    return sum(t.load_time_ms for t in tensors)


def byte_budget(interp: MemoryTransferInterpolator | None, window_ms: float, tensors: list[TensorStatistics]) -> float:
    """Bytes that can move inside ``window_ms`` (measured per-tensor rates if no interpolator)."""
    if window_ms <= 0:
        return 0.0
    if interp is not None:
        return interp.duration_to_bytes(window_ms)
    tot_b = sum(t.size_bytes for t in tensors)
    tot_ms = sum(t.load_time_ms for t in tensors)
    if tot_b <= 0 or tot_ms <= 0:
        return float("inf")
    return window_ms * tot_b / tot_ms


def eligible(tensors: list[TensorStatistics], threshold_mb: float) -> list[TensorStatistics]:
    return [t for t in tensors if t.size_bytes > threshold_mb * MB]


def build_block_data(
    strategy_map: dict[str, list[TensorStatistics]],
    layer_stats: list[LayerStatistics],
    n_blocks: int | None,
    assignment=None,
) -> BlockStrategyData | None:
    """Slots for every transferring label; ``n_blocks`` 0/None disables block planning."""
    if not n_blocks:
        return None
    sizes = compute_label_to_size_map(layer_stats, strategy_map)
    if not sizes:
        return BlockStrategyData({}, {}, {}, {}, {})
    order = list(sizes)
    t2c = calculate_transfer_to_compute_map(layer_stats, strategy_map)
    pos = {l.label: i for i, l in enumerate(layer_stats)}
    cyclic = any(pos[t2c[t]] <= pos[t] for t in order if t in t2c and t2c[t] in pos)  # schedule wraps
    if assignment is None:
        planner = MemoryBlockPlanner(sizes, cyclic=cyclic)
        alloc = planner.optimize_block_distribution(max(planner.find_minimum_blocks_sequential(), n_blocks))
        where = {l: b for b, ls in alloc.items() for l in ls}
    elif isinstance(assignment, StrictRoundRobinAssignment):
        where = assignment.assign(sizes, n_blocks)
    else:
        where = assignment.assign(sizes, n_blocks)
    alloc = allocation_from_assignment(order, where)
    block_sizes = {b: max(sizes[l] for l in ls) for b, ls in alloc.items()}
    return BlockStrategyData(
        label_to_size_map=dict(sizes),
        allocation_ordered=alloc,
        block_sizes=block_sizes,
        label_to_block_id={l: where[l] for l in order},
        transfer_to_compute_map=t2c,
    )


# --------------------------------------------------------------------------- scoring


@dataclass
class StrategyScore:
    strategy_name: str
    peak_memory_bytes: int
    estimated_overhead: float
    consecutive_violations: int
    is_valid: bool

    def __lt__(self, other: "StrategyScore") -> bool:
        if self.is_valid != other.is_valid:
            return self.is_valid
        if not self.is_valid:
            return self.peak_memory_bytes < other.peak_memory_bytes
        if not math.isclose(self.estimated_overhead, other.estimated_overhead, rel_tol=1e-9, abs_tol=1e-12):
            return self.estimated_overhead < other.estimated_overhead
        return self.peak_memory_bytes < other.peak_memory_bytes


def peak_memory(result: StrategyResult, layer_stats: list[LayerStatistics]) -> int:
    blocks = 0
    if result.block_data is not None:
        bs = result.block_data.block_sizes
        blocks = sum(bs.values()) if isinstance(bs, dict) else sum(bs)
    total = sum(t.size_bytes for l in layer_stats for t in l.tensors)
    off = sum(t.size_bytes for ts in result.strategy_map.values() for t in ts)
    return blocks + total - off


def estimated_overhead(
    strategy_map: dict[str, list[TensorStatistics]],
    layer_stats: list[LayerStatistics],
    interp: MemoryTransferInterpolator | None,
) -> float:
    if interp is None:
        return 0.0
    t2c = calculate_transfer_to_compute_map(layer_stats, strategy_map)
    c2t = reverse_transfer_to_compute_map(t2c)
    idx = {l.label: i for i, l in enumerate(layer_stats)}
    total = sum(l.duration for l in layer_stats)
    sync = 0.0
    for i, layer in enumerate(layer_stats):
        tl = c2t.get(layer.label)
        if tl is None:
            continue
        nbytes = sum(t.size_bytes for t in strategy_map.get(tl, ()))
        if nbytes <= 0:
            continue
        ti = idx.get(tl)
        if ti is None:
            raise ValueError(f"Transfer label '{tl}' not found in layer statistics")
        window = sum(layer_stats[j].duration for j in range(ti, i))
        cost = interp.bytes_to_duration(nbytes)
        if cost > window:
            sync += cost - window
    return 0.0 if total <= 0 else sync / total


def count_violations(block_data: BlockStrategyData, strategy_map, layer_stats) -> int:
    l2b = block_data.label_to_block_id
    seq = [l.label for l in layer_stats if l.label in l2b and strategy_map.get(l.label)]
    return sum(1 for a, b in zip(seq, seq[1:]) if l2b[a] == l2b[b])


def evaluate_strategy_result(
    result: StrategyResult,
    layer_stats: list[LayerStatistics],
    strategy_name: str,
    interpolator: MemoryTransferInterpolator | None = None,
    max_gpu_mem_bytes: int | None = None,
) -> StrategyScore:
    peak = peak_memory(result, layer_stats)
    over = estimated_overhead(result.strategy_map, layer_stats, interpolator) if interpolator else 0.0
    viol = count_violations(result.block_data, result.strategy_map, layer_stats) if result.block_data else 0
    ok = viol == 0 and (max_gpu_mem_bytes is None or peak <= max_gpu_mem_bytes)
    return StrategyScore(strategy_name, peak, over, viol, ok)


def require_layers(layer_stats: list[LayerStatistics], n: int = 2) -> None:
    if len(layer_stats) < n:
        raise StrategyComputeError(f"need at least {n} timed traps to pipeline, got {len(layer_stats)}")


_ = OptimizedRoundRobinAssignment  # re-exported for strategies
