"""Per-trap statistics: the planner's input.

Record types mirror the reference's pydantic models (``src/flextensor/collectors.py:11-30``)
because they are serialised verbatim into ``profile.json`` (``stats`` and the
``load_strategy``/``release_strategy`` lists), so field names and order are part
of the on-disk contract.

The collector keeps, per trap label, the union of tensor ids the trap touched
and every duration sample; the strategy-time view reduces samples by median
(``src/flextensor/collectors.py:167-171``), which is robust to the first
post-transition forward being slow.
"""

from __future__ import annotations

import statistics
from collections import OrderedDict
from collections.abc import Iterable

from pydantic import BaseModel, ConfigDict


class TensorStatistics(BaseModel):
    """One offloadable tensor: identity, name, bytes and measured H2D time."""

    model_config = ConfigDict(frozen=True)

    tensor_id: int
    name: str
    size_bytes: int
    load_time_ms: float


class LayerStatistics(BaseModel):
    """One trap (offload unit): its tensors and its median compute duration (ms)."""

    model_config = ConfigDict(frozen=True)

    label: str
    tensors: list[TensorStatistics]
    duration: float


class IterativeTensorStatistics(TensorStatistics):
    """Collection-time alias of :class:`TensorStatistics`."""


class IterativeLayerStatistics(BaseModel):
    """Partial per-trap row; ``duration`` is ``None`` until a timed sample exists."""

    model_config = ConfigDict(frozen=True)

    label: str
    tensor_ids: list[int] | set[int]
    duration: float | None = None


def extract_memory_transfers_from_layer_stats(layer_stats: Iterable[LayerStatistics]) -> dict[int, float]:
    """Size (bytes) -> mean measured H2D ms over every profiled tensor of that size."""
    acc: dict[int, list[float]] = {}
    for layer in layer_stats:
        for t in layer.tensors:
            if t.load_time_ms > 0:
                acc.setdefault(t.size_bytes, []).append(t.load_time_ms)
    return {s: sum(v) / len(v) for s, v in acc.items()}


class LayerStatisticsCollector:
    """Accumulates :class:`LayerStatistics` rows from known tensor statistics."""

    def __init__(self, tensor_statistics_map: dict[int, TensorStatistics] | None = None) -> None:
        self.tensor_statistics_map = tensor_statistics_map or {}
        self.stats_map: OrderedDict[str, LayerStatistics] = OrderedDict()

    def add_all(self, label: str, tensor_ids: Iterable[int], duration: float) -> None:
        for tid in tensor_ids:
            self.add(label, tid, duration)

    def add(self, label: str, tensor_id: int, duration: float) -> None:
        ts = self.tensor_statistics_map.get(tensor_id)
        if ts is None:
            return
        row = self.stats_map.get(label)
        if row is None:
            row = LayerStatistics(label=label, tensors=[], duration=duration)
            self.stats_map[label] = row
        row.tensors.append(ts)

    def get_layer_stats(self) -> list[LayerStatistics]:
        return list(self.stats_map.values())


class IterativeLayerStatisticsCollector:
    """Per-label tensor-id unions plus duration samples across iterations.

    Labels keep first-seen execution order; a label re-entered in a later
    iteration keeps its original position (the schedule is cyclic per forward).
    """

    def __init__(self) -> None:
        self._ids: OrderedDict[str, set[int]] = OrderedDict()
        self._durations: dict[str, list[float]] = {}
        self.iterations = 0

    def record_tensors(self, label: str, tensor_ids: Iterable[int]) -> None:
        self._ids.setdefault(label, set()).update(tensor_ids)

    def record_duration(self, label: str, duration_ms: float) -> None:
        self._ids.setdefault(label, set())
        self._durations.setdefault(label, []).append(float(duration_ms))

    def clear_durations(self) -> None:
        self._durations.clear()

    def labels(self) -> list[str]:
        return list(self._ids)

    def tensor_ids(self, label: str) -> set[int]:
        return set(self._ids.get(label, ()))

    def samples(self, label: str) -> list[float]:
        return list(self._durations.get(label, ()))

    def all_samples(self) -> dict[str, list[float]]:
        return {k: list(v) for k, v in self._durations.items()}

    def get_layer_stats(self) -> list[IterativeLayerStatistics]:
        out = []
        for label, ids in self._ids.items():
            s = self._durations.get(label)
            out.append(
                IterativeLayerStatistics(
                    label=label, tensor_ids=sorted(ids), duration=(statistics.median(s) if s else None)
                )
            )
        return out

    def drop_label(self, label: str) -> None:
        self._ids.pop(label, None)
        self._durations.pop(label, None)


def compute_layer_statistics(
    rows: Iterable[IterativeLayerStatistics],
    tensor_stats: dict[int, TensorStatistics],
) -> list[LayerStatistics]:
    """Join collection rows with per-tensor stats; drop untimed rows.

    Mirrors ``src/flextensor/tensor_manager.py:356-393``: rows with no duration
    sample cannot be scheduled and are omitted (their tensors stay resident).
    A tensor claimed by several labels is attributed to the first one only,
    which keeps block packing free of duplicates.
    """
    seen: set[int] = set()
    out: list[LayerStatistics] = []
    for row in rows:
        if row.duration is None:
            continue
        tensors = []
        for tid in sorted(row.tensor_ids):
            ts = tensor_stats.get(tid)
            if ts is None or tid in seen:
                continue
            seen.add(tid)
            tensors.append(ts)
        out.append(LayerStatistics(label=row.label, tensors=tensors, duration=float(row.duration)))
    return out
