"""Inference offload timing: per-trap transfer, compute and exposed-wait times.

Measurement model (reference: ``src/flextensor/offload_timing.py:31-852``):

* transfer ms -- copy-stream events around each H2D;
* compute ms  -- compute-stream events at trap ``enter``/``exit``;
* wait ms     -- compute-stream events recorded right before and right after
  the ready-wait; their gap is time the compute stream sat idle on a copy
  (transfer NOT hidden).

``hidden_fraction = 1 - sum(wait) / sum(transfer)`` is the headline "% of
transfer time hidden". Events use ``external=True`` in ``cuda_graph`` mode so
``elapsed_time`` reads the latest replay. Passes are resolved lazily (one
``synchronize`` at collection time, never on the hot path) into a bounded ring
of ``MAX_PASSES`` records.
"""

from __future__ import annotations

import statistics
from collections import deque
from dataclasses import dataclass, field

import torch

MAX_PASSES = 1024


@dataclass(frozen=True, slots=True)
class TrapTimingRecord:
    """One trap in one forward pass (ms); ``wait_ms == 0`` means the copy was fully hidden."""

    label: str
    transfer_ms: float = 0.0
    compute_ms: float = 0.0
    wait_ms: float = 0.0
    transfer_bytes: int = 0


@dataclass(frozen=True, slots=True)
class OffloadTimingSnapshot:
    """One forward pass; totals are derived from ``per_trap``."""

    per_trap: tuple = ()

    @property
    def total_wait_ms(self) -> float:
        return sum(r.wait_ms for r in self.per_trap)

    @property
    def total_transfer_ms(self) -> float:
        return sum(r.transfer_ms for r in self.per_trap)

    @property
    def total_compute_ms(self) -> float:
        return sum(r.compute_ms for r in self.per_trap)


@dataclass(frozen=True, slots=True)
class TrapTimingStats:
    """One trap aggregated over passes."""

    label: str
    compute_min: float = 0.0
    compute_max: float = 0.0
    compute_avg: float = 0.0
    compute_median: float = 0.0
    compute_std: float = 0.0
    transfer_min: float = 0.0
    transfer_max: float = 0.0
    transfer_avg: float = 0.0
    transfer_median: float = 0.0
    transfer_std: float = 0.0
    wait_min: float = 0.0
    wait_max: float = 0.0
    wait_avg: float = 0.0
    wait_median: float = 0.0
    wait_std: float = 0.0
    transfer_bytes: int = 0

    def compute_budget_ms(self, *, conservative: bool = False) -> float:
        """Compute window used as the transfer budget by a replan (median; min when conservative)."""
        order = (self.compute_min, self.compute_median, self.compute_avg) if conservative else (
            self.compute_median, self.compute_avg, self.compute_min)
        for v in order:
            if v and v > 0:
                return float(v)
        return 0.0


def _stats(vals: list[float]) -> tuple[float, float, float, float, float]:
    if not vals:
        return (0.0, 0.0, 0.0, 0.0, 0.0)
    return (min(vals), max(vals), sum(vals) / len(vals), statistics.median(vals),
            statistics.pstdev(vals) if len(vals) > 1 else 0.0)


@dataclass(slots=True)
class OffloadTimingReport:
    """Per-trap aggregates (``per_trap``) and the raw passes (``passes``)."""

    per_trap: tuple = ()
    passes: tuple = ()

    @property
    def num_passes(self) -> int:
        return len(self.passes)

    @property
    def traps(self) -> tuple:
        return self.per_trap

    @property
    def total_compute_sum(self) -> float:
        return sum(s.total_compute_ms for s in self.passes)

    @property
    def total_transfer_sum(self) -> float:
        return sum(s.total_transfer_ms for s in self.passes)

    @property
    def total_wait_sum(self) -> float:
        return sum(s.total_wait_ms for s in self.passes)

    @property
    def total_compute_avg(self) -> float:
        return self.total_compute_sum / self.num_passes if self.num_passes else 0.0

    @property
    def total_transfer_avg(self) -> float:
        return self.total_transfer_sum / self.num_passes if self.num_passes else 0.0

    @property
    def total_wait_avg(self) -> float:
        return self.total_wait_sum / self.num_passes if self.num_passes else 0.0

    @property
    def hidden_fraction(self) -> float:
        """Share of host->device copy time that did not stall compute."""
        tr = self.total_transfer_sum
        return 1.0 if tr <= 0 else max(0.0, 1.0 - self.total_wait_sum / tr)

    def compute_budgets_by_profile_label(self, profile_labels=None, *, conservative: bool = False) -> dict[str, float]:
        """Compute window (ms) per trap label, the input of a replan from production timings."""
        by = {t.label: t.compute_budget_ms(conservative=conservative) for t in self.per_trap}
        if profile_labels is None:
            return by
        return {l: by[l] for l in profile_labels if l in by and by[l] > 0}


def format_offload_timing_table(report: OffloadTimingReport | None) -> str:
    if report is None or not report.per_trap:
        return "(no offload timing samples)"
    rows = [f"{'trap':<32} {'compute ms':>11} {'transfer ms':>12} {'wait ms':>9} {'MB':>9}"]
    for t in report.per_trap:
        rows.append(f"{t.label[:32]:<32} {t.compute_avg:>11.3f} {t.transfer_avg:>12.3f} {t.wait_avg:>9.3f} "
                    f"{t.transfer_bytes / 2**20:>9.1f}")
    rows.append(f"{'TOTAL / pass':<32} {report.total_compute_avg:>11.3f} {report.total_transfer_avg:>12.3f} "
                f"{report.total_wait_avg:>9.3f}  passes={report.num_passes} hidden={report.hidden_fraction * 100:.1f}%")
    return "\n".join(rows)


class _HostStamp:
    """CPU-device stand-in for a CUDA event (copies there are synchronous)."""

    def __init__(self):
        self.t = None

    def record(self, *_):
        import time

        self.t = time.perf_counter()

    def elapsed_time(self, other: "_HostStamp") -> float:
        return (other.t - self.t) * 1e3


class OffloadTimingCollector:
    def __init__(self, device: torch.device, mode: str = "eager"):
        self.device = torch.device(device)
        self.external = mode == "cuda_graph"
        self.enabled = mode != "off"
        self.host_clock = self.device.type != "cuda"  # CPU device: wall-clock stamps
        self._pending: list[tuple[dict, list]] = []
        self._done: deque[OffloadTimingSnapshot] = deque(maxlen=MAX_PASSES)
        self._cur: dict | None = None

    def _ev(self):
        if self.host_clock:
            return _HostStamp()
        return torch.cuda.Event(enable_timing=True, external=self.external) if self.external else \
            torch.cuda.Event(enable_timing=True)

    def _record(self, e) -> None:
        if self.host_clock:
            e.record()
        else:
            e.record(torch.cuda.current_stream(self.device))

    def on_pass_start(self) -> None:
        if self.enabled:
            self._cur = {}

    def on_enter(self, label: str) -> None:
        if self.enabled and self._cur is not None:
            e = self._ev()
            self._record(e)
            self._cur[label] = [e, None]

    def on_exit(self, label: str) -> None:
        if self.enabled and self._cur is not None and label in self._cur:
            e = self._ev()
            self._record(e)
            self._cur[label][1] = e

    def on_pass_end(self, engine) -> None:
        if not self.enabled or self._cur is None:
            return
        self._pending.append((self._cur, engine.take_records()))
        self._cur = None

    def _resolve(self) -> None:
        if not self._pending:
            return
        if not self.host_clock:
            torch.cuda.synchronize(self.device)
        for comp, recs in self._pending:
            vals: dict[str, dict] = {}
            for label, (a, b) in comp.items():
                d = vals.setdefault(label, {})
                if a is not None and b is not None:
                    d["compute_ms"] = a.elapsed_time(b)
            for rec in recs:
                # records are keyed by the compute label that reads the copy
                d = vals.setdefault(rec.key, {})
                d["transfer_bytes"] = rec.nbytes
                if getattr(rec, "transfer_ms", None) is not None:
                    d["transfer_ms"] = rec.transfer_ms
                elif rec.start is not None and rec.end is not None:
                    d["transfer_ms"] = rec.start.elapsed_time(rec.end)
                if getattr(rec, "wait_ms", None) is not None:
                    d["wait_ms"] = rec.wait_ms
                elif rec.wait_start is not None and rec.wait_end is not None:
                    d["wait_ms"] = rec.wait_start.elapsed_time(rec.wait_end)
            self._done.append(OffloadTimingSnapshot(tuple(TrapTimingRecord(l, **d) for l, d in vals.items())))
        self._pending.clear()

    def reset(self) -> None:
        self._pending.clear()
        self._done.clear()

    def report(self) -> OffloadTimingReport | None:
        if not self.enabled:
            return None
        self._resolve()
        passes = tuple(self._done)
        labels: list[str] = []
        for p in passes:
            for r in p.per_trap:
                if r.label not in labels:
                    labels.append(r.label)
        per = []
        for l in labels:
            rs = [r for p in passes for r in p.per_trap if r.label == l]
            c, t, w = _stats([r.compute_ms for r in rs]), _stats([r.transfer_ms for r in rs]), _stats(
                [r.wait_ms for r in rs])
            per.append(TrapTimingStats(l, *c, *t, *w, transfer_bytes=max(r.transfer_bytes for r in rs)))
        return OffloadTimingReport(per_trap=tuple(per), passes=passes)
