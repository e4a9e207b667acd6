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


@dataclass
class TrapTimingRecord:
    label: str
    compute_ms: float = 0.0
    transfer_ms: float = 0.0
    wait_ms: float = 0.0
    transfer_bytes: int = 0


@dataclass
class OffloadTimingSnapshot:
    label: str
    samples: int
    compute_ms: dict[str, float]
    transfer_ms: dict[str, float]
    wait_ms: dict[str, float]
    transfer_bytes: int


def _agg(v: list[float]) -> dict[str, float]:
    if not v:
        return {"min": 0.0, "max": 0.0, "avg": 0.0, "std": 0.0}
    return {"min": min(v), "max": max(v), "avg": sum(v) / len(v), "std": statistics.pstdev(v) if len(v) > 1 else 0.0}


@dataclass
class OffloadTimingReport:
    passes: int
    traps: list[OffloadTimingSnapshot] = field(default_factory=list)

    @property
    def total_transfer_ms(self) -> float:
        return sum(t.transfer_ms["avg"] for t in self.traps)

    @property
    def total_wait_ms(self) -> float:
        return sum(t.wait_ms["avg"] for t in self.traps)

    @property
    def total_compute_ms(self) -> float:
        return sum(t.compute_ms["avg"] for t in self.traps)

    @property
    def hidden_fraction(self) -> float:
        tr = self.total_transfer_ms
        return 1.0 if tr <= 0 else max(0.0, 1.0 - self.total_wait_ms / tr)

    def compute_budgets_by_profile_label(self) -> dict[str, float]:
        """Mean compute ms per trap (input to a replan from production timings)."""
        return {t.label: t.compute_ms["avg"] for t in self.traps}


def format_offload_timing_table(report: OffloadTimingReport | None) -> str:
    if report is None or not report.traps:
        return "(no offload timing samples)"
    rows = [f"{'trap':<32} {'n':>5} {'compute ms':>11} {'transfer ms':>12} {'wait ms':>9} {'MB':>9}"]
    for t in report.traps:
        rows.append(f"{t.label[:32]:<32} {t.samples:>5} {t.compute_ms['avg']:>11.3f} {t.transfer_ms['avg']:>12.3f} "
                    f"{t.wait_ms['avg']:>9.3f} {t.transfer_bytes / 2**20:>9.1f}")
    rows.append(f"{'TOTAL':<32} {report.passes:>5} {report.total_compute_ms:>11.3f} {report.total_transfer_ms:>12.3f} "
                f"{report.total_wait_ms:>9.3f}  hidden={report.hidden_fraction * 100:.1f}%")
    return "\n".join(rows)


class OffloadTimingCollector:
    def __init__(self, device: torch.device, mode: str = "eager"):
        self.device = torch.device(device)
        self.external = mode == "cuda_graph"
        self.enabled = self.device.type == "cuda" and mode != "off"
        self._pending: list[tuple[dict, list]] = []
        self._done: deque[dict[str, TrapTimingRecord]] = deque(maxlen=MAX_PASSES)
        self._cur: dict | None = None

    def _ev(self):
        return torch.cuda.Event(enable_timing=True, external=self.external) if self.external else \
            torch.cuda.Event(enable_timing=True)

    def on_pass_start(self) -> None:
        if self.enabled:
            self._cur = {}

    def on_enter(self, label: str) -> None:
        if self.enabled and self._cur is not None:
            e = self._ev()
            e.record(torch.cuda.current_stream(self.device))
            self._cur[label] = [e, None]

    def on_exit(self, label: str) -> None:
        if self.enabled and self._cur is not None and label in self._cur:
            e = self._ev()
            e.record(torch.cuda.current_stream(self.device))
            self._cur[label][1] = e

    def on_pass_end(self, engine) -> None:
        if not self.enabled or self._cur is None:
            return
        self._pending.append((self._cur, engine.take_records()))
        self._cur = None

    def _resolve(self) -> None:
        if not self._pending:
            return
        torch.cuda.synchronize(self.device)
        for comp, recs in self._pending:
            out: dict[str, TrapTimingRecord] = {}
            for label, (a, b) in comp.items():
                r = out.setdefault(label, TrapTimingRecord(label))
                if a is not None and b is not None:
                    r.compute_ms = a.elapsed_time(b)
            for rec in recs:
                # records are keyed by the compute label that reads the copy
                r = out.setdefault(rec.key, TrapTimingRecord(rec.key))
                r.transfer_bytes = rec.nbytes
                if getattr(rec, "transfer_ms", None) is not None:
                    r.transfer_ms = rec.transfer_ms
                elif rec.start is not None and rec.end is not None:
                    r.transfer_ms = rec.start.elapsed_time(rec.end)
                if getattr(rec, "wait_ms", None) is not None:
                    r.wait_ms = rec.wait_ms
                elif rec.wait_start is not None and rec.wait_end is not None:
                    r.wait_ms = rec.wait_start.elapsed_time(rec.wait_end)
            self._done.append(out)
        self._pending.clear()

    def reset(self) -> None:
        self._pending.clear()
        self._done.clear()

    def report(self) -> OffloadTimingReport | None:
        if not self.enabled:
            return None
        self._resolve()
        if not self._done:
            return OffloadTimingReport(passes=0)
        labels: list[str] = []
        for p in self._done:
            for l in p:
                if l not in labels:
                    labels.append(l)
        traps = []
        for l in labels:
            rs = [p[l] for p in self._done if l in p]
            traps.append(OffloadTimingSnapshot(
                l, len(rs), _agg([r.compute_ms for r in rs]), _agg([r.transfer_ms for r in rs]),
                _agg([r.wait_ms for r in rs]), max(r.transfer_bytes for r in rs)))
        return OffloadTimingReport(passes=len(self._done), traps=traps)
