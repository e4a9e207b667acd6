"""Profiling-quality checks on per-trap duration samples.

Parity with ``src/flextensor/layer_statistics_analyzer.py:20-254``: per-label duration
statistics (mean/median/std/min/max and coefficient of variation), a formatted table,
consistency warnings (too few samples, noisy traps), the untimed-trap report (labels that
own tensors but never got a duration sample, so the planner cannot schedule them and their
tensors stay resident), and ``report_profiling_quality`` which logs all of it on the
``flextensor_b200.diagnostics`` logger.
"""

from __future__ import annotations

import logging
import math
import statistics
from dataclasses import dataclass

from flextensor_b200.core.stats import IterativeLayerStatisticsCollector, LayerStatistics

DIAG = logging.getLogger("flextensor_b200.diagnostics")
RECOMMENDED_SAMPLES = 3
CV_WARN = 0.25


@dataclass(frozen=True)
class LayerDurationStatistics:
    label: str
    samples: int
    mean_ms: float
    median_ms: float
    std_ms: float
    min_ms: float
    max_ms: float

    @property
    def coefficient_of_variation(self) -> float:
        return self.std_ms / self.mean_ms if self.mean_ms > 0 else 0.0


class LayerStatisticsAnalyzer:
    def __init__(self, collector: IterativeLayerStatisticsCollector) -> None:
        self._stats: dict[str, LayerDurationStatistics] = {}
        for label in collector.labels():
            s = collector.samples(label)
            if not s:
                continue
            mean = statistics.fmean(s)
            std = statistics.pstdev(s) if len(s) > 1 else 0.0
            self._stats[label] = LayerDurationStatistics(label, len(s), mean, statistics.median(s), std,
                                                         min(s), max(s))

    def get_statistics(self) -> list[LayerDurationStatistics]:
        return list(self._stats.values())

    def get_layer_statistics(self, label: str) -> LayerDurationStatistics | None:
        return self._stats.get(label)

    def format_statistics_table(self) -> str:
        rows = [f"{'label':<32} {'n':>3} {'median ms':>10} {'mean ms':>10} {'std ms':>9} {'cv':>6}"]
        for st in self._stats.values():
            rows.append(f"{st.label[:32]:<32} {st.samples:>3} {st.median_ms:>10.3f} {st.mean_ms:>10.3f} "
                        f"{st.std_ms:>9.3f} {st.coefficient_of_variation:>6.2f}")
        return "\n".join(rows)

    def check_measurement_consistency(self, *, min_samples: int = RECOMMENDED_SAMPLES,
                                      cv_threshold: float = CV_WARN, max_listed: int = 5) -> list[str]:
        """Human-readable warnings; empty when every trap looks well measured."""
        out = []
        few = [s for s in self._stats.values() if s.samples < min_samples]
        if few:
            listed = ", ".join(f"'{s.label}' ({s.samples} samples)" for s in few[:max_listed])
            more = f" and {len(few) - max_listed} more" if len(few) > max_listed else ""
            out.append(f"Low sample count for {len(few)} trap(s): {listed}{more}. "
                       f"Use profiling_iters >= {min_samples} for reliable plans.")
        noisy = [s for s in self._stats.values() if s.samples > 1 and s.coefficient_of_variation > cv_threshold]
        if noisy:
            listed = ", ".join(f"'{s.label}' (cv={s.coefficient_of_variation:.2f})" for s in noisy[:max_listed])
            more = f" and {len(noisy) - max_listed} more" if len(noisy) > max_listed else ""
            out.append(f"High duration variance for {len(noisy)} trap(s): {listed}{more}; the median is used.")
        return out


def format_effective_layer_duration_table(layer_stats: list[LayerStatistics]) -> str:
    rows = [f"{'label':<32} {'duration ms':>12} {'tensors':>8} {'MB':>10}"]
    for ls in layer_stats:
        mb = sum(t.size_bytes for t in ls.tensors) / 1e6
        rows.append(f"{ls.label[:32]:<32} {ls.duration:>12.3f} {len(ls.tensors):>8} {mb:>10.2f}")
    return "\n".join(rows)


class UntimedTrapsReport:
    """Labels that own tensors but recorded no duration (their tensors stay resident)."""

    def __init__(self, collector: IterativeLayerStatisticsCollector) -> None:
        self.labels = [l for l in collector.labels() if not collector.samples(l) and collector.tensor_ids(l)]

    def is_empty(self) -> bool:
        return not self.labels

    def format(self) -> str:
        return (f"{len(self.labels)} trap(s) were never timed and cannot be scheduled "
                f"(tensors stay GPU-resident): {', '.join(self.labels[:10])}"
                + (" ..." if len(self.labels) > 10 else ""))


def report_profiling_quality(collector: IterativeLayerStatisticsCollector, *, verbose: bool = False,
                             logger: logging.Logger = DIAG) -> list[str]:
    """Log sample-count / variance warnings and untimed traps; returns the warnings."""
    an = LayerStatisticsAnalyzer(collector)
    warns = an.check_measurement_consistency()
    untimed = UntimedTrapsReport(collector)
    if not untimed.is_empty():
        warns.append(untimed.format())
    for w in warns:
        logger.warning(w)
    if verbose:
        logger.info("per-trap durations:\n%s", an.format_statistics_table())
    return warns


def _finite(x: float) -> bool:
    return not (math.isnan(x) or math.isinf(x))
