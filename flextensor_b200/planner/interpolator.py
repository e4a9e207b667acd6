"""Host->device transfer cost model: bytes <-> milliseconds.

Behaviour matches ``src/flextensor/memory_transfer_interpolator.py:10-165``:
piecewise-linear interpolation in log-log space over measured (bytes, ms)
points, with linear extrapolation from the first/last segment. A copy-engine
transfer is affine in bytes (latency + bytes/bandwidth); on log-log axes that
curve is smooth and nearly straight at both ends, which is why the end
segments extrapolate well.
"""

from __future__ import annotations

import math
from bisect import bisect_left

# Results are bounded at 2**62 (bytes or ms): a nearly flat end segment (noisy timings of small
# copies) extrapolates with a huge log-log slope, and exp() of it would overflow.
_MAX_LOG = 62 * math.log(2.0)


class MemoryTransferInterpolator:
    def __init__(self, memory_transfers: dict[int, float]):
        if not memory_transfers:
            raise ValueError("memory_transfers dictionary cannot be empty")
        pts = sorted((float(b), float(ms)) for b, ms in memory_transfers.items())
        if any(b <= 0 for b, _ in pts):
            raise ValueError("All byte values must be positive")
        if any(ms <= 0 for _, ms in pts):
            raise ValueError("All duration values must be positive")
        self.bytes_array = [b for b, _ in pts]
        self.duration_array = [ms for _, ms in pts]
        self.min_bytes, self.max_bytes = self.bytes_array[0], self.bytes_array[-1]
        self.min_duration, self.max_duration = self.duration_array[0], self.duration_array[-1]
        self._lx = [math.log(b) for b in self.bytes_array]
        self._ly = [math.log(d) for d in self.duration_array]

    @staticmethod
    def _eval(xs: list[float], ys: list[float], x: float) -> float:
        n = len(xs)
        if n == 1:
            return ys[0]
        if x <= xs[0]:
            i = 0
        elif x >= xs[-1]:
            i = n - 2
        else:
            i = max(0, bisect_left(xs, x) - 1)
        dx = xs[i + 1] - xs[i]
        if dx == 0:
            # a zero-width end segment extrapolates flat from its outer point: the first point
            # below the range, the last point above it (reference memory_transfer_interpolator.py:121-139)
            if x >= xs[-1]:
                return ys[-1]
            return ys[i]
        return ys[i] + (ys[i + 1] - ys[i]) * (x - xs[i]) / dx

    def bytes_to_duration(self, size_bytes: int | float) -> float:
        if size_bytes <= 0:
            raise ValueError(f"size_bytes must be positive, got {size_bytes}")
        return math.exp(min(self._eval(self._lx, self._ly, math.log(float(size_bytes))), _MAX_LOG))

    def duration_to_bytes(self, duration_ms: float) -> float:
        if duration_ms <= 0:
            raise ValueError(f"duration_ms must be positive, got {duration_ms}")
        # durations are monotone in bytes for real measurements; sort defensively
        pairs = sorted(zip(self._ly, self._lx))
        ly = [p[0] for p in pairs]
        lx = [p[1] for p in pairs]
        return math.exp(min(self._eval(ly, lx, math.log(float(duration_ms))), _MAX_LOG))

    def get_bandwidth_mbps(self) -> float:
        return (self.bytes_array[-1] / (1024 * 1024)) / (self.duration_array[-1] / 1000.0)

    def __repr__(self) -> str:
        return (
            f"MemoryTransferInterpolator(bytes_range=[{self.min_bytes:.0f}, {self.max_bytes:.0f}], "
            f"duration_range=[{self.min_duration:.2f}, {self.max_duration:.2f}] ms, "
            f"bandwidth~{self.get_bandwidth_mbps():.2f} MB/s)"
        )


def create_interpolator_from_benchmarks(memory_transfers: dict[int, float]) -> MemoryTransferInterpolator:
    return MemoryTransferInterpolator(memory_transfers)
