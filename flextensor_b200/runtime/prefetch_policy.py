"""Detect prefetches that a CUDA-graph piece boundary forces onto the critical path.

When a forward is captured piecewise (one CUDA graph per piece, as serving engines do), every
piece must join the copy stream before its capture ends. A prefetch issued in one piece and
consumed in a later one is then completed at the boundary: still correct, but its transfer no
longer overlaps compute. The loader reports every schedule (transfer label -> compute label)
and every wait; at a piece join, prefetches still outstanding are reported (``warn``) or raise
(``error``). At the last layer of a forward, prefetches for compute labels already consumed
in this pass belong to the next forward (the cyclic wrap-around) and are not reported.

Parity with ``src/flextensor/piecewise_prefetch_policy.py:40-151`` (modes ``off``/``warn``/
``error``, config field ``piecewise_prefetch``, env ``FT_PIECEWISE_PREFETCH``).
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

LOGGER = logging.getLogger(__name__)


class PiecewisePrefetchPolicyError(RuntimeError):
    pass


@dataclass(frozen=True, slots=True)
class OutstandingPrefetch:
    schedule_label: str
    compute_label: str


class PiecewisePrefetchPolicy:
    def __init__(self, *, enabled: bool = False, strict: bool = False) -> None:
        self.enabled = enabled
        self.strict = strict
        self._open: dict[str, str] = {}        # compute label -> schedule label
        self._consumed: set[str] = set()       # compute labels waited in this pass
        self.hits: list[OutstandingPrefetch] = []

    @classmethod
    def from_mode(cls, mode: str) -> "PiecewisePrefetchPolicy":
        if mode not in ("off", "warn", "error"):
            raise ValueError(f"piecewise_prefetch must be off|warn|error, got {mode!r}")
        return cls(enabled=mode != "off", strict=mode == "error")

    def reset(self) -> None:
        self._open.clear()
        self._consumed.clear()

    def on_schedule(self, schedule_label: str, compute_label: str) -> None:
        if self.enabled:
            self._open[compute_label] = schedule_label

    def on_wait(self, compute_label: str) -> None:
        if self.enabled:
            self._open.pop(compute_label, None)
            self._consumed.add(compute_label)

    def on_piece_join(self, *, at_last_layer: bool = False) -> list[OutstandingPrefetch]:
        if not self.enabled:
            return []
        pending = [OutstandingPrefetch(s, c) for c, s in self._open.items()
                   if not (at_last_layer and c in self._consumed)]
        if at_last_layer:
            self._consumed.clear()
        if pending:
            self.hits.extend(pending)
            msg = ("piecewise graph join before the consuming trap waited: "
                   + ", ".join(f"{p.schedule_label}->{p.compute_label}" for p in pending)
                   + " (the H2D completes on the critical path of the earlier piece)")
            if self.strict:
                raise PiecewisePrefetchPolicyError(msg)
            LOGGER.warning(msg)
        return pending
