"""Transfer windows: how much compute time can hide the prefetch that feeds a trap.

Parity with ``src/flextensor/strategy/transfer_window.py:28-108``:

* :class:`SingleLayerWindow` -- only the trap right before the consumer;
* :class:`GapAwareWindow`    -- the preceding trap plus every earlier consecutive trap that
  issues no transfer of its own (those gaps are free copy-engine time).

``plan`` maps a transfer label to the tensors it streams; a label with an empty or missing
entry issues nothing. ``scale`` multiplies the window (a planner's safety factor).
"""

from __future__ import annotations

from typing import Protocol

from flextensor_b200.core.stats import LayerStatistics


class TransferWindowCalculator(Protocol):
    def compute_window(self, layer_stats: list[LayerStatistics], consumer_index: int,
                       plan: dict[str, list] | None = None, scale: float = 1.0) -> float: ...


class SingleLayerWindow:
    def compute_window(self, layer_stats, consumer_index, plan=None, scale=1.0) -> float:
        prev = (consumer_index - 1) % len(layer_stats)
        return layer_stats[prev].duration * scale


class GapAwareWindow:
    def __init__(self, cyclic: bool = True) -> None:
        self.cyclic = cyclic

    def compute_window(self, layer_stats, consumer_index, plan=None, scale=1.0) -> float:
        plan = plan or {}
        n = len(layer_stats)
        i = consumer_index - 1
        total = 0.0
        steps = 0
        while steps < n - 1:
            if i < 0:
                if not self.cyclic:
                    break
                i += n
            total += layer_stats[i].duration
            steps += 1
            j = i - 1
            if j < 0 and not self.cyclic:
                break
            if plan.get(layer_stats[j % n].label):
                break  # the trap before has its own transfer: the window ends here
            i = j
        return total * scale
