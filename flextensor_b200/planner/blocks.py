"""GPU ring-slot planning: which transfer label lands in which slot, and slot sizes.

Constraint (``src/flextensor/memory_block_planner.py:24-122``): two transfer
labels adjacent in execution order may not share a slot, otherwise the H2D for
the second would overwrite weights the first trap is still reading. That is a
colouring of a path graph (cyclic when the schedule wraps across forwards);
each slot's size is the largest label it hosts.

Two assignment policies are provided, named after the reference's
(``src/flextensor/strategy/assignment.py:37-326``):

* :class:`StrictRoundRobinAssignment` -- label ``k`` (k-th transferring label)
  goes to slot ``k % n``.
* :class:`OptimizedRoundRobinAssignment` -- for every slot count in
  ``[min_blocks, max_blocks]`` it packs labels by a size-aware greedy colouring
  (largest labels first into the slot whose current maximum grows least while
  respecting the adjacency and wrap-around constraints) and keeps the count
  with the smallest total slot bytes. This is a different search from the
  reference's exhaustive/greedy hybrid; it targets the same objective.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Protocol


class MemoryBlockPlanner:
    """Path-graph colouring of labels (execution order) onto slots."""

    def __init__(self, layer_sizes: OrderedDict[str, int] | dict[str, int], cyclic: bool = False):
        """``cyclic``: the schedule wraps across forwards (the last transfer label feeds the first
        compute label of the next forward), so the first and last labels are adjacent too; an
        odd number of labels then needs three slots."""
        self.layer_sizes = OrderedDict(layer_sizes)
        self.layers = list(self.layer_sizes)
        self.cyclic = cyclic and len(self.layers) > 2

    def _neighbours(self, idx: int) -> set[str]:
        out = set()
        n = len(self.layers)
        if idx > 0:
            out.add(self.layers[idx - 1])
        elif self.cyclic:
            out.add(self.layers[-1])
        if idx + 1 < n:
            out.add(self.layers[idx + 1])
        elif self.cyclic:
            out.add(self.layers[0])
        return out

    def find_minimum_blocks_sequential(self) -> int:
        if not self.layers:
            return 0
        if len(self.layers) == 1:
            return 1
        return 3 if self.cyclic and len(self.layers) % 2 else 2

    def optimize_block_distribution(self, num_blocks: int) -> dict[int, list[str]]:
        """Balanced colouring with ``num_blocks`` slots (fewest-labels slot first)."""
        need = self.find_minimum_blocks_sequential()
        if num_blocks < need:
            raise ValueError(f"Need at least {need} blocks")
        blocks: dict[int, list[str]] = {i: [] for i in range(num_blocks)}
        where: dict[str, int] = {}
        for idx, label in enumerate(self.layers):
            banned = {where[n] for n in self._neighbours(idx) if n in where}
            choices = [b for b in range(num_blocks) if b not in banned]
            if not choices:
                raise ValueError(f"Cannot place layer {label} in any block")
            best = min(choices, key=lambda b: (len(blocks[b]), b))
            blocks[best].append(label)
            where[label] = best
        return {b: v for b, v in blocks.items() if v}

    def allocate_blocks(self, num_blocks: int, block_capacity: int | None = None) -> dict[int, list[str]]:
        """First-fit colouring that also respects a per-slot cumulative capacity."""
        if num_blocks <= 0:
            raise ValueError("Number of blocks must be positive")
        blocks: dict[int, list[str]] = {i: [] for i in range(num_blocks)}
        used = dict.fromkeys(range(num_blocks), 0)
        where: dict[str, int] = {}

        def place(i: int) -> bool:
            if i == len(self.layers):
                return True
            label = self.layers[i]
            size = self.layer_sizes[label]
            banned = {where[n] for n in self._neighbours(i) if n in where}
            for b in range(num_blocks):
                if b in banned or (block_capacity is not None and used[b] + size > block_capacity):
                    continue
                blocks[b].append(label)
                used[b] += size
                where[label] = b
                if place(i + 1):
                    return True
                blocks[b].pop()
                used[b] -= size
                del where[label]
            return False

        if place(0):
            return blocks
        raise ValueError(f"Cannot allocate {len(self.layers)} layers to {num_blocks} blocks with given constraints")

    def find_minimum_blocks(self, block_capacity: int | None = None) -> tuple[int, dict[int, list[str]]]:
        if not self.layers:
            return 0, {}
        lo, hi = 1, len(self.layers)
        while lo < hi:
            mid = (lo + hi) // 2
            try:
                self.allocate_blocks(mid, block_capacity)
                hi = mid
            except ValueError:
                lo = mid + 1
        return lo, self.allocate_blocks(lo, block_capacity)

    def find_minimum_block_sizes(self, allocation: dict[int, list[str]]) -> dict[int, int]:
        return {b: max((self.layer_sizes[l] for l in labels), default=0) for b, labels in allocation.items()}


# --------------------------------------------------------------------------- assignment policies


class AssignmentStrategy(Protocol):
    def assign(self, label_sizes: OrderedDict[str, int]) -> dict[str, int]: ...


def _valid(order: list[str], where: dict[str, int], cyclic: bool) -> bool:
    for a, b in zip(order, order[1:]):
        if where[a] == where[b]:
            return False
    if cyclic and len(order) > 2 and where[order[0]] == where[order[-1]]:
        return False
    return True


class StrictRoundRobinAssignment:
    """k-th transferring label -> slot ``k % n_blocks``."""

    def __init__(self, n_blocks: int | None = None):
        self.n_blocks = n_blocks

    def assign(self, label_sizes: OrderedDict[str, int], n_blocks: int | None = None) -> dict[str, int]:
        n = n_blocks or self.n_blocks or 2
        return {label: k % n for k, label in enumerate(label_sizes)}


class OptimizedRoundRobinAssignment:
    """Size-aware colouring minimising total slot bytes over a range of slot counts."""

    def __init__(self, min_blocks: int | None = 2, max_blocks: int | None = 4, cyclic: bool = True):
        self.min_blocks = max(2, min_blocks or 2)
        self.max_blocks = max(self.min_blocks, max_blocks or self.min_blocks)
        self.cyclic = cyclic

    def _pack(self, order: list[str], sizes: dict[str, int], n: int) -> dict[str, int] | None:
        pos = {l: i for i, l in enumerate(order)}
        where: dict[str, int] = {}
        cap = [0] * n
        for label in sorted(order, key=lambda l: (-sizes[l], pos[l])):
            i = pos[label]
            nbrs = []
            if i > 0:
                nbrs.append(order[i - 1])
            if i + 1 < len(order):
                nbrs.append(order[i + 1])
            if self.cyclic and len(order) > 2:
                if i == 0:
                    nbrs.append(order[-1])
                if i == len(order) - 1:
                    nbrs.append(order[0])
            banned = {where[x] for x in nbrs if x in where}
            choices = [b for b in range(n) if b not in banned]
            if not choices:
                return None
            best = min(choices, key=lambda b: (max(cap[b], sizes[label]) - cap[b], b))
            where[label] = best
            cap[best] = max(cap[best], sizes[label])
        return where

    def assign(self, label_sizes: OrderedDict[str, int], n_blocks: int | None = None) -> dict[str, int]:
        order = list(label_sizes)
        if not order:
            return {}
        sizes = dict(label_sizes)
        lo = self.min_blocks
        hi = max(lo, n_blocks or self.max_blocks)
        best: tuple[int, int, dict[str, int]] | None = None
        for n in range(lo, hi + 1):
            where = self._pack(order, sizes, n)
            if where is None or not _valid(order, where, self.cyclic):
                # fall back to round robin for this n
                where = {l: k % n for k, l in enumerate(order)}
                if not _valid(order, where, False):
                    continue
            total = sum(max((sizes[l] for l in order if where[l] == b), default=0) for b in range(n))
            key = (total, n)
            if best is None or key < best[:2]:
                best = (total, n, where)
        if best is None:
            return {l: k % 2 for k, l in enumerate(order)}
        # renumber slots densely in first-use order
        remap: dict[int, int] = {}
        for l in order:
            remap.setdefault(best[2][l], len(remap))
        return {l: remap[best[2][l]] for l in order}


def allocation_from_assignment(order: list[str], where: dict[str, int]) -> dict[int, list[str]]:
    out: dict[int, list[str]] = {}
    for l in order:
        out.setdefault(where[l], []).append(l)
    return dict(sorted(out.items()))
