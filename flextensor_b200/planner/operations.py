"""Plan rewrites shared by strategies.

Parity with ``src/flextensor/strategy_operations.py`` (``rearrange_transfers`` 623-759,
``find_transfers_for_preload`` 761-798, ``remove_layers_compound`` 282,
``create_allocation_ordered`` 841). A plan maps a *transfer label* (the trap during which a
copy is issued) to the tensors it streams; ``t2c`` maps the transfer label to the *compute
label* that consumes it.
"""

from __future__ import annotations

from flextensor_b200.core.stats import LayerStatistics, TensorStatistics
from flextensor_b200.planner.interpolator import MemoryTransferInterpolator


def create_allocation_ordered(order: list[str], label_to_block: dict[str, int]) -> dict[int, list[str]]:
    """Block id -> its transfer labels in execution order."""
    out: dict[int, list[str]] = {}
    for l in order:
        if l in label_to_block:
            out.setdefault(label_to_block[l], []).append(l)
    return out


def find_transfers_for_preload(order: list[str], t2c: dict[str, str]) -> list[str]:
    """Transfer labels whose consumer runs no later than the transfer itself in one pass: they
    wrap around the forward, so their first copy must be issued before the first pass."""
    idx = {l: i for i, l in enumerate(order)}
    return [t for t, c in t2c.items() if t in idx and c in idx and idx[c] <= idx[t]]


def remove_layers_compound(layer_stats: list[LayerStatistics], operations: list[dict]) -> list[LayerStatistics]:
    """Merge or drop traps before planning.

    Each operation is ``{"op": "remove", "labels": [...]}`` (the trap leaves the schedule: its
    tensors are no longer planned, so they stay resident, and its compute time is added to
    the previous trap, whose window it still extends) or ``{"op": "merge", "labels": [a, b,
    ...]}`` (consecutive traps become one labelled ``a``; an analysis view -- the runtime
    applies only ``remove``)."""
    rows = [[l.label, list(l.tensors), l.duration] for l in layer_stats]  # mutable working copy
    for op in operations:
        kind, labels = op.get("op"), list(op.get("labels", []))
        if kind == "remove":
            for lab in labels:
                i = next((k for k, r in enumerate(rows) if r[0] == lab), None)
                if i is None or len(rows) < 2:
                    continue
                gone = rows.pop(i)
                rows[(i - 1) % len(rows)][2] += gone[2]
        elif kind == "merge":
            pos = [k for k, r in enumerate(rows) if r[0] in labels]
            if len(pos) < 2:
                continue
            if pos != list(range(pos[0], pos[0] + len(pos))):
                raise ValueError(f"merge needs consecutive traps, got {labels}")
            head = rows[pos[0]]
            for k in pos[1:]:
                head[1] += rows[k][1]
                head[2] += rows[k][2]
            del rows[pos[0] + 1:pos[-1] + 1]
        else:
            raise ValueError(f"unknown remove-layers operation {kind!r}")
    return [LayerStatistics(label=r[0], tensors=r[1], duration=r[2]) for r in rows]


def rearrange_transfers(plan: dict[str, list[TensorStatistics]], t2c: dict[str, str],
                        layer_stats: list[LayerStatistics], interp: MemoryTransferInterpolator | None,
                        *, gap: int = 1, cyclic: bool = True) -> tuple[dict[str, list[TensorStatistics]], dict[str, str]]:
    """Move each transfer to the earliest free trap that still hides it.

    A transfer currently issued at trap T for consumer C may move to an earlier trap S when
    (1) no transfer is issued at S, (2) S is at least ``gap`` traps before C, (3) the copy
    time (interpolated) fits the compute between S and C, and (4) no other transfer's
    [issue, consume) interval overlaps it (one copy in flight per slot pair). Returns the new
    plan and transfer->compute map; the consumer of every tensor is unchanged."""
    n = len(layer_stats)
    if n < 3 or not plan:
        return dict(plan), dict(t2c)
    order = [l.label for l in layer_stats]
    idx = {l: i for i, l in enumerate(order)}
    dur = [l.duration for l in layer_stats]

    def ms(ts):
        b = sum(t.size_bytes for t in ts)
        return interp.bytes_to_duration(b) if interp is not None else 0.0

    def dist(a: int, b: int) -> int:  # traps from a forward to b
        d = b - a
        return d % n if cyclic else d

    occupied = {idx[t] for t in plan if plan[t]}
    new_plan: dict[str, list[TensorStatistics]] = {}
    new_t2c: dict[str, str] = {}
    for t in sorted(plan, key=lambda x: idx[x]):
        ts = plan[t]
        if not ts or t not in t2c:
            continue
        c, here = idx[t2c[t]], idx[t]
        need = ms(ts)
        best = here
        for back in range(max(1, gap), n):
            s_ = (c - back) % n if cyclic else c - back
            if s_ < 0:
                break
            if s_ != here and s_ in occupied:
                break  # another transfer is issued there: never jump over it
            window = sum(dur[(s_ + k) % n] for k in range(dist(s_, c)))
            if window >= need:
                best = s_  # latest issue point that still hides the copy
                break
        if best != here:
            occupied.discard(here)
            occupied.add(best)
        new_plan[order[best]] = ts
        new_t2c[order[best]] = order[c]
    return new_plan, new_t2c
