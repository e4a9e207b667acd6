"""Race check of the prefetch schedule without a GPU: for random profiles and every planner,
simulate the block loader's slot schedule (preloads, enter = wait for the own slot then issue
the next copy, exit = release the slot) over several forwards and assert that no copy ever
overwrites a slot whose weights a compute trap has not finished reading, and that every trap
finds its own weights in its slot."""

import random

import pytest

from flextensor_b200.core.stats import LayerStatistics, TensorStatistics
from flextensor_b200.planner import (
    BudgetFillStrategy,
    GreedyStrategy,
    KnapsackBlockStrategy,
    NthLayerStrategy,
)


def _profile(rng, n):
    out = []
    tid = 0
    for i in range(n):
        ts = []
        for _ in range(rng.randint(1, 3)):
            ts.append(TensorStatistics(tensor_id=tid, name=f"l{i}.t{tid}", size_bytes=rng.randint(1, 64) << 20,
                                       load_time_ms=1.0))
            tid += 1
        out.append(LayerStatistics(label=f"l{i}", tensors=ts, duration=rng.uniform(0.5, 20.0)))
    return out


def _simulate(layer_stats, result, passes=3):
    bd = result.block_data
    if bd is None or not result.strategy_map:
        return
    order = [l.label for l in layer_stats]
    idx = {l: i for i, l in enumerate(order)}
    t2c = dict(bd.transfer_to_compute_map)
    slot_of = dict(bd.label_to_block_id)
    compute_slot = {c: slot_of[t] for t, c in t2c.items()}
    content: dict[int, str | None] = {}
    busy: set[str] = set()           # compute traps that may still read their slot
    for t in t2c:                    # construction-time preloads (schedules that wrap)
        if idx[t2c[t]] <= idx[t]:
            content[slot_of[t]] = t2c[t]
    for p in range(passes):
        for label in order:
            if label in compute_slot:
                s = compute_slot[label]
                assert content.get(s) == label, f"pass {p}: {label} finds {content.get(s)} in slot {s}"
                busy.add(label)
            if label in slot_of:
                s = slot_of[label]
                cur = content.get(s)
                assert cur is None or cur not in busy or cur == t2c[label], \
                    f"pass {p}: copy for {t2c[label]} at {label} overwrites slot {s} still read by {cur}"
                if p > 0 or cur is None or cur not in busy:
                    pass
                content[s] = t2c[label]
            busy.discard(label)


PLANNERS = [
    lambda: NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True),
    lambda: NthLayerStrategy(2, threshold_mb=0.0, n_blocks=2, cyclic=True),
    lambda: NthLayerStrategy(1, threshold_mb=0.0, n_blocks=3, cyclic=False),
    lambda: GreedyStrategy(n_blocks=2),
    lambda: KnapsackBlockStrategy(n_blocks=2),
    lambda: BudgetFillStrategy(n_blocks=2, threshold_mb=0.0, enable_layer_de=False, enable_tensor_de=False, seed=0),
]


@pytest.mark.parametrize("planner", range(len(PLANNERS)))
def test_no_write_while_read(planner):
    rng = random.Random(planner)
    for trial in range(25):
        n = rng.randint(2, 9)
        stats = _profile(rng, n)
        total = sum(t.size_bytes for l in stats for t in l.tensors)
        mem = {1 << 20: 0.05, 1 << 30: 50.0}
        strat = PLANNERS[planner]()
        try:
            budget = int(total * rng.uniform(0.3, 0.9)) if isinstance(strat, BudgetFillStrategy) else None
            result = strat.compute(stats, mem, budget)
        except Exception as e:  # noqa: BLE001 - a planner may refuse an impossible budget
            if "budget" in str(e).lower() or "unreachable" in str(e).lower():
                continue
            raise
        _simulate(stats, result)
