"""Transfer windows, plan rewrites, profiling-quality checks and the piecewise prefetch policy."""

import logging

import pytest

from flextensor_b200.core.stats import IterativeLayerStatisticsCollector, LayerStatistics, TensorStatistics
from flextensor_b200.planner.interpolator import MemoryTransferInterpolator
from flextensor_b200.planner.operations import (
    create_allocation_ordered,
    find_transfers_for_preload,
    rearrange_transfers,
    remove_layers_compound,
)
from flextensor_b200.planner.windows import GapAwareWindow, SingleLayerWindow
from flextensor_b200.runtime.prefetch_policy import PiecewisePrefetchPolicy, PiecewisePrefetchPolicyError
from flextensor_b200.runtime.profiling_quality import LayerStatisticsAnalyzer, report_profiling_quality


def _layers(durs, mb=1.0):
    out = []
    for i, d in enumerate(durs):
        t = TensorStatistics(tensor_id=i, name=f"l{i}.w", size_bytes=int(mb * 1e6), load_time_ms=1.0)
        out.append(LayerStatistics(label=f"l{i}", tensors=[t], duration=d))
    return out


def test_windows():
    ls = _layers([1, 2, 3, 4])
    assert SingleLayerWindow().compute_window(ls, 2) == 2
    assert SingleLayerWindow().compute_window(ls, 0) == 4  # wraps to the last trap
    plan = {"l0": ls[1].tensors}  # l0 issues a transfer; l1 does not
    assert GapAwareWindow().compute_window(ls, 3, plan) == 3 + 2  # l2 + l1, stops before l0 (busy)
    assert GapAwareWindow(cyclic=False).compute_window(ls, 1, {}) == 1


def test_preload_and_allocation_order():
    order = ["a", "b", "c"]
    assert find_transfers_for_preload(order, {"a": "b", "c": "a"}) == ["c"]
    assert create_allocation_ordered(order, {"c": 0, "a": 0, "b": 1}) == {0: ["a", "c"], 1: ["b"]}


def test_remove_and_merge():
    ls = _layers([1, 2, 3, 4])
    out = remove_layers_compound(ls, [{"op": "remove", "labels": ["l1"]}])
    assert [l.label for l in out] == ["l0", "l2", "l3"] and out[0].duration == 3 and len(out[1].tensors) == 1
    out = remove_layers_compound(ls, [{"op": "merge", "labels": ["l2", "l3"]}])
    assert [l.label for l in out] == ["l0", "l1", "l2"] and out[2].duration == 7
    with pytest.raises(ValueError):
        remove_layers_compound(ls, [{"op": "merge", "labels": ["l0", "l2"]}])


def test_rearrange_moves_to_hide_copy():
    # l3's tensors take 5 ms to copy; l2 alone (1 ms) cannot hide it, l1+l2 (1+10) can.
    ls = _layers([1, 10, 1, 1])
    interp = MemoryTransferInterpolator({1 << 20: 5.0, 1 << 22: 20.0})
    plan = {"l2": ls[3].tensors}
    new_plan, new_t2c = rearrange_transfers(plan, {"l2": "l3"}, ls, interp)
    assert new_t2c == {"l1": "l3"} and new_plan["l1"] == ls[3].tensors
    # already hidden: unchanged
    ls2 = _layers([1, 1, 10, 1])
    assert rearrange_transfers(plan, {"l2": "l3"}, ls2, interp)[1] == {"l2": "l3"}


def test_profiling_quality_and_untimed(caplog):
    col = IterativeLayerStatisticsCollector()
    col.record_tensors("a", [1])
    col.record_tensors("b", [2])
    col.record_tensors("c", [3])
    for d in (1.0, 1.0, 1.0):
        col.record_duration("a", d)
    col.record_duration("b", 1.0)
    col.record_duration("b", 3.0)
    an = LayerStatisticsAnalyzer(col)
    assert an.get_layer_statistics("a").coefficient_of_variation == 0
    assert an.get_layer_statistics("b").samples == 2
    with caplog.at_level(logging.WARNING, logger="flextensor_b200.diagnostics"):
        warns = report_profiling_quality(col)
    assert any("Low sample count" in w for w in warns)
    assert any("High duration variance" in w for w in warns)
    assert any("never timed" in w and "c" in w for w in warns)


def test_piecewise_policy():
    p = PiecewisePrefetchPolicy.from_mode("error")
    p.on_schedule("l0", "l1")
    p.on_wait("l1")
    assert p.on_piece_join() == []
    p.on_schedule("l1", "l3")
    with pytest.raises(PiecewisePrefetchPolicyError):
        p.on_piece_join()
    q = PiecewisePrefetchPolicy.from_mode("warn")
    q.on_schedule("l3", "l0")  # wrap-around prefetch for the next forward...
    q.on_wait("l0")            # ...whose consumer already ran in this pass
    q.on_schedule("l3", "l0")
    assert q.on_piece_join(at_last_layer=True) == []
    off = PiecewisePrefetchPolicy.from_mode("off")
    off.on_schedule("a", "b")
    assert off.on_piece_join() == []
    with pytest.raises(ValueError):
        PiecewisePrefetchPolicy.from_mode("loud")
