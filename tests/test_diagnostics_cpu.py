"""Plan diagnostics: the duration, transfer and plan tables logged when a plan is built with
``enable_diagnostics``, and the plan table's copy-window arithmetic."""

import logging
import types

import torch
from torch import nn

import flextensor_b200 as ft
from flextensor_b200.planner import NthLayerStrategy
from flextensor_b200.runtime.diagnostics import plan_rows, plan_table, transfer_table


def _ls(label, ms, nbytes):
    t = types.SimpleNamespace(size_bytes=nbytes)
    return types.SimpleNamespace(label=label, duration=ms, tensors=[t])


def test_copy_window_and_exposed_time():
    """Trap b's block is copied during a (window = a's compute); trap a's block is copied during c
    of the previous pass (window = c wraps to a: c only)."""
    layers = [_ls("a", 2.0, 1000), _ls("b", 3.0, 1000), _ls("c", 1.0, 1000)]
    plan = types.SimpleNamespace(transfer_slot={"b": 0, "a": 1}, t2c={"b": "a", "a": "c"}, slot_bytes={0: 1024, 1: 1024},
                                 host_blocks={})
    res = types.SimpleNamespace(strategy_map={"a": [types.SimpleNamespace(size_bytes=1000)],
                                              "b": [types.SimpleNamespace(size_bytes=1000)]})
    tm = types.SimpleNamespace(layer_stats=layers, loader=types.SimpleNamespace(plan=plan), strategy_result=res,
                               memory_stats={1000: 1.5, 2000: 3.0}, unmapped_bytes=1000, strategy=None)
    rows, tot = plan_rows(tm)
    by = {r["label"]: r for r in rows}
    assert by["b"]["window_ms"] == 2.0 and abs(by["b"]["copy_ms"] - 1.5) < 1e-6 and by["b"]["exposed_ms"] == 0.0
    assert by["a"]["window_ms"] == 1.0 and abs(by["a"]["exposed_ms"] - 0.5) < 1e-6
    assert by["c"]["streamed"] == 0 and by["c"]["exposed_ms"] == 0.0
    assert abs(tot["hidden_pct"] - 100.0 * (1 - 0.5 / 3.0)) < 1e-6
    assert tot["slot_users"] == {0: ["b"], 1: ["a"]}
    text = plan_table(tm)
    assert "slot 0" in text and "hidden" in text


def test_transfer_table_bandwidth():
    t = transfer_table({1 << 20: 0.5})
    assert "2.10" in t  # 1 MiB in 0.5 ms = 2.10 GB/s
    assert transfer_table(None) == "(no transfer benchmark)"


def test_tables_logged_when_a_plan_is_built(caplog):
    torch.manual_seed(0)
    m = nn.Sequential(nn.Linear(64, 256), nn.GELU(), nn.Linear(256, 64))
    x = torch.randn(4, 64)
    conf = ft.OffloadConfig(pinned_memory=False, include_patterns=["0", "2"], profiling_iters=2, num_blocks=2,
                            min_blocks=2, enable_diagnostics=True,
                            load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    om = ft.get_offload_manager("diag")
    mm = om.offload(m, conf)
    with caplog.at_level(logging.INFO, logger="flextensor_b200.diagnostics"):
        for _ in range(om.iters_before_inference + 1):
            with torch.no_grad():
                mm(x)
    text = "\n".join(r.getMessage() for r in caplog.records if r.name == "flextensor_b200.diagnostics")
    assert "per-trap durations" in text and "transfer benchmark" in text and "offload plan" in text
    assert "slot 0" in text
    ft.release("diag")


def test_restored_plan_logs_its_durations(tmp_path, caplog):
    torch.manual_seed(0)
    conf = ft.OffloadConfig(pinned_memory=False, include_patterns=["0", "2"], profiling_iters=2, num_blocks=2,
                            min_blocks=2, enable_diagnostics=True,
                            load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))

    def build():
        torch.manual_seed(0)
        return nn.Sequential(nn.Linear(64, 256), nn.GELU(), nn.Linear(256, 64))

    x = torch.randn(4, 64)
    om = ft.get_offload_manager("diag_save")
    mm = om.offload(build(), conf)
    with torch.no_grad():
        for _ in range(om.iters_before_inference + 1):
            mm(x)
    ft.save_profile(str(tmp_path), name="diag_save")
    ft.release("diag_save")
    with caplog.at_level(logging.INFO, logger="flextensor_b200.diagnostics"):
        mm2 = ft.offload_from_profile(build(), str(tmp_path), config=conf, name="diag_load")
        with torch.no_grad():
            mm2(x)
    text = "\n".join(r.getMessage() for r in caplog.records if r.name == "flextensor_b200.diagnostics")
    assert "trap durations" in text and "offload plan" in text
    ft.release("diag_load")
