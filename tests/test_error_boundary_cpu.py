"""Error boundary: a failure inside a phase transition (here: the planner raising while the
inference plan is built) surfaces unchanged, is preceded by one diagnostic line (manager, phase,
iteration, host RSS), and leaves the manager releasable with the model's weights intact; a fresh
manager then works."""

import logging

import pytest
import torch
from torch import nn

import flextensor_b200 as ft
from flextensor_b200.planner import NthLayerStrategy


class _Boom:
    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None):
        raise RuntimeError("planner exploded")


def _model():
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(32, 64), nn.GELU(), nn.Linear(64, 32))


def test_planner_failure_is_logged_and_releasable(caplog):
    x = torch.randn(2, 32)
    conf = ft.OffloadConfig(pinned_memory=False, include_patterns=["0", "2"], profiling_iters=1, load_strategy=_Boom())
    om = ft.get_offload_manager("boom")
    m0 = _model()
    want0 = m0(x).detach().clone()
    mm = om.offload(m0, conf)
    with caplog.at_level(logging.ERROR):
        with pytest.raises(RuntimeError, match="planner exploded"):
            with torch.no_grad():
                for _ in range(om.iters_before_inference + 1):
                    mm(x)
    snaps = [r.getMessage() for r in caplog.records if "host_rss=" in r.getMessage()]
    assert snaps, "no diagnostic snapshot was logged"
    assert "manager='boom'" in snaps[-1] and "phase=" in snaps[-1] and "iteration=" in snaps[-1]
    ft.release("boom")
    with torch.no_grad():
        assert torch.equal(m0(x), want0)  # the released model still holds its weights

    om2 = ft.get_offload_manager("after_boom")
    conf2 = ft.OffloadConfig(pinned_memory=False, include_patterns=["0", "2"], profiling_iters=1, num_blocks=2,
                             min_blocks=2, load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    m = _model()
    want = m(x).detach().clone()
    mm2 = om2.offload(m, conf2)
    with torch.no_grad():
        for _ in range(om2.iters_before_inference + 1):
            got = mm2(x)
    assert torch.equal(got, want)
    ft.release("after_boom")


def test_failed_block_construction_leaves_the_model_intact(monkeypatch):
    """Packing copies every streamed tensor into the host arena before its parameter is pointed at
    the copy, so a failure later in the construction (here: the transfer engine) leaves every
    parameter holding its values; the released model computes what it computed before."""
    import flextensor_b200.runtime.tensor_manager as TM

    def no_engine(*a, **k):
        raise RuntimeError("engine construction failed")

    monkeypatch.setattr(TM, "make_engine", no_engine)
    x = torch.randn(2, 32)
    m = _model()
    want = m(x).detach().clone()
    conf = ft.OffloadConfig(pinned_memory=False, include_patterns=["0", "2"], profiling_iters=1, num_blocks=2,
                            min_blocks=2, load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    om = ft.get_offload_manager("noengine")
    mm = om.offload(m, conf)
    with pytest.raises(RuntimeError, match="engine construction failed"):
        with torch.no_grad():
            for _ in range(om.iters_before_inference + 1):
                mm(x)
    ft.release("noengine")
    with torch.no_grad():
        assert torch.equal(m(x), want)
