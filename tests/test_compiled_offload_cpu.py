"""Compiled-offload lifecycle on the CPU device: compiled view-profile (compile at PROFILING, an
unmeasured compile warm-up, then measured compiled forwards), eager profile + compiled inference
with the automatic warm -> measure -> replan tail, transfer-mode validation, dynamo limit bumps,
and a real ``torch.compile`` per unit over many identical blocks."""

import pytest
import torch
from torch import nn

import flextensor_b200 as ft
from flextensor_b200.planner import NthLayerStrategy
from flextensor_b200.runtime import compiled as co


class Block(nn.Module):
    def __init__(self, d=64):
        super().__init__()
        self.fc = nn.Linear(d, d)

    def forward(self, x):
        return torch.tanh(self.fc(x)) + x


class Net(nn.Module):
    def __init__(self, n=4, d=64):
        super().__init__()
        self.blocks = nn.ModuleList([Block(d) for _ in range(n)])

    def forward(self, x):
        for b in self.blocks:
            x = b(x)
        return x


def cfg(**kw):
    base = dict(pinned_memory=False, include_patterns=["blocks.*"], profiling_iters=2, num_blocks=2, min_blocks=2,
                load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    base.update(kw)
    return ft.OffloadConfig(**base)


class CountingCompiler:
    """A compile_fn that records which units it compiled and how often they ran."""

    def __init__(self):
        self.compiled = 0
        self.calls = 0

    def __call__(self, core):
        self.compiled += 1
        outer = self

        class Wrapped(nn.Module):
            def __init__(self):
                super().__init__()
                self.core = core

            def forward(self, *a, **k):
                outer.calls += 1
                return self.core(*a, **k)

        return Wrapped()


def _run(mm, x, n):
    with torch.no_grad():
        return [mm(x) for _ in range(n)]


def test_compiled_view_profile_measures_compiled_forwards():
    torch.manual_seed(0)
    net, x = Net(), torch.randn(4, 64)
    ref = net(x).detach()
    om = ft.get_offload_manager("cv")
    comp = CountingCompiler()
    mm = om.offload(net, cfg(), compile_fn=comp)
    assert om._compiled_offload.mode == "view_profile"
    n = om.iters_before_inference
    assert n == 1 + 2 + co.PROFILE_COMPILE_WARMUP_FORWARDS  # discovery + profiling + compile warm-up
    _run(mm, x, 1)  # discovery: not compiled yet
    assert comp.compiled == 4 and str(om.phase).endswith("PROFILING")
    outs = _run(mm, x, n - 1)
    assert str(om.phase).endswith("INFERENCE")
    assert comp.calls == 4 * (n - 1)  # every profiling forward ran the compiled units
    # only the measured forwards' durations were kept
    stats = om.get_tensor_manager().collector
    assert all(len(v) == 2 for v in stats.all_samples().values())
    for y in outs + _run(mm, x, 3):
        assert torch.allclose(y, ref, atol=1e-6)
    om.release()


def test_eager_profile_compiled_inference_arms_replan_tail():
    torch.manual_seed(1)
    net, x = Net(), torch.randn(4, 64)
    ref = net(x).detach()
    om = ft.get_offload_manager("ct")
    comp = CountingCompiler()
    mm = om.offload(net, cfg(profile_mode="getter"), compile_fn=comp)
    assert om._compiled_offload.mode == "inference_tail"
    _run(mm, x, om.iters_before_inference)
    assert comp.compiled == 4
    st = om.strategy_replan_status
    assert st.state == "in_progress"
    outs = _run(mm, x, co.COMPILED_WARMUP_FORWARDS + 2)
    st = om.strategy_replan_status
    assert st.state == "done" and st.applied is not None
    for y in outs + _run(mm, x, 2):
        assert torch.allclose(y, ref, atol=1e-6)
    om.release()


def test_strategy_transfer_mode_rejected_with_compile_fn():
    om = ft.get_offload_manager("cbad")
    with pytest.raises(ValueError, match="block transfer_mode"):
        om.offload(Net(), cfg(transfer_mode="strategy"), compile_fn=lambda m: m)
    assert om._compiled_offload.mode == "off"


def test_dynamo_limits_raised_and_restored():
    import torch._dynamo.config as dcfg

    key = "recompile_limit" if hasattr(dcfg, "recompile_limit") else "cache_size_limit"
    before = getattr(dcfg, key)
    old = co.bump_dynamo_limits(40)
    assert getattr(dcfg, key) >= 160
    co.restore_dynamo_limits(old)
    assert getattr(dcfg, key) == before


def test_torch_compile_per_unit_over_many_identical_blocks():
    """20 blocks share one forward code object: each gets its own compiled entry (no silent
    eager fallback past dynamo's default limit of 8), outputs unchanged."""
    import torch._dynamo

    torch._dynamo.reset()
    torch.manual_seed(2)
    net, x = Net(n=20, d=32), torch.randn(2, 32)
    ref = net(x).detach()
    om = ft.get_offload_manager("ctc")
    mm = om.offload(net, cfg(include_patterns=["blocks.*"]),
                    compile_fn=lambda m: torch.compile(m, backend="eager", dynamic=False))
    outs = _run(mm, x, om.iters_before_inference + 2)
    for y in outs:
        assert torch.allclose(y, ref, atol=1e-5)
    om.release()
    torch._dynamo.reset()
