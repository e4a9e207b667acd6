"""CPU plumbing configuration (BASELINE config #1) and runtime lifecycle on the CPU device."""

import uuid

import pytest
import torch
from torch import nn

import flextensor_b200 as ft
from flextensor_b200.planner import NthLayerStrategy


class MLP(nn.Module):
    """4-layer MLP: Linear 256->1024, GELU, Linear 1024->256 (two Linear layers to offload)."""

    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(256, 1024)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(1024, 256)

    def forward(self, x):
        return self.fc2(self.act(self.fc1(x)))


def make():
    torch.manual_seed(0)
    m = MLP()
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0.0, 0.02)
    x = torch.randn(8, 256)
    return m, x


def cfg(**kw):
    base = dict(pinned_memory=False, include_patterns=["fc1", "fc2"], profiling_iters=2, num_blocks=2, min_blocks=2,
                load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    base.update(kw)
    return ft.OffloadConfig(**base)


@pytest.mark.parametrize("shm", [False, True])
def test_plumbing_bitwise(shm, tmp_path):
    m, x = make()
    ref = m(x).detach().clone()
    kw = dict(shm_enabled=True, shm_namespace=f"fttest{uuid.uuid4().hex[:8]}") if shm else {}
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg(**kw))
    assert om.iters_before_inference == 3
    for i in range(6):
        with torch.no_grad():
            y = mm(x)
        assert torch.equal(y, ref), f"forward {i} ({om.phase}) differs"
    assert om.phase.value == "inference"
    tm = om.get_tensor_manager()
    assert set(tm.strategy_result.strategy_map) == {"fc1", "fc2"}  # both layers stream through the ring
    usage = ft.get_gpu_memory_usage()
    assert usage.blocks_bytes > 0 and usage.unmapped_tensors_bytes == 0
    if shm:
        assert tm.shm_store is not None and len(tm.shm_store.segments) == 2
        names = [sg.path for sg in tm.shm_store.segments.values()]
    ft.release()
    if shm:
        import os

        assert not any(os.path.exists(n) for n in names)
    assert torch.equal(m(x), ref)


def test_profile_roundtrip(tmp_path):
    m, x = make()
    ref = m(x).detach().clone()
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg())
    for _ in range(om.iters_before_inference):
        mm(x)
    om.save_profile(str(tmp_path))
    st = ft.TensorManagerState.load_from_file(tmp_path / "profile.json")
    assert st.loader_type == "allocation_block_transfer" and set(st.load_strategy) == {"fc1", "fc2"}
    ft.release()
    m2, _ = make()
    mm2 = ft.offload_from_profile(m2, str(tmp_path), config=cfg())
    assert ft.get_offload_manager().phase.value == "inference"
    with torch.no_grad():
        assert torch.equal(mm2(x), ref)


def test_latency_mode_adaptive_default():
    m, x = make()
    ref = m(x).detach().clone()
    mm = ft.offload(m, ft.OffloadConfig(pinned_memory=False, include_patterns=["fc1", "fc2"], profiling_iters=2,
                                        num_blocks=2, min_blocks=2))
    for _ in range(5):
        with torch.no_grad():
            assert torch.equal(mm(x), ref)


def test_strategy_loader_mode():
    m, x = make()
    ref = m(x).detach().clone()
    mm = ft.offload(m, cfg(transfer_mode="strategy"))
    for _ in range(5):
        with torch.no_grad():
            assert torch.equal(mm(x), ref)


def test_skip_discovery_and_phases():
    m, x = make()
    om = ft.get_offload_manager()
    om.offload(m, cfg(skip_discovery=True, profiling_iters=1))
    assert om.skip_discovery_honored and om.phase.value == "profiling" and om.iters_before_inference == 1
    m(x)
    assert om.phase.value == "inference"
    with pytest.raises(RuntimeError):
        om.set_config(cfg(skip_discovery=False))


def test_suspend_profiling_freezes_counter():
    m, x = make()
    om = ft.get_offload_manager()
    om.offload(m, cfg(skip_discovery=True, profiling_iters=2))
    om.suspend_profiling()
    for _ in range(3):
        m(x)
    assert om.phase.value == "profiling"
    om.resume_profiling()
    m(x)
    m(x)
    assert om.phase.value == "inference"


def test_nested_traps_rejected():
    om = ft.get_offload_manager()
    om.init(cfg())
    with om.offload_block("a"):
        with pytest.raises(RuntimeError, match="nested"):
            with om.offload_block("b"):
                pass


def test_abort_recovery():
    m, x = make()
    ref = m(x).detach().clone()
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg())
    for _ in range(om.iters_before_inference):
        mm(x)
    orig = m.fc2.forward

    def boom(*a, **k):
        raise RuntimeError("injected")

    m.fc2.forward = boom
    with pytest.raises(RuntimeError, match="injected"):
        mm(x)
    m.fc2.forward = orig
    with torch.no_grad():
        assert torch.equal(mm(x), ref)


def test_units_and_release_restore():
    m, x = make()
    om = ft.get_offload_manager()
    om.offload(m, cfg())
    assert [n for n, _ in ft.offload_units()] == ["fc1", "fc2"]
    ft.release(preserve_model=True)
    assert "forward" not in m.fc1.__dict__
    assert m.fc1.weight.device.type == "cpu"


def test_disabled_preloads():
    m, x = make()
    ref = m(x).detach().clone()
    mm = ft.offload(m, cfg(enabled=False))
    assert torch.equal(mm(x), ref)


def test_custom_ops_external_compile_path():
    from flextensor_b200.runtime import custom_ops  # noqa: F401  (registers the ops)

    m, x = make()
    ref = m(x).detach().clone()
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg(external_compile=True))
    for _ in range(om.iters_before_inference):
        mm(x)
    assert om.phase.value == "inference"
    for _ in range(3):
        with torch.no_grad():
            assert torch.equal(mm(x), ref)
    # the boundary ops are registered with a fake impl (traceable by dynamo / opcheck)
    t = torch.zeros(1)
    torch.library.opcheck(torch.ops.flextensor_b200.pre_compute.default, (t, "nope", 0),
                          test_utils=("test_schema", "test_faketensor"))


def test_strategy_replan_tail():
    from flextensor_b200.runtime.manager import StrategyReplanStatus

    m, x = make()
    ref = m(x).detach().clone()
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg())
    with torch.no_grad():
        for _ in range(om.iters_before_inference):
            mm(x)
    assert om.strategy_replan_status == StrategyReplanStatus("idle", True, None)
    n = om.request_strategy_replan(warmup_forwards=1, measure_forwards=2)
    assert n == 3 and om.strategy_replan_status.state == "in_progress"
    with pytest.raises(RuntimeError):
        om.request_strategy_replan()
    with torch.no_grad():
        for i in range(n):
            y = mm(x)
            assert torch.equal(y, ref)
    st = om.strategy_replan_status
    assert st.state == "done" and st.can_request and st.applied is True
    with torch.no_grad():
        assert torch.equal(mm(x), ref)  # rebuilt loader still streams correctly


def test_plain_tensor_attributes_follow_the_model():
    class WithTable(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = nn.Linear(8, 8)
            self.table = torch.arange(8.0)          # plain attribute, not a buffer
            self.pair = (torch.ones(8), torch.zeros(8))

        def forward(self, x):
            return self.fc(x) + self.table + self.pair[0]

    torch.manual_seed(0)
    m = WithTable()
    x = torch.randn(2, 8)
    ref = m(x).detach()
    mm = ft.offload(m, ft.OffloadConfig(pinned_memory=False, include_patterns=["fc"], profiling_iters=1,
                                        num_blocks=2, min_blocks=2,
                                        load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True)))
    with torch.no_grad():
        for _ in range(4):
            assert torch.allclose(mm(x), ref)
