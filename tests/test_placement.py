"""Placement snapshots, capacity-safe transition ordering and plan adoption targets (CPU)."""

import pytest
import torch
from torch import nn

import flextensor_b200 as ft
from flextensor_b200.core.placement import (
    HostAllocation,
    MemoryCapacity,
    ModelPlacementState,
    StorageState,
    TensorState,
    TransitionSpec,
    capture_model_state,
    plan_state_transition,
    target_from_profile,
)
from flextensor_b200.planner import NthLayerStrategy


class Tied(nn.Module):
    def __init__(self):
        super().__init__()
        self.emb = nn.Embedding(16, 8)
        self.head = nn.Linear(8, 16, bias=False)
        self.head.weight = self.emb.weight  # two names, one storage
        self.register_buffer("scale", torch.ones(8))
        self.extra = torch.zeros(3)  # plain attribute: reachable, unregistered


def test_capture_aliases_buffers_and_roundtrip():
    st = capture_model_state(Tied())
    by_name = {n: t for t in st.tensors for n in t.names}
    assert by_name["emb.weight"] is by_name["head.weight"]
    assert by_name["scale"].kind == "buffer"
    assert any(t.kind == "tensor" and t.names == () for t in st.tensors)
    assert len(st.storages) == 3
    assert ModelPlacementState.from_dict(st.to_dict()) == st


def test_from_dict_rejects_bad_input():
    good = capture_model_state(Tied()).to_dict()
    with pytest.raises(ValueError, match="version"):
        ModelPlacementState.from_dict({**good, "version": 2})
    bad = {**good, "storages": good["storages"][1:]}
    with pytest.raises(ValueError, match="exactly match"):
        ModelPlacementState.from_dict(bad)
    pinned_gpu = {**good, "storages": [{**good["storages"][0], "device": "cuda:0", "pinned": True}]
                  + good["storages"][1:]}
    with pytest.raises(ValueError, match="cannot be pinned"):
        ModelPlacementState.from_dict(pinned_gpu)


def _state(placements):
    ts = tuple(TensorState(f"t{i}", (f"w{i}",), f"s{i}", n, "parameter") for i, (n, _) in enumerate(placements))
    ss = tuple(StorageState(f"s{i}", d, n, False) for i, (n, d) in enumerate(placements))
    return ModelPlacementState(ts, ss)


def test_ordering_frees_gpu_before_promoting():
    # GPU holds a (100) and b (100); target swaps them with host c (150). GPU headroom 60:
    # promotions only fit after a demotion freed room.
    cur = _state([(100, "cuda:0"), (100, "cuda:0"), (150, "cpu")])
    tgt = _state([(100, "cpu"), (100, "cpu"), (150, "cuda:0")])
    plan = plan_state_transition(cur, tgt, transition=TransitionSpec(), capacity=MemoryCapacity(1000, 60))
    kinds = [m.destination_device for m in plan.migrations]
    assert kinds.index("cuda:0") > kinds.index("cpu")
    assert plan.peak_gpu_bytes <= 60 and plan.peak_host_bytes <= 1000


def test_ordering_infeasible_raises():
    cur = _state([(100, "cpu")])
    tgt = _state([(100, "cuda:0")])
    with pytest.raises(RuntimeError, match="Insufficient capacity"):
        plan_state_transition(cur, tgt, transition=TransitionSpec(), capacity=MemoryCapacity(0, 50))


def test_loader_extra_and_host_allocations_counted():
    cur = _state([(100, "cuda:0")])
    tgt = _state([(100, "cpu")])
    spec = TransitionSpec(extra_gpu_bytes=30, host_allocations=(HostAllocation(100, 100),),
                          release_host_storage_ids=("s0",))
    plan = plan_state_transition(cur, tgt, transition=spec, capacity=MemoryCapacity(300, 30))
    assert plan.peak_host_bytes == 300 and plan.peak_gpu_bytes == 0  # the demotion freed 100 first
    with pytest.raises(RuntimeError):
        plan_state_transition(cur, tgt, transition=spec, capacity=MemoryCapacity(299, 30))


def test_cross_gpu_and_unpin_rejected():
    cur = _state([(10, "cuda:0")])
    with pytest.raises(ValueError, match="Cross-device"):
        plan_state_transition(cur, _state([(10, "cuda:1")]), transition=TransitionSpec(),
                              capacity=MemoryCapacity(100, 100))


class MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(64, 128)
        self.fc2 = nn.Linear(128, 64)

    def forward(self, x):
        return self.fc2(torch.relu(self.fc1(x)))


def test_target_from_saved_plan():
    torch.manual_seed(0)
    m, x = MLP(), torch.randn(4, 64)
    om = ft.get_offload_manager()
    cfg = ft.OffloadConfig(pinned_memory=False, include_patterns=["fc1", "fc2"], profiling_iters=1, num_blocks=2,
                           min_blocks=2, load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2))
    mm = om.offload(m, cfg)
    for _ in range(om.iters_before_inference):
        mm(x)
    state = om.get_tensor_manager().export_state()
    ft.release()
    streamed = {s.name for v in state.load_strategy.values() for s in v}
    assert streamed, "the plan streams something"
    fresh = MLP()
    cur = capture_model_state(fresh)
    target, spec = target_from_profile(cur, state, target_device="cuda:0", pinning="copy", use_shm=False)
    dev_of = {n: s.device for t in target.tensors for n in t.names for s in target.storages if s.id == t.storage_id}
    for n in dev_of:
        assert dev_of[n] == ("cpu" if n in streamed else "cuda:0"), n
    assert spec.extra_gpu_bytes > 0
    assert set(spec.release_host_storage_ids) == {t.storage_id for t in target.tensors if set(t.names) & streamed}
    plan = plan_state_transition(cur, target, transition=spec, capacity=MemoryCapacity(1 << 30, 1 << 30))
    assert {m.destination_device for m in plan.migrations} == {"cuda:0"}  # non-streamed params move up
