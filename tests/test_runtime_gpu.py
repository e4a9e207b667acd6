"""The streaming runtime on a GPU: native transfer engine, slot views, graphs, timing."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("CUDA device required", allow_module_level=True)

import flextensor_b200 as ft  # noqa: E402
from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402
from flextensor_b200.planner import NthLayerStrategy  # noqa: E402

DEV = torch.device("cuda", 0)


def tiny(impl="fused", layers=4):
    cfg = tiny_config(num_layers=layers)
    torch.manual_seed(0)
    m = WanDiT(cfg, impl=impl).to(torch.bfloat16)
    init_wan_params_(m, seed=0)
    lat = torch.randn(1, cfg.in_channels, 2, 16, 16, device=DEV, dtype=torch.bfloat16)
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=DEV, dtype=torch.bfloat16)
    ts = torch.tensor([321.0], device=DEV)
    return m, (lat, ts, ctx)


def cfg(**kw):
    base = dict(include_patterns=["blocks.*"], skip_discovery=True, profiling_iters=1, num_blocks=2, min_blocks=2,
                load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    base.update(kw)
    return ft.OffloadConfig(**base)


def test_streamed_equals_resident_bitwise():
    m, inp = tiny()
    ref_m, _ = tiny()
    ref_m = ref_m.to(DEV)
    with torch.no_grad():
        want = ref_m(*inp)
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg())
    with torch.no_grad():
        for _ in range(4):
            assert torch.equal(mm(*inp), want)
    tm = om.get_tensor_manager()
    assert type(tm.loader.engine).__name__ == "NativeTransferEngine"
    assert native.device_error(reset=True) == 0


@pytest.mark.parametrize("mode", ["torch", "host_register"])
def test_pinning_modes(mode):
    m, inp = tiny(layers=2)
    ref = tiny(layers=2)[0].to(DEV)
    with torch.no_grad():
        want = ref(*inp)
    mm = ft.offload(m, cfg(pinned_memory_mode=mode))
    with torch.no_grad():
        for _ in range(3):
            assert torch.equal(mm(*inp), want)
    blocks = ft.get_offload_manager().get_tensor_manager().loader.plan.host_blocks.values()
    assert all(b.data.is_pinned() for b in blocks)


def test_cuda_graph_capture_of_streamed_forward():
    m, inp = tiny()
    ref = tiny()[0].to(DEV)
    with torch.no_grad():
        want = ref(*inp)
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg())
    with torch.no_grad():
        for _ in range(3):
            mm(*inp)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g):
                out = mm(*inp)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)


def test_offload_timing_reports_hidden_fraction():
    m, inp = tiny()
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg(offload_timing="eager"))
    with torch.no_grad():
        for _ in range(5):
            mm(*inp)
    rep = ft.collect_offload_timing()
    assert rep is not None and rep.num_passes >= 3 and rep.per_trap
    assert 0.0 <= rep.hidden_fraction <= 1.0
    assert rep.total_transfer_sum > 0
    print(ft.format_offload_timing_table(rep))


def test_memory_budget_mode_plans_under_budget():
    m, inp = tiny(layers=6)
    total = sum(p.numel() * p.element_size() for p in m.parameters())
    frac = 0.5 * total / torch.cuda.get_device_properties(0).total_memory
    om = ft.get_offload_manager()
    mm = om.offload(m, ft.OffloadConfig(include_patterns=["blocks.*"], skip_discovery=True, profiling_iters=2,
                                        num_blocks=2, min_blocks=2, max_gpu_mem_fraction=frac,
                                        load_strategy=ft.BudgetFillStrategy(n_blocks=2, enable_tensor_de=False,
                                                                            seed=0, epoch=5)))
    with torch.no_grad():
        for _ in range(4):
            mm(*inp)
    assert om.phase.value == "inference"


def test_state_adoption_into_gpu_loaded_model():
    """A saved plan adopted into a model that already sits on the GPU (serving-engine path):
    only the streamed storages move to the host, in a capacity-checked order."""
    m, inp = tiny()
    with torch.no_grad():
        want = tiny()[0].to(DEV)(*inp)
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg())
    with torch.no_grad():
        for _ in range(om.iters_before_inference):
            mm(*inp)
    state = om.get_tensor_manager().export_state()
    ft.release()
    streamed = {s.name for v in state.load_strategy.values() for s in v}

    fresh = tiny()[0].to(DEV)
    tm_plan = ft.get_offload_manager("adopt")
    mm2 = tm_plan.offload_from_state(fresh, state, cfg(), adopt=True)
    assert tm_plan.phase.value == "inference"
    with torch.no_grad():
        for _ in range(3):
            assert torch.equal(mm2(*inp), want)
    host = tm_plan.get_tensor_manager().host
    names = tm_plan.get_tensor_manager().id_to_name
    assert {names[t] for t in host} == streamed
    tm = tm_plan.get_tensor_manager()
    assert all(p.device == DEV for t, p in tm.params_by_tid.items() if names[t] not in streamed)
    ft.release("adopt")


@pytest.mark.parametrize("hold", [True, False])
def test_device_start_model_keeps_one_host_copy(hold):
    """A model that starts on the GPU: after planning, every streamed weight's host bytes are its
    view in the packed pinned arena (no per-tensor host copy stays alive beside it)."""
    m, inp = tiny()
    m = m.to(DEV)
    with torch.no_grad():
        want = tiny()[0].to(DEV)(*inp)
    om = ft.get_offload_manager()
    mm = om.offload(m, cfg(hold_device_weights=hold))
    with torch.no_grad():
        for _ in range(4):
            assert torch.equal(mm(*inp), want)
    tm = om.get_tensor_manager()
    spans = [(b.data.data_ptr(), b.data.data_ptr() + b.data.numel()) for b in tm.loader.plan.host_blocks.values()]
    assert tm.host
    for h in tm.host.values():
        assert h.device.type == "cpu" and h.is_pinned()
        assert any(lo <= h.data_ptr() < hi for lo, hi in spans)
    assert not tm._held_ptr_to_tid
    ft.release()


class _PeerBlock(torch.nn.Module):
    def __init__(self, d):
        super().__init__()
        self.lin = torch.nn.Linear(d, d, bias=False)
        self._peer = []          # another block whose weight this one also reads (not registered)

    def forward(self, x):
        y = self.lin(x)
        for p in self._peer:
            y = y + torch.nn.functional.linear(x, p.lin.weight)
        return y


class _PeerNet(torch.nn.Module):
    def __init__(self, d=256, n=4):
        super().__init__()
        self.blocks = torch.nn.ModuleList([_PeerBlock(d) for _ in range(n)])
        self.blocks[2]._peer.append(self.blocks[0])

    def forward(self, x):
        for b in self.blocks:
            x = torch.tanh(b(x))
        return x


def test_discovery_finds_cross_unit_read_of_a_device_held_weight():
    torch.manual_seed(0)
    m = _PeerNet().to(DEV)
    x = torch.randn(8, 256, device=DEV)
    with torch.no_grad():
        want = m(x).clone()
    om = ft.get_offload_manager()
    mm = om.offload(m, ft.OffloadConfig(include_patterns=["blocks.*"], discovery_iters=1, profiling_iters=1,
                                        num_blocks=2, min_blocks=2,
                                        load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2,
                                                                       cyclic=True)))
    with torch.no_grad():
        for _ in range(4):
            torch.testing.assert_close(mm(x), want, rtol=0, atol=0)
    tm = om.get_tensor_manager()
    shared = tm.name_to_id["blocks.0.lin.weight"]
    assert shared in tm.resident and shared not in tm.host
    ft.release()


def test_exact_size_pinned_arena():
    """Large pinned host buffers come from one exact-size page-locked allocation (no power-of-two
    rounding) that supports asynchronous copies both ways and is freed with its last view."""
    from flextensor_b200.core.host_store import EXACT_PIN_MIN, alloc_host_bytes

    n = EXACT_PIN_MIN + 4096 * 3
    h = alloc_host_bytes(n, pinned=True)
    assert h.numel() == n and h.is_pinned() and h.dtype == torch.uint8
    src = torch.randint(0, 255, (n,), dtype=torch.uint8, device=DEV)
    v = h[4096:]
    v.copy_(src[4096:], non_blocking=True)
    back = torch.empty_like(src)
    back[4096:].copy_(v, non_blocking=True)
    torch.cuda.synchronize()
    assert torch.equal(back[4096:], src[4096:])
    del h, v
    small = alloc_host_bytes(1024, pinned=True)
    assert small.is_pinned() and small.numel() == 1024
