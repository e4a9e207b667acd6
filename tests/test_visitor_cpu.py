"""The generic tensor visitor: nested containers, plain objects, tensor inner fields, Parameter
preservation, shared tensors, cycles, compiled-module unwrapping, custom handlers; and the
offload runtime keeping a quantized-style weight's metadata."""

import collections

import torch
from torch import nn

import flextensor_b200 as ft
from flextensor_b200.core.visitor import TensorVisitor, carry_inner_fields, iter_tensors
from flextensor_b200.planner import NthLayerStrategy

Pair = collections.namedtuple("Pair", "a b")


class Holder:
    def __init__(self, t):
        self.t = t
        self.me = self  # cycle


class Deep(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc = nn.Linear(4, 4)
        self.shared = torch.ones(4)
        self.nested = {"x": [torch.zeros(4), (torch.full((4,), 2.0), {"deep": self.shared})]}
        self.od = collections.OrderedDict(k=torch.full((4,), 3.0))
        self.pair = Pair(torch.full((4,), 4.0), 7)
        self.bag = {torch.full((4,), 5.0)}
        self.obj = Holder(torch.full((4,), 6.0))
        self.loop = []
        self.loop.append(self.loop)  # self-referential list


def _tag(t):
    return t.double()


def test_every_nested_tensor_is_mapped_once():
    m = Deep()
    TensorVisitor(_tag).apply(m)
    assert m.shared.dtype == torch.float64
    assert m.nested["x"][0].dtype == torch.float64
    assert m.nested["x"][1][0].dtype == torch.float64
    assert m.nested["x"][1][1]["deep"] is m.shared  # shared tensor: one mapped copy everywhere
    assert isinstance(m.od, collections.OrderedDict) and m.od["k"].dtype == torch.float64
    assert isinstance(m.pair, Pair) and m.pair.a.dtype == torch.float64 and m.pair.b == 7
    assert next(iter(m.bag)).dtype == torch.float64
    assert m.obj.t.dtype == torch.float64 and m.obj.me is m.obj
    assert m.fc.weight.dtype == torch.float32  # registered parameters not requested


def test_unchanged_containers_keep_identity():
    m = Deep()
    before = (m.nested, m.od, m.pair, m.bag)
    TensorVisitor(lambda t: t).apply(m)
    assert (m.nested, m.od, m.pair, m.bag) == before
    assert m.nested is before[0] and m.pair is before[2]


def test_parameters_keep_object_and_inner_fields():
    lin = nn.Linear(4, 4)
    w = lin.weight
    w.weight_scale = torch.full((4,), 0.5)
    w.weight_loader = "loader-fn"
    w.output_dim = 0
    TensorVisitor(_tag, params=True, attributes=False).apply(lin)
    assert lin.weight is w and w.dtype == torch.float64
    assert w.weight_scale.dtype == torch.float64  # inner tensor field mapped with its parent
    assert w.weight_loader == "loader-fn" and w.output_dim == 0


def test_replaced_parameter_attribute_stays_a_parameter_with_metadata():
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.extra = [nn.Parameter(torch.ones(3), requires_grad=False)]
            self.extra[0].tag = "keep"

    m = M()
    TensorVisitor(_tag).apply(m)
    p = m.extra[0]
    assert isinstance(p, nn.Parameter) and p.dtype == torch.float64 and not p.requires_grad
    assert p.tag == "keep"


def test_read_only_walk_and_iteration():
    m = Deep()
    ts = iter_tensors(m)
    ids = {id(t) for t in ts}
    assert id(m.shared) in ids and id(m.obj.t) in ids and id(m.fc.weight) in ids
    before = m.nested["x"][0]
    TensorVisitor(_tag, update=False).apply(m)
    assert m.nested["x"][0] is before


def test_custom_handler_runs_first():
    class Box:
        __slots__ = ("payload",)

        def __init__(self, t):
            self.payload = t

    class BoxHandler:
        def can_handle(self, v):
            return isinstance(v, Box)

        def process_attribute(self, v, ctx):
            v.payload = ctx.dispatch(v.payload)
            return v

    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.box = Box(torch.ones(2))

    m = M()
    v = TensorVisitor(_tag)
    v.register_handler(BoxHandler())
    v.apply(m)
    assert m.box.payload.dtype == torch.float64


def test_compiled_wrapper_is_unwrapped():
    class OptimizedModule(nn.Module):  # same name as torch.compile's wrapper class
        def __init__(self, inner):
            super().__init__()
            self._orig_mod = inner

    inner = Deep()
    TensorVisitor(_tag).apply(OptimizedModule(inner))
    assert inner.shared.dtype == torch.float64


def test_carry_inner_fields_copies_metadata():
    a = nn.Parameter(torch.ones(2))
    a.weight_loader = "f"
    a.scale = torch.ones(1)
    b = nn.Parameter(torch.zeros(2))
    carry_inner_fields(a, b)
    assert b.weight_loader == "f" and b.scale is a.scale


class QuantLike(nn.Module):
    """A layer whose weight carries its dequantisation scale and loader metadata as tensor
    attributes (the shape vLLM's quantized linear layers use)."""

    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(8, 8) * 0.1, requires_grad=False)
        self.weight.weight_scale = torch.full((8, 1), 2.0)
        self.weight.output_dim = 0
        self.cache = {"rows": [torch.arange(8.0)]}

    def forward(self, x):
        return x @ (self.weight * self.weight.weight_scale).t() + self.cache["rows"][0]


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.q1 = QuantLike()
        self.q2 = QuantLike()

    def forward(self, x):
        return self.q2(self.q1(x))


def test_offload_keeps_quantized_weight_metadata():
    torch.manual_seed(0)
    net = Net()
    x = torch.randn(3, 8)
    ref = net(x).detach()
    mm = ft.offload(net, ft.OffloadConfig(pinned_memory=False, include_patterns=["q1", "q2"], profiling_iters=1,
                                          num_blocks=2, min_blocks=2,
                                          load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2,
                                                                         cyclic=True)))
    with torch.no_grad():
        for _ in range(4):
            assert torch.allclose(mm(x), ref)
    assert net.q1.weight.output_dim == 0 and net.q1.weight.weight_scale.shape == (8, 1)
    ft.get_offload_manager().release()


def test_getter_profile_serves_trap_copies_without_touching_parameters():
    """profile_mode='getter': during PROFILING the modules read their weights through property
    getters of a per-module subclass; the Parameter objects keep their host tensors (no .data
    rebinding) and the original classes come back for INFERENCE."""
    torch.manual_seed(3)
    net = Net()
    x = torch.randn(3, 8)
    ref = net(x).detach()
    w = net.q1.weight
    w_data_ptr = w.data_ptr()
    om = ft.get_offload_manager("getter")
    mm = om.offload(net, ft.OffloadConfig(pinned_memory=False, include_patterns=["q1", "q2"], profiling_iters=2,
                                          num_blocks=2, min_blocks=2, profile_mode="getter",
                                          load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2,
                                                                         cyclic=True)))
    seen_classes = []
    with torch.no_grad():
        assert torch.allclose(mm(x), ref)  # discovery
        assert str(om.phase).endswith("PROFILING")
        seen_classes.append(type(net.q1))
        assert type(net.q1) is not QuantLike and isinstance(net.q1, QuantLike)
        assert torch.allclose(mm(x), ref)
        assert w.data_ptr() == w_data_ptr or w.device.type == "cpu"  # the Parameter object kept its storage
        for _ in range(3):
            assert torch.allclose(mm(x), ref)
    assert str(om.phase).endswith("INFERENCE")
    assert type(net.q1) is QuantLike and type(net.q2) is QuantLike
    assert net.q1.weight is w and w.output_dim == 0
    om.release()


def test_trace_tensor_marks_do_not_spread():
    from flextensor_b200.runtime.benchmark_modes import BenchmarkReplace, TraceTensor, is_trace_tensor, \
        wrap_trace_tensor

    w = wrap_trace_tensor(torch.ones(3, 3), "blk.weight")
    assert isinstance(w, TraceTensor) and w.trace_name == "blk.weight"
    y = w @ torch.ones(3)
    assert not is_trace_tensor(y) and type(y) is torch.Tensor   # results are plain tensors
    w.mul_(2.0)
    assert is_trace_tensor(w) and float(w[0, 0]) == 2.0          # in-place keeps the mark
    assert wrap_trace_tensor(w) is w
    # on a CPU-only device nothing moves; the mode passes calls through and counts them
    with BenchmarkReplace("cpu", trace=True) as m:
        torch.add(torch.ones(2), 1)
    assert m.calls["add"] == 1 and m.moved_bytes == 0


def test_trace_tensor_flag_validation_and_is_traced():
    from flextensor_b200.runtime.tensor_manager import TensorManager

    strat = NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True)
    import pytest as _pt

    with _pt.raises(ValueError, match="incompatible"):
        TensorManager("cpu", strat, profile_mode="view", _use_trace_tensor=True)
    tm = TensorManager("cpu", strat, profile_mode="getter", _use_trace_tensor=True)
    from flextensor_b200.runtime.benchmark_modes import wrap_trace_tensor

    assert tm.is_traced(wrap_trace_tensor(torch.ones(1)))
    assert not tm.is_traced(torch.ones(1))
