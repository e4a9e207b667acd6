"""Host-first vLLM model loader (``load_format="flextensor"``): unit discovery, holding back
post-load weight processing while the checkpoint streams in, parameter-subclass replacement,
and registration with vLLM. CPU only (fake modules stand in for vLLM's quantized layers)."""

import pytest
import torch
from torch import nn

from flextensor_b200.contrib.vllm import loader as L


class _QuantMethod:
    def __init__(self):
        self.calls = 0

    def process_weights_after_loading(self, layer):
        self.calls += 1


class _QLinear(nn.Linear):
    def __init__(self, qm):
        super().__init__(4, 4)
        self.quant_method = qm


class _Block(nn.Module):
    def __init__(self, qm):
        super().__init__()
        self.proj = _QLinear(qm)
        self.norm = nn.LayerNorm(4)


class _Model(nn.Module):
    def __init__(self, qm, n=3):
        super().__init__()
        self.embed = nn.Embedding(8, 4)
        self.layers = nn.ModuleList([_Block(qm) for _ in range(n)])
        self.lm_head = _QLinear(qm)


@pytest.mark.parametrize("name,unit", [("model.layers.3.self_attn.qkv_proj", "model.layers.3"),
                                       ("layers.0.mlp", "layers.0"), ("blocks.12", "blocks.12"),
                                       ("lm_head", None), ("model.embed_tokens", None)])
def test_unit_name(name, unit):
    assert L.unit_name(name) == unit


def test_processing_units_and_loose_modules():
    qm = _QuantMethod()
    m = _Model(qm)
    units, loose = L.processing_units(m)
    assert list(units) == ["layers.0", "layers.1", "layers.2"]
    assert units["layers.1"] is m.layers[1]
    assert [n for n, _ in loose] == ["lm_head"]


def test_post_load_hooks_are_held_and_restored():
    qm = _QuantMethod()
    m = _Model(qm)
    with L.hold_post_load_hooks(m) as held:
        assert held == 1  # one shared method object
        qm.process_weights_after_loading(m.lm_head)
        assert qm.calls == 0
    qm.process_weights_after_loading(m.lm_head)
    assert qm.calls == 1
    assert "process_weights_after_loading" not in vars(qm)  # the class method is back


def test_plain_parameters_replaces_subclasses():
    class Tagged(nn.Parameter):
        pass

    m = nn.Linear(3, 2)
    m.weight = Tagged(m.weight.detach().clone())
    before = m.weight.detach().clone()
    assert L.plain_parameters(m) == 1
    assert type(m.weight) is nn.Parameter and torch.equal(m.weight.detach(), before)
    assert L.plain_parameters(m) == 0


def test_loader_registered_with_vllm():
    pytest.importorskip("vllm")
    from vllm.model_executor import model_loader

    assert L.FlexTensorModelLoader is not None
    assert model_loader._LOAD_FORMAT_TO_MODEL_LOADER["flextensor"] is L.FlexTensorModelLoader


def test_drafter_moved_before_takeover():
    pytest.importorskip("vllm")
    from types import SimpleNamespace

    from flextensor_b200.contrib.vllm.worker import ensure_drafter_on_device

    moved = []

    class _M(nn.Module):
        def to(self, *a, **k):
            moved.append(a)
            return self

    assert ensure_drafter_on_device(SimpleNamespace(), "cuda:0") is False
    assert ensure_drafter_on_device(SimpleNamespace(drafter=SimpleNamespace(model=None)), "cuda:0") is False
    assert ensure_drafter_on_device(SimpleNamespace(drafter=SimpleNamespace(model=_M())), "cuda:3") is True
    assert moved == [("cuda:3",)]
