"""Profile-driven lazy model construction on the CPU: parameters built on ``meta`` and
materialised from a safetensors file keep their nested links (``weight.scale is scale``), their
plain attribute flags and their ties, and load the saved values."""

import types

import pytest
import torch
from torch import nn

from flextensor_b200.runtime.lazy_init import (LinkTracker, create_split_device_model_with_tracking,
                                               load_model_from_profile)


class QuantLinear(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(d, d))
        self.scale = nn.Parameter(torch.ones(d))
        self.weight.scale = self.scale          # nested link to another registered parameter
        self.weight.is_packed = True            # plain flag
        self.register_buffer("zero_point", torch.zeros(d))
        self.weight.zp = self.zero_point        # link to a buffer

    def forward(self, x):
        return (x @ self.weight.t()) * self.weight.scale + self.weight.zp


class Net(nn.Module):
    def __init__(self, vocab=32, d=16):
        super().__init__()
        self.embed = nn.Embedding(vocab, d)
        self.blocks = nn.ModuleList([QuantLinear(d) for _ in range(2)])
        self.head = nn.Linear(d, vocab, bias=False)
        self.head.weight = self.embed.weight    # tied

    def forward(self, ids):
        x = self.embed(ids)
        for b in self.blocks:
            x = torch.tanh(b(x))
        return self.head(x)


def _checkpoint(tmp_path):
    pytest.importorskip("safetensors")
    from safetensors.torch import save_file

    torch.manual_seed(0)
    ref = Net()
    with torch.no_grad():
        for b in ref.blocks:
            b.scale.uniform_(0.5, 1.5)
            b.zero_point.uniform_(-0.1, 0.1)
    sd = {k: v.contiguous() for k, v in ref.state_dict().items() if k != "head.weight"}
    path = tmp_path / "w.safetensors"
    save_file(sd, str(path))
    return ref, str(path)


def test_tracker_records_links_flags_and_ties():
    with torch.device("meta"):
        m = Net()
    t = LinkTracker.capture(m)
    assert t.links[("blocks.0.weight", "scale")] == "blocks.0.scale"
    assert t.links[("blocks.1.weight", "zp")] == "blocks.1.zero_point"
    assert t.plain[("blocks.0.weight", "is_packed")] is True
    assert t.ties == {"head.weight": "embed.weight"}


def test_load_model_from_profile_keeps_links_and_values(tmp_path):
    ref, path = _checkpoint(tmp_path)
    state = types.SimpleNamespace(gpu_tensors_names=["embed.weight", "blocks.0.scale"])
    tm = types.SimpleNamespace(device=torch.device("cpu"), load_state=lambda d: state)
    m = load_model_from_profile(tm, str(tmp_path), Net, safetensor_path=path, buffer_device="cpu", diagnose=True)
    for b in m.blocks:
        assert b.weight.scale is b.scale
        assert b.weight.zp is b.zero_point
        assert b.weight.is_packed is True
    assert m.head.weight is m.embed.weight
    ids = torch.randint(0, 32, (3, 5))
    with torch.no_grad():
        torch.testing.assert_close(m(ids), ref(ids), rtol=0, atol=0)


def test_restore_after_load_state_dict_assign(tmp_path):
    ref, _ = _checkpoint(tmp_path)
    m, tracker = create_split_device_model_with_tracking(Net, buffer_device="cpu")
    m.load_state_dict(ref.state_dict(), assign=True)   # new tensor objects: links are gone
    assert not hasattr(m.blocks[0].weight, "scale")
    assert tracker.restore(m) == len(tracker)
    assert m.blocks[0].weight.scale is m.blocks[0].scale
    assert m.head.weight is m.embed.weight
