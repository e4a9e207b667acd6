import torch
from torch import nn

from flextensor_b200.runtime.units import select_units
from flextensor_b200.utils.patterns import matches_any_class_pattern, matches_any_pattern, partition_patterns


def test_star_semantics():
    assert matches_any_pattern("layers.0", ["layers.*"], recursive_star=False)
    assert not matches_any_pattern("layers.0.attn", ["layers.*"], recursive_star=False)
    assert matches_any_pattern("layers.0.attn.weight", ["*.weight"], recursive_star=True)
    assert not matches_any_pattern("layers.0.attn.weight", ["*.weight"], recursive_star=False)
    assert matches_any_pattern("attention.q", ["attention.?"])
    assert matches_any_pattern("encoder.block_12", ["encoder.block_*"])


def test_partition_and_class():
    names, classes = partition_patterns(["layers.*", "name:embed", "class:MoELayer"])
    assert names == ["layers.*", "embed"] and classes == ["MoELayer"]
    assert matches_any_class_pattern(nn.Linear, ["Lin*"])
    assert matches_any_class_pattern(nn.Linear, ["torch.nn.*.Linear"])
    assert not matches_any_class_pattern(nn.Linear, ["*Expert*"])


class Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = nn.Linear(4, 4)
        self.norm = nn.LayerNorm(4)

    def forward(self, x):
        return self.norm(self.attn(x))


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.embed = nn.Linear(4, 4)
        self.layers = nn.ModuleList([Block() for _ in range(3)])
        self.head = nn.Linear(4, 4)


def test_unit_selection():
    net = Net()
    us = select_units(net, ["layers.*"], [])
    assert [u.label for u in us] == ["layers.0", "layers.1", "layers.2"]
    us = select_units(net, ["*"], [])  # ModuleList expands into its children
    assert [u.label for u in us] == ["embed", "layers.0", "layers.1", "layers.2", "head"]
    us = select_units(net, ["layers.*"], ["layers.1", "*.norm"])
    assert [u.label for u in us] == ["layers.0", "layers.2"]
    assert all(all(".norm." not in n for n, _ in u.params) for u in us)
    us = select_units(net, ["layers.*.weight"], [])
    assert all(n.endswith("weight") for u in us for n, _ in u.params)
    assert all(any(n.endswith("bias") for n, _ in u.kept) for u in us)
    us = select_units(net, ["class:Block"], ["class:LayerNorm"])
    assert len(us) == 3 and all(all("norm" not in n for n, _ in u.params) for u in us)
