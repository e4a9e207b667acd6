import json

import pytest

from flextensor_b200.core.state import TensorManagerState
from flextensor_b200.core.stats import LayerStatistics, TensorStatistics


def state():
    t = lambda i, n: TensorStatistics(tensor_id=i, name=n, size_bytes=100, load_time_ms=0.1)  # noqa: E731
    return TensorManagerState(
        loader_type="allocation_block_transfer", tensor_id_to_name_map={0: "a.w", 1: "b.w"},
        allocation_ordered={0: ["a"], 1: ["b"]}, label_to_size_map={"a": 100, "b": 100}, block_sizes={0: 256, 1: 256},
        load_strategy={"a": [t(1, "b.w")], "b": [t(0, "a.w")]}, release_strategy={},
        label_to_block_id={"a": 0, "b": 1},
        stats=[LayerStatistics(label="a", tensors=[t(0, "a.w")], duration=1.0),
               LayerStatistics(label="b", tensors=[t(1, "b.w")], duration=1.0)],
        transfer_to_compute_map={"a": "b", "b": "a"}, view_tensors_ids=[0, 1], view_tensors_names=["a.w", "b.w"],
        gpu_tensors_names=[], shm_block_name_map=None)


def test_dict_roundtrip(tmp_path):
    s = state()
    d = s.to_dict()
    assert d["version"] == 3 and d["tensor_id_to_name_map"] == {"0": "a.w", "1": "b.w"}
    assert list(d) == ["version", "loader_type", "tensor_id_to_name_map", "allocation_ordered", "label_to_size_map",
                       "block_sizes", "load_strategy", "release_strategy", "label_to_block_id", "stats",
                       "transfer_to_compute_map", "view_tensors_ids", "view_tensors_names", "gpu_tensors_names",
                       "shm_block_name_map", "managed_tensor_dtypes", "managed_tensor_layouts"]
    TensorManagerState.save_to_file(tmp_path / "p.json", s)
    assert TensorManagerState.load_from_file(tmp_path / "p.json") == s
    b = TensorManagerState.save_state_to_bytes(s)
    assert int.from_bytes(b[:4], "big") == len(b) - 4
    assert TensorManagerState.load_state_from_bytes(b) == s


def test_version_gate(tmp_path):
    d = state().to_dict()
    d["version"] = 2
    with pytest.raises(ValueError, match="outdated"):
        TensorManagerState.from_dict(d)
    d["version"] = 4
    with pytest.raises(ValueError, match="newer"):
        TensorManagerState.from_dict(d)


def test_validation_catches_inconsistency():
    d = state().to_dict()
    d["block_sizes"]["0"] = 10
    with pytest.raises(ValueError, match="larger than its block"):
        TensorManagerState.from_dict(d)
    d = state().to_dict()
    d["transfer_to_compute_map"]["a"] = "zzz"
    with pytest.raises(ValueError):
        TensorManagerState.from_dict(d)


def test_short_buffers():
    with pytest.raises(ValueError):
        TensorManagerState.load_state_from_bytes(b"\x00\x00")
    with pytest.raises(ValueError):
        TensorManagerState.load_state_from_bytes(b"\x00\x00\x00\x09{}")
