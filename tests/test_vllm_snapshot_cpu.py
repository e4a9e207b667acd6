"""Memory snapshot workers: lifecycle snapshots, the JSON dump (file name, fields, parameter
metadata without values) and the worker classes' lifecycle hooks. CPU only (device memory
queries are faked)."""

import json
from types import SimpleNamespace

import pytest
import torch
from torch import nn

from flextensor_b200.contrib.vllm import snapshot as S


class _Host(S.MemorySnapshotMixin):
    def __init__(self):
        self.rank, self.local_rank, self.device = 3, 1, torch.device("cuda", 1)
        self.vllm_config = SimpleNamespace(model_config=SimpleNamespace(model="tiny"))
        self.model_runner = SimpleNamespace(model=nn.Sequential(nn.Linear(4, 2), nn.LayerNorm(2)))


@pytest.fixture
def fake_cuda(monkeypatch):
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda d: (30 << 30, 180 << 30))
    monkeypatch.setattr(torch.cuda, "memory_reserved", lambda d: 100 << 30)
    monkeypatch.setattr(torch.cuda, "max_memory_allocated", lambda d: 90 << 30)


def test_snapshots_and_dump(tmp_path, monkeypatch, fake_cuda):
    monkeypatch.setenv(S.OUTPUT_DIR_ENV, str(tmp_path))
    h = _Host()
    h._take_snapshot("after_load_model")
    h._take_snapshot("after_kv_cache_init")
    path = h._dump_snapshots()
    assert path.name.startswith("gpu_snapshots_rank3_device1_") and path.suffix == ".json"
    data = json.loads(path.read_text())
    assert [s["label"] for s in data["snapshots"]] == ["after_load_model", "after_kv_cache_init"]
    g = data["snapshots"][0]["gpu_memory"]
    assert g["cuda_memory"] == 150 << 30 and g["non_torch_memory"] == 50 << 30 and g["torch_peak"] == 90 << 30
    mods = {m["name"]: m["tensors_map"] for m in data["modules"]}
    assert mods["0"]["weight"] == {"shape": [2, 4], "dtype": "torch.float32", "numel": 8, "size_bytes": 32}
    assert "1" in mods and data["model"] == "tiny"


def test_no_output_dir_no_file(monkeypatch, fake_cuda):
    monkeypatch.delenv(S.OUTPUT_DIR_ENV, raising=False)
    h = _Host()
    h._take_snapshot("x")
    assert h._dump_snapshots() is None


def test_worker_classes_hook_the_lifecycle():
    pytest.importorskip("vllm")
    for cls in (S.SnapshotWorker, S.FlexTensorSnapshotWorker):
        for hook in ("init_device", "load_model", "determine_available_memory", "initialize_from_config",
                     "compile_or_warm_up_model"):
            assert hook in vars(cls.__mro__[1]), (cls, hook)
    from flextensor_b200.contrib.vllm.worker import FlexTensorOffloadWorker

    assert issubclass(S.FlexTensorSnapshotWorker, FlexTensorOffloadWorker)
