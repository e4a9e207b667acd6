"""GPU / host memory snapshots at the vLLM worker's lifecycle points, written as one JSON file.

    vllm serve <model> --worker-cls flextensor_b200.contrib.vllm.snapshot.SnapshotWorker
    FT_ENABLED=1 vllm serve <model> \\
        --worker-cls flextensor_b200.contrib.vllm.snapshot.FlexTensorSnapshotWorker

With ``FT_VLLM_SNAPSHOT_OUTPUT_DIR`` set, the worker records a snapshot after each of these:
``init_device``, ``load_model``, ``determine_available_memory``, the KV-cache setup and the
compile / warm-up step. After the last one it writes
``gpu_snapshots_rank<r>_device<d>_<UTC time>.json`` holding the snapshots plus shape / dtype /
size metadata of every module's parameters (never values). A snapshot records, for the
worker's device:

* total and free device memory, and the driver-level use (total - free);
* what PyTorch's caching allocator holds (reserved), the rest (non-torch: NCCL, CUDA graphs,
  FlexTensor's symmetric heaps) and the allocator's peak;
* the host's memory (RSS of this process, available system memory).

Reference behaviour: ``src/flextensor/contrib/vllm/snapshot.py:118-260`` (same environment
variable, file name and lifecycle points).
"""

from __future__ import annotations

import json
import logging
import os
import time
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

import torch

from flextensor_b200.config import _register_env_var

LOGGER = logging.getLogger("vllm.flextensor_b200.snapshot")
OUTPUT_DIR_ENV = "FT_VLLM_SNAPSHOT_OUTPUT_DIR"
_register_env_var(OUTPUT_DIR_ENV)
_GIB = float(1 << 30)


def device_memory(device: torch.device) -> dict[str, int | float]:
    """Device memory figures in bytes (plus a wall-clock timestamp)."""
    free, total = torch.cuda.mem_get_info(device)
    reserved = torch.cuda.memory_reserved(device)
    used = total - free
    return {"total_memory": total, "free_memory": free, "cuda_memory": used, "torch_memory": reserved,
            "non_torch_memory": max(used - reserved, 0), "torch_peak": torch.cuda.max_memory_allocated(device),
            "timestamp": time.time()}


def host_memory() -> dict[str, int]:
    try:
        import psutil

        vm = psutil.virtual_memory()
        return {"rss_bytes": psutil.Process().memory_info().rss, "available_bytes": vm.available,
                "total_bytes": vm.total}
    except Exception:  # noqa: BLE001 - psutil missing: host figures are optional
        return {}


def module_parameter_metadata(model: Any) -> list[dict[str, Any]]:
    """Per module with own parameters: name -> shape / dtype / numel / bytes (no values)."""
    out = []
    for name, mod in model.named_modules():
        params = {pn: p for pn, p in getattr(mod, "_parameters", {}).items() if p is not None}
        if params:
            out.append({"name": name, "tensors_map": {
                pn: {"shape": list(p.shape), "dtype": str(p.dtype), "numel": p.numel(),
                     "size_bytes": p.numel() * p.element_size()} for pn, p in params.items()}})
    return out


class MemorySnapshotMixin:
    """Collects snapshots on the host worker (needs ``rank``, ``local_rank``, ``device``,
    ``vllm_config``) and writes them when ``FT_VLLM_SNAPSHOT_OUTPUT_DIR`` is set."""

    def _take_snapshot(self, label: str) -> None:
        snaps = self.__dict__.setdefault("_ft_snapshots", [])
        entry = {"label": label, "gpu_memory": device_memory(self.device), "host_memory": host_memory()}
        snaps.append(entry)
        g = entry["gpu_memory"]
        LOGGER.info("memory snapshot [%s]: free %.2f GiB, in use %.2f GiB (torch %.2f GiB)", label,
                    g["free_memory"] / _GIB, g["cuda_memory"] / _GIB, g["torch_memory"] / _GIB)

    def _dump_snapshots(self) -> Path | None:
        out_dir = os.environ.get(OUTPUT_DIR_ENV, "")
        if not out_dir:
            return None
        d = Path(out_dir)
        d.mkdir(parents=True, exist_ok=True)
        stamp = datetime.now(tz=timezone.utc).strftime("%Y%m%d_%H%M%S")
        path = d / f"gpu_snapshots_rank{self.rank}_device{self.local_rank}_{stamp}.json"
        data: dict[str, Any] = {"worker_type": type(self).__name__, "model": self.vllm_config.model_config.model,
                                "rank": self.rank, "local_rank": self.local_rank, "device": str(self.device),
                                "snapshots": self.__dict__.get("_ft_snapshots", [])}
        model = getattr(getattr(self, "model_runner", None), "model", None)
        if model is not None:
            try:
                data["modules"] = module_parameter_metadata(model)
            except Exception:  # noqa: BLE001 - metadata is best effort
                LOGGER.warning("module metadata for %s failed", type(model).__name__, exc_info=True)
        path.write_text(json.dumps(data, indent=2))
        LOGGER.info("memory snapshots written to %s", path)
        return path


def _with_snapshots(base: type) -> type:
    class _Snapshotting(MemorySnapshotMixin, base):  # type: ignore[misc, valid-type]
        def init_device(self) -> None:
            super().init_device()
            self._take_snapshot("after_init_device")

        def load_model(self, *args, **kwargs) -> None:
            super().load_model(*args, **kwargs)
            self._take_snapshot("after_load_model")

        def determine_available_memory(self) -> int:
            r = super().determine_available_memory()
            self._take_snapshot("after_determine_available_memory")
            return r

        def initialize_from_config(self, kv_cache_config) -> None:
            super().initialize_from_config(kv_cache_config)
            self._take_snapshot("after_kv_cache_init")

        def compile_or_warm_up_model(self):
            r = super().compile_or_warm_up_model()
            self._take_snapshot("after_compile_warmup")
            self._dump_snapshots()
            return r

    return _Snapshotting


try:
    from vllm.v1.worker.gpu_worker import Worker as _VllmWorker
except Exception:  # noqa: BLE001 - vLLM absent: the helpers above still import
    _VllmWorker = None

if _VllmWorker is not None:
    from flextensor_b200.contrib.vllm.worker import FlexTensorOffloadWorker

    SnapshotWorker = type("SnapshotWorker", (_with_snapshots(_VllmWorker),), {
        "__doc__": "vLLM's worker with memory snapshots at its lifecycle points."})
    FlexTensorSnapshotWorker = type("FlexTensorSnapshotWorker", (_with_snapshots(FlexTensorOffloadWorker),), {
        "__doc__": "The FlexTensor worker with memory snapshots at its lifecycle points."})
