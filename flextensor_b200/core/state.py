"""Offload plan persistence: ``profile.json`` schema v3 and its SHM byte form.

The on-disk format is a compatibility contract with the reference
(``src/flextensor/state_handler.py:161-479`` fields/``to_dict``/``from_dict``,
``:1422-1496`` file and byte IO), so field names, key stringification
(int keys become JSON strings) and the version gate (== 3) are identical:

* file form: the ``to_dict()`` object written atomically as JSON;
* SHM form: 4-byte big-endian length + compact JSON (``separators=(",", ":")``).

Validation (:meth:`TensorManagerState.validate_internal`) is this package's own
consistency check of the plan: every block label is a transfer label, block
sizes cover their labels, load-strategy tensors are named, and so on.
"""

from __future__ import annotations

import json
import os
import pathlib
import struct
import tempfile
from dataclasses import dataclass, field
from typing import Any, ClassVar

from flextensor_b200.core.stats import LayerStatistics, TensorStatistics


def atomic_write_json(file_path: str | pathlib.Path, data: dict[str, Any]) -> None:
    """Write JSON to a temp file in the target directory, fsync, then rename over the target."""
    path = pathlib.Path(file_path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".tmp", dir=path.parent)
    try:
        with os.fdopen(fd, "w") as f:
            json.dump(data, f, indent=2)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
    except BaseException:
        try:
            os.unlink(tmp)
        except FileNotFoundError:
            pass
        raise


@dataclass
class LoaderInputData:
    allocation_ordered: dict[int, list[str]]
    label_to_block_id: dict[str, int]
    transfer_to_compute_map: dict[str, str]
    label_to_size_map: dict[str, int] = field(default_factory=dict)
    block_sizes: dict[int, int] = field(default_factory=dict)
    shm_block_name_map: dict[str, str] | None = None
    release_strategy: dict[str, list[TensorStatistics]] = field(default_factory=dict)


def _mismatch(detail: str) -> ValueError:
    return ValueError(f"Saved state mismatch: {detail}. Re-profile the model.")


@dataclass
class TensorManagerState:
    SCHEMA_VERSION: ClassVar[int] = 3

    loader_type: str
    tensor_id_to_name_map: dict[int, str]
    allocation_ordered: dict[int, list[str]]
    label_to_size_map: dict[str, int]
    block_sizes: dict[int, int]
    load_strategy: dict[str, list[TensorStatistics]]
    release_strategy: dict[str, list[TensorStatistics]]
    label_to_block_id: dict[str, int]
    stats: list[LayerStatistics]
    transfer_to_compute_map: dict[str, str]
    view_tensors_ids: list[int]
    view_tensors_names: list[str]
    gpu_tensors_names: list[str]
    shm_block_name_map: dict[str, str] | None
    managed_tensor_dtypes: dict[str, str] = field(default_factory=dict)
    managed_tensor_layouts: dict[str, dict[str, list[int]]] = field(default_factory=dict)

    # ------------------------------------------------------------------ validation
    def validate_internal(self) -> None:
        from flextensor_b200.config import OFFLOAD_TRANSFER_MODES

        if self.loader_type not in OFFLOAD_TRANSFER_MODES:
            raise _mismatch(f"unknown loader_type {self.loader_type!r}")
        names = set(self.tensor_id_to_name_map.values())
        labels = [s.label for s in self.stats]
        if len(set(labels)) != len(labels):
            raise _mismatch("duplicate labels in stats")
        label_set = set(labels)
        for lbl, ts in self.load_strategy.items():
            if lbl not in label_set:
                raise _mismatch(f"load_strategy label {lbl!r} not in stats")
            for t in ts:
                if t.tensor_id in self.tensor_id_to_name_map and self.tensor_id_to_name_map[t.tensor_id] != t.name:
                    raise _mismatch(f"tensor id {t.tensor_id} name {t.name!r} disagrees with id map")
                if t.name not in names:
                    raise _mismatch(f"load_strategy tensor {t.name!r} has no id mapping")
        for t, c in self.transfer_to_compute_map.items():
            if t not in label_set or c not in label_set:
                raise _mismatch(f"transfer_to_compute_map entry {t!r}->{c!r} references unknown label")
        if self.loader_type != "strategy":
            flat = [l for ls in self.allocation_ordered.values() for l in ls]
            if len(flat) != len(set(flat)):
                raise _mismatch("a label is assigned to two blocks")
            for b, ls in self.allocation_ordered.items():
                if b not in self.block_sizes:
                    raise _mismatch(f"block {b} has no size")
                for l in ls:
                    if self.label_to_block_id.get(l) != b:
                        raise _mismatch(f"label {l!r} block id disagrees with allocation")
                    if self.label_to_size_map.get(l, 0) > self.block_sizes[b]:
                        raise _mismatch(f"label {l!r} larger than its block")
            for lbl, ts in self.load_strategy.items():
                if ts and lbl not in self.label_to_block_id:
                    raise _mismatch(f"transfer label {lbl!r} has no block")
        if len(self.view_tensors_ids) != len(self.view_tensors_names):
            raise _mismatch("view tensor ids/names length differ")
        if self.shm_block_name_map is not None and not isinstance(self.shm_block_name_map, dict):
            raise _mismatch("shm_block_name_map must be an object")

    # ------------------------------------------------------------------ dict form
    def to_dict(self) -> dict[str, Any]:
        return {
            "version": self.SCHEMA_VERSION,
            "loader_type": self.loader_type,
            "tensor_id_to_name_map": {str(k): v for k, v in self.tensor_id_to_name_map.items()},
            "allocation_ordered": {str(k): v for k, v in self.allocation_ordered.items()},
            "label_to_size_map": {str(k): v for k, v in self.label_to_size_map.items()},
            "block_sizes": {str(k): v for k, v in self.block_sizes.items()},
            "load_strategy": {k: [t.model_dump() for t in v] for k, v in self.load_strategy.items()},
            "release_strategy": {k: [t.model_dump() for t in v] for k, v in self.release_strategy.items()},
            "label_to_block_id": self.label_to_block_id,
            "stats": [s.model_dump() for s in self.stats],
            "transfer_to_compute_map": self.transfer_to_compute_map,
            "view_tensors_ids": self.view_tensors_ids,
            "view_tensors_names": self.view_tensors_names,
            "gpu_tensors_names": self.gpu_tensors_names,
            "shm_block_name_map": self.shm_block_name_map,
            "managed_tensor_dtypes": self.managed_tensor_dtypes,
            "managed_tensor_layouts": self.managed_tensor_layouts,
        }

    @staticmethod
    def _check_version(data: dict[str, Any]) -> None:
        v = data.get("version", 1)
        cur = TensorManagerState.SCHEMA_VERSION
        if v > cur:
            raise ValueError(f"State file schema version {v} is newer than supported version {cur}. "
                             "Upgrade to load this file.")
        if v < cur:
            raise ValueError(f"State file schema version {v} is outdated (current: {cur}). "
                             "Re-run profiling to generate a new profile.")

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "TensorManagerState":
        cls._check_version(data)
        ts = lambda rows: [TensorStatistics(**r) for r in rows]  # noqa: E731
        st = cls(
            loader_type=data["loader_type"],
            tensor_id_to_name_map={int(k): v for k, v in data["tensor_id_to_name_map"].items()},
            allocation_ordered={int(k): list(v) for k, v in data["allocation_ordered"].items()},
            label_to_size_map={str(k): int(v) for k, v in data["label_to_size_map"].items()},
            block_sizes={int(k): int(v) for k, v in data["block_sizes"].items()},
            load_strategy={k: ts(v) for k, v in data["load_strategy"].items()},
            release_strategy={k: ts(v) for k, v in data["release_strategy"].items()},
            label_to_block_id={k: int(v) for k, v in data["label_to_block_id"].items()},
            stats=[LayerStatistics(**s) for s in data["stats"]],
            transfer_to_compute_map=dict(data["transfer_to_compute_map"]),
            view_tensors_ids=list(data["view_tensors_ids"]),
            view_tensors_names=list(data["view_tensors_names"]),
            gpu_tensors_names=list(data["gpu_tensors_names"]),
            shm_block_name_map=data["shm_block_name_map"],
            managed_tensor_dtypes=data.get("managed_tensor_dtypes", {}),
            managed_tensor_layouts=data.get("managed_tensor_layouts", {}),
        )
        st.validate_internal()
        return st

    def to_loader_input_data(self) -> LoaderInputData:
        return LoaderInputData(
            allocation_ordered=self.allocation_ordered,
            label_to_block_id=self.label_to_block_id,
            transfer_to_compute_map=self.transfer_to_compute_map,
            label_to_size_map=self.label_to_size_map,
            block_sizes=self.block_sizes,
            shm_block_name_map=self.shm_block_name_map,
            release_strategy=self.release_strategy,
        )

    # ------------------------------------------------------------------ IO
    @staticmethod
    def save_to_file(file_path: str | pathlib.Path, state: "TensorManagerState") -> None:
        atomic_write_json(file_path, state.to_dict())

    @staticmethod
    def load_from_file(file_path: str | pathlib.Path) -> "TensorManagerState":
        with pathlib.Path(file_path).open() as f:
            data = json.load(f)
        if not isinstance(data, dict):
            raise ValueError("Saved state must be a JSON object")
        try:
            return TensorManagerState.from_dict(data)
        except AttributeError as exc:
            raise ValueError("Saved state contains malformed nested data") from exc

    @staticmethod
    def save_state_to_bytes(state: "TensorManagerState") -> bytes:
        payload = json.dumps(state.to_dict(), separators=(",", ":")).encode("utf-8")
        return struct.pack("!I", len(payload)) + payload

    @staticmethod
    def load_state_from_bytes(data: bytes | bytearray | memoryview) -> "TensorManagerState":
        if len(data) < 4:
            raise ValueError(f"Buffer too short: expected at least 4 bytes for length prefix, got {len(data)}")
        (n,) = struct.unpack("!I", bytes(data[:4]))
        if len(data) < 4 + n:
            raise ValueError(f"Buffer too short: length prefix indicates {n} bytes, "
                             f"but only {len(data) - 4} bytes available after prefix")
        return TensorManagerState.from_dict(json.loads(bytes(data[4:4 + n])))


PROFILE_FILENAME = "profile.json"
