"""SHM-backed weight blocks for the TensorManager (``{ns}_w{i}`` segments).

The creator allocates one segment per transfer label, packs the label's
tensors into it and page-locks it (``cudaHostRegister``); followers attach to
the same segments and register them too, so every local worker streams from
ONE host copy. ``load_from_shm`` (set by the session) tells the TensorManager
the bytes are already packed and must not be overwritten.
"""

from __future__ import annotations

import torch

from flextensor_b200.core.host_store import packed_layout, tensor_nbytes
from flextensor_b200.shm.namespace import weight_block_name
from flextensor_b200.shm.segment import ShmSegment, shm_exists, shm_unlink


class ShmWeightStore:
    def __init__(self, namespace: str, pinned: bool = True):
        self.ns = namespace
        self.pinned = pinned
        self.segments: dict[str, ShmSegment] = {}
        self._names: dict[str, str] = {}
        self._next = 0

    def block_buffer(self, label: str, items: list[tuple[int, str, torch.Tensor]],
                     must_exist: bool = False) -> torch.Tensor:
        _, total = packed_layout([tensor_nbytes(t) for _, _, t in items])
        name = weight_block_name(self.ns, self._next)
        self._next += 1
        if must_exist and not shm_exists(name):
            raise FileNotFoundError(f"SHM weight block {name} for {label!r} does not exist; the creator has not "
                                    "published it (or already released it)")
        if shm_exists(name):
            seg = ShmSegment.attach(name)
            if seg.size < total:
                seg.close()
                raise ValueError(f"SHM block {name} holds {seg.size} bytes, plan needs {total}")
        else:
            seg = ShmSegment.create(name, total)
        if self.pinned and torch.cuda.is_available():
            seg.pin()
        self.segments[label] = seg
        self._names[label] = name
        return seg.tensor()[:max(total, 1)]

    def block_name_map(self) -> dict[str, str]:
        return dict(self._names)

    def close(self, unlink: bool = False) -> None:
        """Drop the mappings (live tensor views keep their pages); unlink only segments this process created."""
        for seg in self.segments.values():
            created = seg.created
            seg.close()
            if unlink and created:
                shm_unlink(seg.name)
        self.segments.clear()
