"""Symmetric device heap shared by all ranks of a node through CUDA IPC.

Every rank ``cudaMalloc``s the same number of bytes, exports an IPC handle,
all-gathers the handles over the process group (control plane; any backend)
and opens every peer's heap, so kernels on this GPU can load from and store to
any peer's heap with plain pointers over NVLink/NVSwitch. Offsets are identical
on every rank (same layout), which is what makes the heap "symmetric".
"""

from __future__ import annotations

import torch

from flextensor_b200.ops import native


class _DevBuf:
    """Minimal ``__cuda_array_interface__`` wrapper so torch can view raw device memory."""

    def __init__(self, ptr: int, nbytes: int, device: int, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3, "strides": None,
        }
        self.device = device


class SymmetricHeap:
    def __init__(self, nbytes: int, group=None, device: int | None = None):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("symmetric heaps span one node (at most 8 ranks)")
        self.device = torch.cuda.current_device() if device is None else device
        self.nbytes = int(nbytes)
        lib = native.lib()
        with torch.cuda.device(self.device):
            self.base = lib.device_malloc(self.nbytes)
            handle = lib.ipc_handle(self.base)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, (self.rank, handle), group=group)
        self.ptrs = [0] * self.world
        self._opened = []
        with torch.cuda.device(self.device):
            for r, h in handles:
                if r == self.rank:
                    self.ptrs[r] = self.base
                else:
                    p = lib.ipc_open(h)
                    self.ptrs[r] = p
                    self._opened.append(p)
        self.local = torch.as_tensor(_DevBuf(self.base, self.nbytes, self.device, self), device=f"cuda:{self.device}")
        self._closed = False

    def view(self, offset: int, nbytes: int) -> torch.Tensor:
        return self.local[offset:offset + nbytes]

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        lib = native.lib()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib.ipc_close(p)
        self._opened.clear()
        self.local = None
        lib.device_free(self.base)
