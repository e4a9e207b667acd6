"""Host-side weight store: pinned packing of offloaded tensors into per-label blocks.

Each transfer label owns one contiguous host block holding all tensors it
streams, packed in plan order at ``PACK_ALIGN``-byte offsets, so one trap's
prefetch is ONE ``cudaMemcpyAsync`` of a contiguous pinned range (the copy
engine's best case) straight into the label's GPU ring slot, and each
parameter's ``.data`` is a typed view at the same offset inside the slot.

Packing is the reference's allocation-block layout in spirit
(``src/flextensor/utils.py:114-127`` uses 128 B); 256 B is used here so every
view also meets TMA's 16-byte base and 128-byte swizzle-atom alignment.

Pinning policies mirror ``src/flextensor/host_pinning.py:171-480``: ``torch``
copies into a fresh page-locked allocation, ``host_register`` page-locks the
existing allocation in place with ``cudaHostRegister`` (native helper).
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field

import torch

logger = logging.getLogger(__name__)

PACK_ALIGN = 256


def packed_layout(sizes: list[int], align: int = PACK_ALIGN) -> tuple[list[int], int]:
    offs, cur = [], 0
    for s in sizes:
        offs.append(cur)
        cur = (cur + s + align - 1) // align * align
    return offs, cur


def tensor_nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _cuda_ok() -> bool:
    return torch.cuda.is_available()


class HostPinRegistry:
    """Tracks in-place registrations so every ``cudaHostRegister`` gets its unregister."""

    def __init__(self) -> None:
        self._ptrs: dict[int, int] = {}

    def __len__(self) -> int:
        return len(self._ptrs)

    def is_registered(self, ptr: int) -> bool:
        return ptr in self._ptrs

    def pin_in_place(self, t: torch.Tensor) -> torch.Tensor:
        from flextensor_b200.ops import native

        ptr, n = t.data_ptr(), tensor_nbytes(t)
        if n == 0 or ptr in self._ptrs or t.is_pinned():
            return t
        native.host_register(ptr, n)
        self._ptrs[ptr] = n
        return t

    def release(self, ptr: int) -> bool:
        if ptr not in self._ptrs:
            return False
        from flextensor_b200.ops import native

        native.host_unregister(ptr)
        del self._ptrs[ptr]
        return True

    def release_all(self) -> None:
        for p in list(self._ptrs):
            try:
                self.release(p)
            except Exception:  # noqa: BLE001 - best effort at teardown
                logger.warning("cudaHostUnregister failed for 0x%x", p, exc_info=True)
                self._ptrs.pop(p, None)


class HostPinner:
    def __init__(self, mode: str = "torch", registry: HostPinRegistry | None = None) -> None:
        self.mode = mode
        self.registry = registry if registry is not None else HostPinRegistry()

    def pin(self, t: torch.Tensor) -> torch.Tensor:
        if t.device.type != "cpu" or not _cuda_ok() or tensor_nbytes(t) == 0 or t.is_pinned():
            return t
        if self.mode == "host_register":
            return self.registry.pin_in_place(t.contiguous())
        return t.pin_memory()

    def is_pinned(self, t: torch.Tensor) -> bool:
        return t.device.type == "cpu" and _cuda_ok() and (t.is_pinned() or self.registry.is_registered(t.data_ptr()))

    def release_all(self) -> None:
        self.registry.release_all()


class NoOpHostPinner(HostPinner):
    def __init__(self) -> None:
        super().__init__("torch")

    def pin(self, t: torch.Tensor) -> torch.Tensor:
        return t


def make_host_pinner(pinned_memory: bool, mode: str) -> HostPinner:
    if not pinned_memory:
        return NoOpHostPinner()
    if mode not in ("torch", "host_register"):
        raise ValueError(f"unknown pinned_memory_mode {mode!r}")
    return HostPinner(mode)


EXACT_PIN_MIN = 16 << 20


def alloc_host_bytes(nbytes: int, pinned: bool) -> torch.Tensor:
    """``nbytes`` of host memory, page-locked when ``pinned``. Large pinned requests get exactly
    their size from the native extension (one cudaHostAlloc freed with the last view): torch's
    caching host allocator would round each up to a power of two, which for a multi-GB packed
    arena pins up to twice its bytes."""
    if pinned and _cuda_ok():
        if nbytes >= EXACT_PIN_MIN:
            from flextensor_b200.ops import native

            if native.available():
                return native.pinned_empty(int(nbytes))
        return torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    return torch.empty(nbytes, dtype=torch.uint8)


@dataclass
class PackedEntry:
    tensor_id: int
    name: str
    offset: int
    nbytes: int
    dtype: torch.dtype
    shape: tuple[int, ...]


@dataclass
class HostBlock:
    """One label's packed host bytes plus where each tensor sits inside them."""

    label: str
    data: torch.Tensor
    entries: list[PackedEntry] = field(default_factory=list)
    shm_name: str | None = None
    total: int | None = None                  # packed size when ``data`` holds only one stripe
    stripe: tuple[int, int] | None = None     # [b0, b1) of the packed bytes held in ``data``

    @property
    def nbytes(self) -> int:
        """Size of the whole packed block (what a device slot holds)."""
        return self.total if self.total is not None else self.data.numel()

    @property
    def stripe_only(self) -> bool:
        return self.stripe is not None

    def view(self, e: PackedEntry, base: torch.Tensor | None = None) -> torch.Tensor:
        if base is None and self.stripe is not None:
            raise RuntimeError(f"host block {self.label!r} holds one stripe; whole tensors live on the device only")
        buf = self.data if base is None else base
        return buf[e.offset:e.offset + e.nbytes].view(e.dtype).view(e.shape)


def stripe_len(total: int, world: int) -> int:
    """Stripe length of a packed block: ceil(total / world) rounded up to 256 bytes (the native
    engine and the gather kernel use the same rule)."""
    return ((total + world - 1) // world + 255) // 256 * 256


def stripe_range(total: int, rank: int, world: int) -> tuple[int, int]:
    s = stripe_len(total, world)
    b0 = min(rank * s, total)
    return b0, min(b0 + s, total)


def pack_tensors_stripe(label: str, items: list[tuple[int, str, torch.Tensor]], rank: int, world: int,
                        pinned: bool = True, release_sources=None, buffer: torch.Tensor | None = None) -> HostBlock:
    """Pack only stripe ``rank`` of ``world`` of a label's block into host memory.

    The layout (offsets, total) is the one :func:`pack_tensors` would produce, so every rank
    agrees on it; each rank keeps ``stripe_len(total)`` bytes, and the full block only ever
    exists in the device slot after the peers' stripes were gathered. Sources may live on the
    device (copied D2H slice by slice) or on the host.
    """
    sizes = [tensor_nbytes(t) for _, _, t in items]
    offs, total = packed_layout(sizes)
    b0, b1 = stripe_range(total, rank, world)
    data = buffer if buffer is not None else alloc_host_bytes(max(b1 - b0, 256), pinned)
    if data.numel() < b1 - b0:
        raise ValueError(f"stripe buffer for {label!r} holds {data.numel()} bytes, needs {b1 - b0}")
    blk = HostBlock(label, data, total=total, stripe=(b0, b1))
    for (tid, name, t), off, n in zip(items, offs, sizes):
        blk.entries.append(PackedEntry(tid, name, off, n, t.dtype, tuple(t.shape)))
        lo, hi = max(off, b0), min(off + n, b1)
        if hi > lo:
            src = t.detach().contiguous().reshape(-1).view(torch.uint8)[lo - off:hi - off]
            data[lo - b0:hi - b0].copy_(src)
        if release_sources is not None:
            release_sources(tid)
    return blk


def pack_tensors(label: str, items: list[tuple[int, str, torch.Tensor]], buffer: torch.Tensor | None = None,
                 pinned: bool = True, release_sources=None) -> HostBlock:
    """Copy ``(tensor_id, name, tensor)`` items into one packed host block.

    ``release_sources(tensor_id)`` (optional) is called right after each copy
    so peak host memory stays ~one block above the model size.
    """
    sizes = [tensor_nbytes(t) for _, _, t in items]
    offs, total = packed_layout(sizes)
    data = buffer if buffer is not None else alloc_host_bytes(max(total, PACK_ALIGN), pinned)
    if data.numel() < total:
        raise ValueError(f"host buffer for {label!r} holds {data.numel()} bytes, needs {total}")
    blk = HostBlock(label, data)
    for (tid, name, t), off, n in zip(items, offs, sizes):
        e = PackedEntry(tid, name, off, n, t.dtype, tuple(t.shape))
        if n:
            blk.view(e).copy_(t.detach())  # a device source is copied straight into the block
        blk.entries.append(e)
        if release_sources is not None:
            release_sources(tid)
    return blk
