"""Striped host streaming across the GPUs of one node.

With N ranks each running a replica of the same offloaded model, every ring slot
lives in a symmetric heap. When a trap's weights are prefetched, rank r copies
only stripe r (1/N of the packed host block) over its own PCIe link, then the
other N-1 stripes come from the peers' slots over NVLink: by the copy engines between
two one-warp signalling kernels (``FT_STRIPED_GATHER=ce``, the default; see
``ops/csrc/p2p.cu``) or by a pull kernel of small CTAs (``FT_STRIPED_GATHER=sm``).
Host-link bytes per rank drop N-fold, so the node's
aggregate PCIe bandwidth -- and, with the shared-memory store, one host copy of
the weights -- serves all ranks.

Enable before ``offload()``::

    flextensor_b200.parallel.enable_striped_streaming()      # default process group

or set ``FT_STRIPED_STREAMING=1`` (the TensorManager then uses the default group).
"""

from __future__ import annotations

import os

import torch

from flextensor_b200.config import _register_env_var
from flextensor_b200.ops import native
from flextensor_b200.parallel.symm import SymmetricHeap
from flextensor_b200.instrumentation.core import instrumentable

_register_env_var("FT_STRIPED_STREAMING")
_register_env_var("FT_STRIPED_GATHER")
_register_env_var("FT_STRIPED_GATHER_CTAS")

GATHER_MODES = {"sm": 0, "ce": 1}


def gather_mode() -> str:
    """How the peers' stripes cross NVLink: ``ce`` (default) -- the copy engines (one
    cudaMemcpyAsync per peer stripe between a one-warp bounded flag wait and an acknowledgement
    kernel), which leaves the SMs to the compute kernels; ``sm`` -- a pull kernel of small CTAs
    on the copy stream. ``FT_STRIPED_GATHER`` selects it. On the 2-GPU Wan-14B-shape bench the
    copy engines gave 1.490 s/step against 1.501 for the pull kernel."""
    m = os.environ.get("FT_STRIPED_GATHER", "ce").strip().lower() or "ce"
    if m not in GATHER_MODES:
        raise ValueError(f"FT_STRIPED_GATHER={m!r}: expected one of {sorted(GATHER_MODES)}")
    return m


_STATE = {"enabled": False, "group": None}
HEADER_ALIGN = 4096
SLOT_ALIGN = 4096


def enable_striped_streaming(group=None) -> None:
    _STATE["enabled"] = True
    _STATE["group"] = group


def disable_striped_streaming() -> None:
    _STATE["enabled"] = False
    _STATE["group"] = None


def striping_group():
    """The group to stripe over, or ``None`` when striping is off / single process."""
    import torch.distributed as dist

    on = _STATE["enabled"] or os.environ.get("FT_STRIPED_STREAMING", "0") not in ("", "0", "false", "False")
    if not on or not dist.is_available() or not dist.is_initialized():
        return None
    g = _STATE["group"] if _STATE["group"] is not None else dist.group.WORLD
    return g if dist.get_world_size(g) > 1 else None


@instrumentable
class StripedTransferEngine:
    """Native engine in striped mode; owns the symmetric heap that backs the ring slots."""

    def __init__(self, device: torch.device, slot_bytes: dict[int, int], group=None, timing: bool = False,
                 gather_ctas: int | None = None, max_keys: int = 4096, gather: str | None = None):
        if gather_ctas is None:
            gather_ctas = int(os.environ.get("FT_STRIPED_GATHER_CTAS", "16"))
        self.gather = gather or gather_mode()
        if self.gather not in GATHER_MODES:
            raise ValueError(f"gather={self.gather!r}: expected one of {sorted(GATHER_MODES)}")
        self.device = torch.device(device)
        n_slots = max(slot_bytes) + 1 if slot_bytes else 1
        import torch.distributed as dist

        world = dist.get_world_size(group)
        hdr = world * n_slots * 8 * 2 + n_slots * 4
        hdr = (hdr + HEADER_ALIGN - 1) // HEADER_ALIGN * HEADER_ALIGN
        offs, cur = [0] * n_slots, hdr
        for s in range(n_slots):
            offs[s] = cur
            cur += (slot_bytes.get(s, 0) + SLOT_ALIGN - 1) // SLOT_ALIGN * SLOT_ALIGN
        self.group = group
        self.heap = SymmetricHeap(cur, group, self.device.index or 0)
        self.slot_offsets = offs
        self.slot_bytes = slot_bytes
        self.n_slots = n_slots
        flags = [p for p in self.heap.ptrs]
        acks = [p + world * n_slots * 8 for p in self.heap.ptrs]
        counters = self.heap.base + 2 * world * n_slots * 8
        self._keys: dict[str, int] = {}
        self._names: list[str] = []
        self._e = native.lib().TransferEngine(self.device.index or 0, n_slots, max_keys, bool(timing))
        self._e.enable_striping(list(self.heap.ptrs), flags, acks, self.heap.rank, n_slots, offs, counters,
                                gather_ctas, GATHER_MODES[self.gather])
        self.timing = timing
        dist.barrier(group=group)  # every rank's heap is open before anyone publishes into it

    # slots are views of the symmetric heap
    def slot_tensor(self, slot: int, nbytes: int) -> torch.Tensor:
        return self.heap.view(self.slot_offsets[slot], max(nbytes, 256))

    def _k(self, key: str) -> int:
        k = self._keys.get(key)
        if k is None:
            k = len(self._names)
            self._keys[key] = k
            self._names.append(key)
        return k

    def begin(self) -> None:
        self._e.begin()

    def submit(self, slot: int, dst: torch.Tensor, src: torch.Tensor, key: str) -> None:
        """``src`` is the whole packed host block; this rank copies its stripe of it."""
        self._e.submit_striped(int(slot), src, self._k(key))

    def kernel_launches(self) -> int:
        return int(self._e.kernel_launches())

    @property
    def device_bytes(self) -> int:
        """Device memory held outside torch's allocator (the symmetric heap)."""
        return self.heap.nbytes if self.heap is not None else 0

    def submit_stripe(self, slot: int, stripe: torch.Tensor, key: str, total_bytes: int) -> None:
        """``stripe`` holds only this rank's stripe of a packed block of ``total_bytes``."""
        self._e.submit_striped(int(slot), stripe, self._k(key), int(total_bytes))

    def take_phase_samples(self) -> dict[str, float]:
        """Copy-stream time per phase (ms) summed over the transfers since the last call, in
        timing mode: ``wait_acks`` (peers still reading the slot's previous stripe),
        ``h2d_stripe`` (this rank's host-link copy), ``gather`` (publish + the peers' stripes
        over NVLink, including the wait for their flags); ``transfers`` counts them."""
        out = {"wait_acks": 0.0, "h2d_stripe": 0.0, "gather": 0.0, "transfers": 0}
        for _, a, h, g in self._e.take_phase_samples():
            out["wait_acks"] += a
            out["h2d_stripe"] += h
            out["gather"] += g
            out["transfers"] += 1
        return out

    def wait_ready(self, key: str) -> None:
        k = self._keys.get(key)
        if k is not None:
            self._e.wait_ready(k)

    def finish_use(self, slot: int) -> None:
        self._e.finish_use(int(slot))

    def join(self) -> None:
        self._e.join()

    def synchronize(self) -> None:
        self._e.synchronize()

    def reset(self) -> None:
        self._e.synchronize()

    def take_records(self):
        from flextensor_b200.runtime.engine import TransferRecord

        out = []
        for key, nbytes, tms, wms in self._e.take_samples():
            r = TransferRecord(self._names[key], nbytes)
            r.transfer_ms, r.wait_ms = tms, wms
            out.append(r)
        return out

    def close(self) -> None:
        """Free the heap once no peer can still read or write it.

        Peers read this rank's stripes and write flags/acks into its heap; the heap is an
        IPC export, so it may only be freed after (1) every peer acknowledged the latest
        stripe of every slot (bounded device-side wait) and (2) all ranks reached close
        (a barrier on the striping group, so no peer publishes into a freed heap)."""
        if self.heap is None:
            return
        import torch.distributed as dist

        try:
            self._e.drain_striped()
        finally:
            err = native.device_error(reset=False)
            if dist.is_initialized():
                dist.barrier(group=self.group)
            self.heap.close()
            self.heap = None
        if err:
            raise RuntimeError(f"striped streaming: device wait timed out (error word {err}) before the heap was freed")
