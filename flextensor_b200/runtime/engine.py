"""Transfer engine: ring-slot H2D ordering on a dedicated copy stream.

Contract (same ordering rules as ``src/flextensor/core/transfer.py:26-146``):

* ``begin()`` forks the copy stream from the compute stream (so a CUDA-graph
  capture that starts on the compute stream also captures the copies);
* ``submit(slot, dst, src, key)`` makes the copy stream wait until the slot's
  previous reader finished (``finish_use``), issues the H2D, and records a
  ready event under ``key`` (the compute label that will read it);
* ``wait_ready(key)`` makes the compute stream wait for that copy;
* ``finish_use(slot)`` records "slot no longer read" on the compute stream;
* ``join()`` merges the copy stream back into the compute stream.

On CUDA devices the native engine in ``flextensor_b200._C`` (C++, CUDA runtime
API) is used: one call per trap boundary, no Python-side event objects. The
pure-Python engine here is the CPU-device implementation (the CPU plumbing
configuration) and the specification the native one is tested against.

Stall measurement: with ``timing=True`` the engine records an event on the
compute stream right before and right after every ready-wait; the elapsed time
between the two is the time compute sat idle waiting for a copy (exposed
transfer), and copy-stream start/end events give each transfer's duration.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from flextensor_b200.instrumentation.core import instrumentable


@dataclass
class TransferRecord:
    key: str
    nbytes: int
    start: object = None
    end: object = None
    wait_start: object = None
    wait_end: object = None
    transfer_ms: float | None = None   # precomputed by the native engine
    wait_ms: float | None = None


@instrumentable
class PyTransferEngine:
    """Reference engine; exact on CPU (synchronous copies), event-ordered on CUDA."""

    def __init__(self, device: torch.device, n_slots: int, timing: bool = False, external_events: bool = False):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.n_slots = n_slots
        self.timing = timing and self.cuda
        self._external = external_events
        if self.cuda:
            self.copy_stream = torch.cuda.Stream(device=self.device, priority=-1)
            self._slot_free = [None] * n_slots
            self._ready: dict[str, torch.cuda.Event] = {}
        self.records: dict[str, TransferRecord] = {}
        self.pending_keys: set[str] = set()

    def _event(self, timing: bool = False):
        if self._external:
            return torch.cuda.Event(enable_timing=timing, external=True)
        return torch.cuda.Event(enable_timing=timing)

    def begin(self) -> None:
        if self.cuda:
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))

    def submit(self, slot: int, dst: torch.Tensor, src: torch.Tensor, key: str) -> None:
        rec = TransferRecord(key, src.numel() * src.element_size())
        if not self.cuda:
            dst.copy_(src)
            self.records[key] = rec
            self.pending_keys.add(key)
            return
        with torch.cuda.stream(self.copy_stream):
            ev = self._slot_free[slot]
            if ev is not None:
                self.copy_stream.wait_event(ev)
            if self.timing:
                rec.start = self._event(True)
                rec.start.record(self.copy_stream)
            dst.copy_(src, non_blocking=True)
            ready = self._event(self.timing)
            ready.record(self.copy_stream)
            if self.timing:
                rec.end = ready
        self._ready[key] = ready
        self.records[key] = rec
        self.pending_keys.add(key)

    def wait_ready(self, key: str) -> None:
        self.pending_keys.discard(key)
        if not self.cuda:
            return
        ev = self._ready.get(key)
        if ev is None:
            return
        cs = torch.cuda.current_stream(self.device)
        rec = self.records.get(key)
        if self.timing and rec is not None:
            rec.wait_start = self._event(True)
            rec.wait_start.record(cs)
        cs.wait_event(ev)
        if self.timing and rec is not None:
            rec.wait_end = self._event(True)
            rec.wait_end.record(cs)

    def finish_use(self, slot: int) -> None:
        if not self.cuda:
            return
        ev = self._event(False)
        ev.record(torch.cuda.current_stream(self.device))
        self._slot_free[slot] = ev

    def join(self) -> None:
        if self.cuda:
            torch.cuda.current_stream(self.device).wait_stream(self.copy_stream)

    def synchronize(self) -> None:
        if self.cuda:
            self.copy_stream.synchronize()

    def reset(self) -> None:
        """Forget tickets after an aborted pass (copies already issued still complete)."""
        self.synchronize()
        self.pending_keys.clear()

    def take_records(self) -> list[TransferRecord]:
        out = list(self.records.values())
        self.records = {}
        return out


def make_engine(device: torch.device, n_slots: int, timing: bool = False, external_events: bool = False):
    """Native engine on CUDA devices (fails loudly if the extension is missing), Python on CPU."""
    device = torch.device(device)
    if device.type == "cuda":
        from flextensor_b200.ops import native

        return native.NativeTransferEngine(device, n_slots, timing=timing, external_events=external_events)
    return PyTransferEngine(device, n_slots, timing=timing)
