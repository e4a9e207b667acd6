"""Prefetch scheduler: per-trap ``enter``/``exit`` driving the transfer engine.

Block loader (``allocation_block_transfer`` / ``raw_block_transfer``), the
counterpart of ``src/flextensor/loaders.py:1473-1858``:

* every offloaded parameter's ``.data`` is a permanent typed view into its
  GPU ring slot, so trap boundaries never rebind tensors (no Python work per
  tensor, and a whole forward can be captured in one CUDA graph);
* ``enter(L)``: first label forks the copy stream; if L computes on streamed
  weights, the compute stream waits for them HERE (as late as possible, which
  also covers plans whose transfer was issued several traps earlier); if L is
  a transfer label, its host block is copied into its slot with ONE H2D;
* ``exit(L)``: marks L's slot free for the next writer; the last label joins.

Wrap-around transfers (compute label earlier than the transfer label) are
issued once at construction so the first forward finds them resident
(``src/flextensor/loaders.py:1508-1531``). A pass that raised before its last
label is recovered at the next pass start by draining the copy stream and
re-issuing those preloads (``src/flextensor/loaders.py:1538-1551``).

Per-tensor loader (``strategy``): each streamed tensor gets its own device
buffer from the caching allocator on the copy stream, bound at the compute
label's ``enter`` and dropped at its ``exit`` (``src/flextensor/loaders.py:677-900``).
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass, field

import torch

from flextensor_b200.config import _register_env_var
from flextensor_b200.core.host_store import HostBlock, PackedEntry
from flextensor_b200.instrumentation.core import instrumentable

logger = logging.getLogger(__name__)


@dataclass
class SlotPlan:
    order: list[str]
    transfer_slot: dict[str, int]          # transfer label -> slot
    t2c: dict[str, str]                    # transfer label -> compute label
    slot_bytes: dict[int, int]
    host_blocks: dict[str, HostBlock]      # transfer label -> packed host bytes
    preload: list[str] = field(default_factory=list)  # transfer labels to issue at construction


# Debug switches (read once at import). FT_DEBUG_CANARY=1: every locally allocated ring slot is
# framed by two 4 KB guard regions filled with 0xA5, verified after each forward, so a kernel or a
# copy that writes past its slot is reported with the slot's id instead of corrupting a neighbour.
# FT_NVTX=1: an NVTX range per trap ("ft:<label>") and per host->device block issue
# ("ft:h2d:<label>") for nsys timelines.
CANARY_BYTES = 4096
CANARY_VALUE = 0xA5
_register_env_var("FT_DEBUG_CANARY")
_register_env_var("FT_NVTX")
DEBUG_CANARY = os.environ.get("FT_DEBUG_CANARY", "0") == "1"
NVTX = os.environ.get("FT_NVTX", "0") == "1"


class SlotGuardError(RuntimeError):
    pass


@instrumentable
class BlockLoader:
    kind = "block"

    def __init__(self, device: torch.device, plan: SlotPlan, engine, timing=None, prefetch_policy=None):
        from flextensor_b200.runtime.prefetch_policy import PiecewisePrefetchPolicy

        self.device = torch.device(device)
        self.plan = plan
        self.engine = engine
        self.timing = timing
        self.policy = prefetch_policy if prefetch_policy is not None else PiecewisePrefetchPolicy()
        self.order = plan.order
        self.first = plan.order[0] if plan.order else None
        self.last = plan.order[-1] if plan.order else None
        self.c2t = {c: t for t, c in plan.t2c.items()}
        self.compute_slot = {c: plan.transfer_slot[t] for t, c in plan.t2c.items()}
        alloc = getattr(engine, "slot_tensor", None)
        self.canary = DEBUG_CANARY and alloc is None  # symmetric-heap slots have no room for guards
        self._guards: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.slots: dict[int, torch.Tensor] = {}
        for s, n in plan.slot_bytes.items():
            if alloc is not None:
                self.slots[s] = alloc(s, n)
            elif self.canary:
                size, g = max(n, 256), CANARY_BYTES
                buf = torch.empty(size + 2 * g, dtype=torch.uint8, device=self.device)
                buf[:g].fill_(CANARY_VALUE)
                buf[g + size:].fill_(CANARY_VALUE)
                self.slots[s] = buf[g:g + size]
                self._guards[s] = (buf[:g], buf[g + size:])
            else:
                self.slots[s] = torch.empty(max(n, 256), dtype=torch.uint8, device=self.device)
        self._pass_active = False
        self._closed = False

    def check_canaries(self) -> list[int]:
        """Slots whose guard regions no longer hold the fill pattern (empty without FT_DEBUG_CANARY)."""
        bad = []
        for s, (lo, hi) in self._guards.items():
            if bool((lo != CANARY_VALUE).any()) or bool((hi != CANARY_VALUE).any()):
                bad.append(s)
        return bad

    # -------------------------------------------------------------- views
    def slot_view(self, transfer_label: str, e: PackedEntry) -> torch.Tensor:
        s = self.slots[self.plan.transfer_slot[transfer_label]]
        return s[e.offset:e.offset + e.nbytes].view(e.dtype).view(e.shape)

    def bind(self, params_by_tid: dict[int, torch.nn.Parameter], setter=None) -> None:
        for t, blk in self.plan.host_blocks.items():
            for e in blk.entries:
                if setter is not None:
                    setter(e.tensor_id, self.slot_view(t, e))
                else:
                    params_by_tid[e.tensor_id].data = self.slot_view(t, e)

    def host_views(self, params_by_tid: dict[int, torch.nn.Parameter]) -> None:
        """Rebind parameters to their packed host bytes (release with preserve_model).

        A stripe-only block (striped streaming) has no whole copy on the host: its
        parameters are copied out of the device slot into fresh host tensors, one slot
        load at a time, before the slots go away.
        """
        for t, blk in self.plan.host_blocks.items():
            if not blk.stripe_only:
                for e in blk.entries:
                    params_by_tid[e.tensor_id].data = blk.view(e)
                continue
            slot = self.plan.transfer_slot[t]
            self.engine.begin()
            self._issue(t)
            self.engine.wait_ready(self.plan.t2c[t])
            self.engine.join()
            for e in blk.entries:
                params_by_tid[e.tensor_id].data = self.slot_view(t, e).to("cpu")
            self.engine.finish_use(slot)

    @property
    def blocks_bytes(self) -> int:
        return sum(t.numel() for t in self.slots.values())

    # -------------------------------------------------------------- schedule
    def _issue(self, t: str) -> None:
        blk = self.plan.host_blocks[t]
        n = blk.nbytes
        slot = self.plan.transfer_slot[t]
        if NVTX:
            torch.cuda.nvtx.range_push(f"ft:h2d:{t}")
        if blk.stripe_only:
            self.engine.submit_stripe(slot, blk.data, self.plan.t2c[t], n)
        else:
            self.engine.submit(slot, self.slots[slot][:n], blk.data, self.plan.t2c[t])
        if NVTX:
            torch.cuda.nvtx.range_pop()
        self.policy.on_schedule(t, self.plan.t2c[t])

    def preload(self) -> None:
        if not self.plan.preload:
            return
        self.engine.begin()
        for t in self.plan.preload:
            self._issue(t)
        for t in self.plan.preload:
            self.engine.wait_ready(self.plan.t2c[t])
        self.engine.join()
        self.engine.synchronize()
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()

    def recover(self) -> None:
        logger.warning("offload pass aborted before its last trap; draining copies and re-issuing preloads")
        self.engine.reset()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self._pass_active = False
        self.preload()

    def enter(self, label: str) -> None:
        if NVTX:
            torch.cuda.nvtx.range_push(f"ft:{label}")
        if label == self.first:
            if self._pass_active:
                self.recover()
            self._pass_active = True
            self.engine.begin()
            if self.timing is not None:
                self.timing.on_pass_start()
        if label in self.compute_slot:
            self.engine.wait_ready(label)
            self.policy.on_wait(label)
        if label in self.plan.transfer_slot:
            self._issue(label)
        if self.timing is not None:
            self.timing.on_enter(label)

    def exit(self, label: str) -> None:
        if self.timing is not None:
            self.timing.on_exit(label)
        if label in self.compute_slot:
            self.engine.finish_use(self.compute_slot[label])
        if label == self.last:
            self.join_after_forward()
        if NVTX:
            torch.cuda.nvtx.range_pop()

    def join_after_forward(self) -> None:
        if self._pass_active:
            self.engine.join()
            self._pass_active = False
            self.policy.on_piece_join(at_last_layer=True)
            if self.timing is not None:
                self.timing.on_pass_end(self.engine)
            if self.canary:
                bad = self.check_canaries()
                if bad:
                    raise SlotGuardError(f"ring slot(s) {bad}: a write went past the slot into its guard region")

    def piece_join(self) -> None:
        """A piecewise CUDA-graph boundary inside the forward: join the copy stream into the
        compute stream (capture needs it) and report prefetches this forces to complete."""
        if self._pass_active:
            self.engine.join()
            self.policy.on_piece_join(at_last_layer=False)

    def sync_prev_onload(self) -> None:
        self.engine.synchronize()

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        try:
            self.engine.synchronize()
        finally:
            self.slots.clear()
            close = getattr(self.engine, "close", None)
            if close is not None:
                close()


@instrumentable
class TensorStrategyLoader:
    """Per-tensor streaming: device buffers come from the caching allocator."""

    kind = "strategy"

    def __init__(self, device, order, load_strategy: dict[str, list[int]], t2c: dict[str, str],
                 host_tensors: dict[int, torch.Tensor], params_by_tid: dict[int, torch.nn.Parameter]):
        self.device = torch.device(device)
        self.order = order
        self.first = order[0] if order else None
        self.last = order[-1] if order else None
        self.load_strategy = load_strategy
        self.t2c = t2c
        self.c2t = {c: t for t, c in t2c.items()}
        self.host = host_tensors
        self.params = params_by_tid
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        self._staged: dict[str, tuple[list[tuple[int, torch.Tensor]], object]] = {}
        self.blocks_bytes = 0

    def bind(self, params_by_tid) -> None:
        for tid, t in self.host.items():
            params_by_tid[tid].data = t

    def host_views(self, params_by_tid) -> None:
        self.bind(params_by_tid)

    def preload(self) -> None:
        pass

    def enter(self, label: str) -> None:
        if label == self.first and self.cuda:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        if label in self.c2t:
            staged = self._staged.pop(label, None)
            if staged is None:  # first pass of a wrap-around transfer: load synchronously
                staged = (self._copy(self.load_strategy.get(self.c2t[label], [])), None)
            bufs, ev = staged
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
            for tid, buf in bufs:
                if self.cuda:
                    buf.record_stream(torch.cuda.current_stream(self.device))
                self.params[tid].data = buf
        if label in self.t2c:
            tids = self.load_strategy.get(label, [])
            if self.cuda:
                with torch.cuda.stream(self.stream):
                    bufs = self._copy(tids)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
            else:
                bufs, ev = self._copy(tids), None
            self._staged[self.t2c[label]] = (bufs, ev)

    def _copy(self, tids):
        return [(tid, self.host[tid].to(self.device, non_blocking=True)) for tid in tids]

    def exit(self, label: str) -> None:
        if label in self.c2t:
            for tid in self.load_strategy.get(self.c2t[label], []):
                self.params[tid].data = self.host[tid]
        if label == self.last and self.cuda:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)

    def join_after_forward(self) -> None:
        if self.cuda:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)

    def sync_prev_onload(self) -> None:
        if self.cuda:
            self.stream.synchronize()

    def close(self) -> None:
        self._staged.clear()
