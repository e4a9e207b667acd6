"""TensorManager: the per-model engine behind the DISCOVERY -> PROFILING -> INFERENCE phases.

Phase work (reference: ``src/flextensor/tensor_manager.py:827-915``, ``1661-1800``):

* ``initialize_warmup`` (DISCOVERY): every offloadable unit parameter moves to
  (pinned) host memory; all other parameters and buffers move to the device.
  Discovery traps materialise their own tensors on the device for the duration
  of the trap and record any *other* unit's host tensor the forward touches
  (``__torch_function__``); such cross-unit tensors become resident, because a
  streamed tensor may only belong to one trap.
* ``initialize_profile`` (PROFILING): ``view`` mode stages each trap's tensors
  into one reusable device buffer with ONE H2D, synchronises, then times only
  the compute with CUDA events; ``getter``/``torch_function`` copy tensor by
  tensor.
* ``initialize_inference``: median durations + per-tensor H2D costs ->
  :class:`LayerStatistics`; a size-sweep H2D benchmark feeds the interpolator;
  the strategy plans under the memory budget; host blocks are packed and
  parameters are bound to ring-slot views.

The plan round-trips through :class:`TensorManagerState` (``profile.json`` v3)
and is restored by tensor *name*.
"""

from __future__ import annotations

import contextlib
import logging
import time
from enum import Enum
from typing import Any

import torch
from torch import nn
from torch.overrides import TorchFunctionMode

from flextensor_b200.core.host_store import HostBlock, make_host_pinner, pack_tensors, tensor_nbytes
from flextensor_b200.core.state import PROFILE_FILENAME, TensorManagerState
from flextensor_b200.core.stats import (
    IterativeLayerStatisticsCollector,
    LayerStatistics,
    TensorStatistics,
    compute_layer_statistics,
)
from flextensor_b200.planner.common import calculate_transfer_to_compute_map
from flextensor_b200.planner.protocol import Strategy, StrategyResult
from flextensor_b200.runtime.engine import make_engine
from flextensor_b200.runtime.loaders import BlockLoader, SlotPlan, TensorStrategyLoader
from flextensor_b200.runtime.timing import OffloadTimingCollector
from flextensor_b200.runtime.units import Unit
from flextensor_b200.types import GPUMemoryUsage
from flextensor_b200.instrumentation.core import instrumentable

logger = logging.getLogger(__name__)


class TMPhase(Enum):
    NONE = 0
    DISCOVERY = 1
    PROFILING = 2
    INFERENCE = 3


class TrapNestingError(RuntimeError):
    pass


class _ForeignReadMode(TorchFunctionMode):
    """During discovery: move host tensors of *other* units to the device and record them."""

    def __init__(self, tm: "TensorManager", label: str):
        super().__init__()
        self.tm, self.label = tm, label
        self.cache: dict[int, torch.Tensor] = {}

    def _swap(self, x):
        if isinstance(x, torch.Tensor) and self.tm._held_ptr_to_tid and x.device == self.tm.device:
            # a device-held weight is read in place; a read from another unit's trap is recorded
            tid = self.tm._held_ptr_to_tid.get(x.data_ptr())
            if tid is not None and self.tm.owner.get(tid) != self.label:
                self.tm._foreign_reads.setdefault(tid, set()).add(self.label)
            return x
        if isinstance(x, torch.Tensor) and x.device.type == "cpu" and self.tm.device.type != "cpu":
            tid = self.tm._host_ptr_to_tid.get(x.data_ptr())
            if tid is not None:
                self.tm._foreign_reads.setdefault(tid, set()).add(self.label)
                d = self.cache.get(tid)
                if d is None:
                    d = x.to(self.tm.device, non_blocking=True)
                    if self.tm.use_trace_tensor:
                        from flextensor_b200.runtime.benchmark_modes import wrap_trace_tensor

                        d = wrap_trace_tensor(d, self.tm.id_to_name.get(tid))
                    self.cache[tid] = d
                return d
        return x

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        args = torch.utils._pytree.tree_map(self._swap, args)
        kwargs = torch.utils._pytree.tree_map(self._swap, kwargs)
        return func(*args, **kwargs)


@instrumentable
class TensorManager:
    """Owns tensors, traps, plan and loader for one model."""

    def __init__(
        self,
        device_gpu: str | torch.device,
        tensor_manager_load_strategy: Strategy,
        loader_type: str = "allocation_block_transfer",
        remove_layers_operations: list[dict[str, Any]] | None = None,
        blocks: int = 4,
        move_top_level_buffers_to_gpu: bool = True,
        *,
        pinned_memory: bool = True,
        pinned_memory_mode: str = "torch",
        profile_mode: str = "view",
        max_gpu_mem_fraction: float | None = None,
        hold_device_weights: bool = True,
        offload_timing: str = "off",
        enable_diagnostics: bool = False,
        shm_store: Any = None,
        piecewise_prefetch: str = "warn",
        _compute_transfer_gap: int | None = None,
        _direct_mode: bool = True,
        _use_trace_tensor: bool = False,
        _rearrange_transfers: bool | None = None,
        _enable_untraced_tensor_discovery: bool = True,
        _offload_timing_log_every: int = 0,
        _offload_timing_measure_max_passes: int = 1024,
    ) -> None:
        self.device = torch.device(device_gpu)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.strategy = tensor_manager_load_strategy
        self.loader_type = loader_type
        self.remove_layers_operations = remove_layers_operations or []
        self.blocks = blocks
        self.move_top_level_buffers_to_gpu = move_top_level_buffers_to_gpu
        self.pinned_memory = pinned_memory and self.device.type == "cuda"
        self.pinner = make_host_pinner(self.pinned_memory, pinned_memory_mode)
        self.profile_mode = profile_mode
        self.max_gpu_mem_fraction = max_gpu_mem_fraction
        self.hold_device_weights = hold_device_weights
        self.offload_timing = offload_timing
        self.enable_diagnostics = enable_diagnostics
        self.shm_store = shm_store
        self.piecewise_prefetch = piecewise_prefetch
        self.rearrange = bool(_rearrange_transfers)
        self.compute_transfer_gap = _compute_transfer_gap
        self.phase = TMPhase.NONE

        self.model: nn.Module | None = None
        self.units: list[Unit] = []
        self.labels: list[str] = []
        self.id_to_name: dict[int, str] = {}
        self.name_to_id: dict[str, int] = {}
        self.params_by_tid: dict[int, nn.Parameter] = {}
        self.owner: dict[int, str] = {}                # offloadable tid -> unit label
        self.unit_tids: dict[str, list[int]] = {}
        self.host: dict[int, torch.Tensor] = {}        # offloadable tid -> host tensor
        self._host_ptr_to_tid: dict[int, int] = {}
        self._held_ptr_to_tid: dict[int, int] = {}     # device-held unit weights (see warmup)
        self.resident: set[int] = set()                # tids permanently on device
        self._foreign_reads: dict[int, set[str]] = {}
        self.collector = IterativeLayerStatisticsCollector()
        self._trap_depth = 0
        self._suspend = 0
        self._staging: torch.Tensor | None = None
        self.loader: BlockLoader | TensorStrategyLoader | None = None
        self.state: TensorManagerState | None = None
        self.layer_stats: list[LayerStatistics] = []
        self.memory_stats: dict[int, float] | None = None
        self.strategy_result: StrategyResult | None = None
        self.timing = OffloadTimingCollector(self.device, offload_timing) if offload_timing != "off" else None
        self._orig_device: dict[int, torch.device] = {}
        self.unmapped_bytes = 0
        self.load_from_shm = False
        self._state_restored_from_profile = False
        self._stripe = None
        self.use_trace_tensor = bool(_use_trace_tensor)
        if self.use_trace_tensor and profile_mode == "view":
            raise ValueError("profile_mode='view' is incompatible with _use_trace_tensor=True "
                             "(view profiling rebinds parameters into a staging buffer)")

    # ================================================================== model / units
    def set_model(self, model: nn.Module) -> None:
        self.model = model
        names = [n for n, _ in model.named_parameters(remove_duplicate=True)]
        self.id_to_name = dict(enumerate(names))
        self.name_to_id = {n: i for i, n in self.id_to_name.items()}
        self.params_by_tid = {self.name_to_id[n]: p for n, p in model.named_parameters(remove_duplicate=True)}

    def set_units(self, units: list[Unit]) -> None:
        self.units = units
        self.labels = [u.label for u in units]
        pid_to_tid = {id(p): t for t, p in self.params_by_tid.items()}
        self.owner, self.unit_tids = {}, {}
        for u in units:
            tids = [pid_to_tid[id(p)] for _, p in u.params if id(p) in pid_to_tid]
            self.unit_tids[u.label] = tids
            for t in tids:
                self.owner[t] = u.label

    def build_parameters_mapping(self, model: nn.Module | dict[str, torch.Tensor]) -> None:
        if isinstance(model, nn.Module):
            self.set_model(model)

    # ================================================================== placement helpers
    def _to_host(self, tid: int) -> None:
        p = self.params_by_tid[tid]
        self._orig_device.setdefault(tid, p.device)
        t = p.data
        p.requires_grad_(False)
        if t.device.type == "meta":
            # follower of a shared store: bytes arrive from SHM weight blocks later
            self.host[tid] = t
            return
        if t.device.type != "cpu":
            t = t.to("cpu")
        if self.pinned_memory:
            t = self.pinner.pin(t)
        p.data = t
        self.host[tid] = t
        self._host_ptr_to_tid[t.data_ptr()] = tid

    def _hold(self, tid: int) -> None:
        """Keep a unit weight that starts on the compute device where it is until the plan exists.

        Discovery and profiling then read it in place, and the plan's streamed weights are
        packed straight from the device into the pinned arena (or this rank's stripe of it),
        so the host never holds a second, per-tensor copy of the model. The bytes count as
        obtainable in the memory-mode budget, since every streamed weight is freed after packing."""
        p = self.params_by_tid[tid]
        self._orig_device.setdefault(tid, p.device)
        p.requires_grad_(False)
        self.host[tid] = p.data
        self._held_ptr_to_tid[p.data.data_ptr()] = tid

    def _held_bytes(self) -> int:
        return sum(tensor_nbytes(h) for h in self.host.values() if h.device == self.device)

    def _to_device(self, tid: int) -> None:
        p = self.params_by_tid[tid]
        self._orig_device.setdefault(tid, p.device)
        if p.device != self.device:
            p.data = p.data.to(self.device)
        self.resident.add(tid)
        old = self.host.pop(tid, None)
        if old is not None:
            self._host_ptr_to_tid.pop(old.data_ptr(), None)
            self._held_ptr_to_tid.pop(old.data_ptr(), None)

    def _move_non_unit_to_device(self) -> None:
        for tid in self.params_by_tid:
            if tid not in self.owner:
                self._to_device(tid)
        for _, b in self.model.named_buffers():
            if b.device != self.device:
                b.data = b.data.to(self.device)
        if self.move_top_level_buffers_to_gpu:
            self._move_attribute_tensors()

    def _move_attribute_tensors(self) -> None:
        """Tensors the model holds outside its registered parameters and buffers follow it to
        the device, as the reference's unmapped-tensor processor does
        (``tensor_processors.py:686-744``): plain module attributes (a cached frequency table),
        tensors nested in lists / tuples / dicts / sets / helper objects at any depth, and the
        tensor-valued inner fields of parameters (``weight.weight_scale`` of a quantized layer).
        A tensor reachable from several places is moved once and every place gets the copy."""
        from flextensor_b200.core.visitor import TensorVisitor, carry_inner_fields

        moved: dict[int, torch.Tensor] = {}
        offloaded = {id(p) for tid, p in self.params_by_tid.items() if tid in self.owner}

        def to_dev(t: torch.Tensor) -> torch.Tensor:
            if t.is_meta or t.device == self.device or id(t) in offloaded:
                return t
            if id(t) not in moved:
                moved[id(t)] = t.to(self.device)
            return moved[id(t)]

        TensorVisitor(to_dev, params=False, buffers=False, attributes=True).apply(self.model)
        for p in self.params_by_tid.values():
            carry_inner_fields(p, p, to_dev)

    # ================================================================== phases
    def _striping(self):
        """(group, rank, world) when striped streaming applies to this manager, else None."""
        if self.device.type != "cuda" or self.loader_type == "strategy" or self.shm_store is not None:
            return None
        from flextensor_b200.parallel.striped import striping_group

        g = striping_group()
        if g is None:
            return None
        import torch.distributed as dist

        return g, dist.get_rank(g), dist.get_world_size(g)

    def initialize_warmup(self, keep_on_device: set[int] | None = None) -> nn.Module:
        """Move every offloadable tensor to the host and everything else to the device.

        ``keep_on_device``: tensor ids a restored plan keeps resident; they go straight to
        the device instead of making a host round trip (state adoption)."""
        assert self.model is not None, "set_model first"
        self._stripe = self._striping()
        with torch.no_grad():
            for tid in self.owner:
                p = self.params_by_tid[tid]
                if keep_on_device is not None and tid in keep_on_device:
                    self._to_device(tid)
                    continue
                if p.device == self.device and self.device.type == "cuda" and (
                        self._stripe is not None or self.hold_device_weights):
                    self._hold(tid)
                    continue
                self._to_host(tid)
            self._move_non_unit_to_device()
        self.phase = TMPhase.DISCOVERY
        return self.model

    def static_discovery(self) -> None:
        """skip_discovery: a trap's tensors are exactly its unit's parameters."""
        for label, tids in self.unit_tids.items():
            self.collector.record_tensors(label, tids)

    def initialize_profile(self) -> nn.Module:
        # cross-unit reads seen in discovery -> resident
        for tid, readers in self._foreign_reads.items():
            if tid in self.owner:
                logger.info("tensor %s is read by %s outside its trap; keeping it resident",
                            self.id_to_name[tid], sorted(readers))
                with torch.no_grad():
                    self._to_device(tid)
                for label in list(self.unit_tids):
                    if tid in self.unit_tids[label]:
                        self.unit_tids[label].remove(tid)
                self.owner.pop(tid, None)
        for label in self.labels:
            if label not in self.collector.labels():
                self.collector.record_tensors(label, self.unit_tids.get(label, []))
        if self.profile_mode == "view":
            need = max((self._trap_bytes(l) for l in self.labels), default=0)
            self._staging = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        elif self.profile_mode == "getter":
            from flextensor_b200.runtime.getter_profile import GetterProfile

            self._getter = GetterProfile(self)
            self._getter.install()
        self.phase = TMPhase.PROFILING
        return self.model

    def is_traced(self, t) -> bool:
        """Whether ``t`` is a tensor this manager manages: with ``_use_trace_tensor`` a
        :class:`~flextensor_b200.runtime.benchmark_modes.TraceTensor` mark, otherwise one of the
        model's offloadable parameters (by identity)."""
        if self.use_trace_tensor:
            from flextensor_b200.runtime.benchmark_modes import is_trace_tensor

            if is_trace_tensor(t):
                return True
        return any(t is self.params_by_tid[tid] for tid in self.owner)

    def promote_resident(self, tid: int) -> None:
        """Keep tensor ``tid`` on the device for good (read outside its own trap)."""
        with torch.no_grad():
            self._to_device(tid)
        for label in list(self.unit_tids):
            if tid in self.unit_tids[label]:
                self.unit_tids[label].remove(tid)
        self.owner.pop(tid, None)

    def _drop_getters(self) -> None:
        g = getattr(self, "_getter", None)
        if g is not None:
            g.uninstall()
            self._getter = None

    def _offloadable(self, label: str) -> list[int]:
        return [t for t in self.unit_tids.get(label, []) if t in self.host]

    def _trap_bytes(self, label: str) -> int:
        from flextensor_b200.core.host_store import packed_layout

        return packed_layout([tensor_nbytes(self.host[t]) for t in self._offloadable(label)])[1]

    # ================================================================== traps
    def is_profiling_suspended(self) -> bool:
        return self._suspend > 0

    def suspend_profiling(self) -> None:
        self._suspend += 1

    def resume_profiling(self) -> None:
        if self._suspend <= 0:
            raise RuntimeError("resume_profiling() without a matching suspend_profiling()")
        self._suspend -= 1

    @contextlib.contextmanager
    def pause_profiling(self):
        self.suspend_profiling()
        try:
            yield
        finally:
            self.resume_profiling()

    def clear_profiling_durations(self) -> None:
        self.collector.clear_durations()

    @contextlib.contextmanager
    def trap(self, name: str):
        if self._trap_depth:
            raise TrapNestingError(f"nested trap {name!r}: offload units may not contain each other")
        self._trap_depth += 1
        try:
            if self.phase == TMPhase.DISCOVERY:
                with self._discovery_trap(name):
                    yield
            elif self.phase == TMPhase.PROFILING:
                with self._profile_trap(name):
                    yield
            elif self.phase == TMPhase.INFERENCE and self.loader is not None:
                self.loader.enter(name)
                try:
                    yield
                finally:
                    self.loader.exit(name)
            else:
                yield
        finally:
            self._trap_depth -= 1

    @contextlib.contextmanager
    def _discovery_trap(self, label: str):
        tids = self._offloadable(label)
        with torch.no_grad():
            for t in tids:
                self.params_by_tid[t].data = self.host[t].to(self.device, non_blocking=True)
        mode = _ForeignReadMode(self, label)
        try:
            with mode:
                yield
        finally:
            if self.device.type == "cuda":
                torch.cuda.current_stream(self.device).synchronize()
            for t in tids:
                self.params_by_tid[t].data = self.host[t]
            self.collector.record_tensors(label, self.unit_tids.get(label, []))

    def _now_events(self):
        if self.device.type == "cuda":
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            return a, b
        return None, None

    @contextlib.contextmanager
    def _profile_trap(self, label: str):
        tids = self._offloadable(label)
        cuda = self.device.type == "cuda"
        getter = getattr(self, "_getter", None)
        with torch.no_grad():
            if getter is not None:
                getter.load(tids)  # served by the module's property getters; Parameters untouched
            elif self.profile_mode == "view" and self._staging is not None:
                from flextensor_b200.core.host_store import packed_layout

                offs, _ = packed_layout([tensor_nbytes(self.host[t]) for t in tids])
                for t, o in zip(tids, offs):
                    h = self.host[t]
                    v = self._staging[o:o + tensor_nbytes(h)].view(h.dtype).view(h.shape)
                    v.copy_(h, non_blocking=True)
                    self.params_by_tid[t].data = v
            else:
                for t in tids:
                    self.params_by_tid[t].data = self.host[t].to(self.device, non_blocking=True)
        if cuda:
            torch.cuda.current_stream(self.device).synchronize()
            start, end = self._now_events()
            start.record()
        t0 = time.perf_counter()
        try:
            yield
        finally:
            if cuda:
                end.record()
                end.synchronize()
                ms = start.elapsed_time(end)
            else:
                ms = (time.perf_counter() - t0) * 1e3
            if getter is not None:
                getter.unload(tids)
            else:
                for t in tids:
                    self.params_by_tid[t].data = self.host[t]
            if not self.is_profiling_suspended():
                self.collector.record_duration(label, ms)

    # ================================================================== inference planning
    def _benchmark_sizes(self, sizes: list[int], reps: int = 3) -> dict[int, float]:
        """Median H2D ms per size from pinned host memory (CPU device: memcpy timing)."""
        from flextensor_b200.core.host_store import alloc_host_bytes

        out: dict[int, float] = {}
        if not sizes:
            return out
        big = max(sizes)
        src = alloc_host_bytes(big, self.pinned_memory)
        dst = torch.empty(big, dtype=torch.uint8, device=self.device)
        for s in sorted(set(sizes)):
            samples = []
            for _ in range(reps):
                if self.device.type == "cuda":
                    a, b = self._now_events()
                    a.record()
                    dst[:s].copy_(src[:s], non_blocking=True)
                    b.record()
                    b.synchronize()
                    samples.append(a.elapsed_time(b))
                else:
                    t0 = time.perf_counter()
                    dst[:s].copy_(src[:s])
                    samples.append(max((time.perf_counter() - t0) * 1e3, 1e-6))
            samples.sort()
            out[s] = max(samples[len(samples) // 2], 1e-6)
        del src, dst
        return out

    def estimate_unit_durations(self) -> dict[str, float]:
        """Per-unit duration estimate: the measured H2D time of the unit's own bytes."""
        sizes = {l: self._trap_bytes(l) for l in self.labels}
        ms = self._benchmark_sizes(sorted({max(n, 1) for n in sizes.values()}), reps=3)
        return {l: ms[max(n, 1)] for l, n in sizes.items()}

    def get_memory_transfer_stats(self) -> dict[int, float] | None:
        return self.memory_stats

    def benchmark_memory_transfers(self, max_bytes: int) -> dict[int, float]:
        """Power-of-two size sweep up to the largest label (capped at 4 GiB)."""
        top = min(max(max_bytes, 1 << 20), 4 << 30)
        sizes, s = [], 1 << 16
        while s < top:
            sizes.append(s)
            s <<= 1
        sizes.append(top)
        return self._benchmark_sizes(sizes)

    def _tensor_statistics(self) -> dict[int, TensorStatistics]:
        sizes = {tensor_nbytes(self.host[t]) for t in self.host}
        ms = self._benchmark_sizes(sorted(sizes), reps=3)
        return {t: TensorStatistics(tensor_id=t, name=self.id_to_name[t], size_bytes=tensor_nbytes(h),
                                    load_time_ms=ms[tensor_nbytes(h)]) for t, h in self.host.items()}

    def _gpu_budget(self) -> int | None:
        if self.max_gpu_mem_fraction is None:
            return None
        from flextensor_b200.runtime.gpu_budget import resolve_gpu_budget

        invisible = sum(tensor_nbytes(self.params_by_tid[t].data) for t in self.resident if t not in self.owner)
        invisible += sum(b.numel() * b.element_size() for b in self.model.buffers())
        return resolve_gpu_budget(self.device, self.max_gpu_mem_fraction, invisible,
                                  reclaimable_bytes=self._held_bytes())

    def initialize_inference(self) -> nn.Module:
        self._staging = None
        self._drop_getters()
        rows = [r for r in self.collector.get_layer_stats() if r.label in self.unit_tids]
        from flextensor_b200.runtime.profiling_quality import report_profiling_quality

        report_profiling_quality(self.collector, verbose=self.enable_diagnostics)
        tstats = self._tensor_statistics()
        tstats = {t: s for t, s in tstats.items() if t in self.owner}
        self.layer_stats = compute_layer_statistics(rows, tstats)
        if self.remove_layers_operations:
            from flextensor_b200.planner.operations import remove_layers_compound

            ops = [o for o in self.remove_layers_operations if o.get("op") == "remove"]
            self.layer_stats = remove_layers_compound(self.layer_stats, ops)
        max_label = max((sum(t.size_bytes for t in l.tensors) for l in self.layer_stats), default=1 << 20)
        self.memory_stats = self.benchmark_memory_transfers(max_label)
        budget = self._gpu_budget()
        result = self.strategy.compute(self.layer_stats, self.memory_stats, budget)
        if self.rearrange and result.strategy_map and self.loader_type != "strategy":
            result = self._rearranged(result)
        result = self._agree_on_plan(result)
        self.strategy_result = result
        self._build_from_result(result)
        if self.enable_diagnostics:
            from flextensor_b200.runtime.diagnostics import log_plan

            log_plan(self)
        return self.model

    def _rearranged(self, result: StrategyResult) -> StrategyResult:
        """Move transfers to the latest earlier trap that hides them (free traps only)."""
        from flextensor_b200.planner.common import build_block_data, calculate_transfer_to_compute_map
        from flextensor_b200.planner.interpolator import create_interpolator_from_benchmarks
        from flextensor_b200.planner.operations import rearrange_transfers

        interp = create_interpolator_from_benchmarks(self.memory_stats) if self.memory_stats else None
        t2c = calculate_transfer_to_compute_map(self.layer_stats, result.strategy_map)
        plan, _ = rearrange_transfers(result.strategy_map, t2c, self.layer_stats, interp,
                                      gap=self.compute_transfer_gap or 1)
        return StrategyResult(plan, build_block_data(plan, self.layer_stats, self.blocks))

    def _agree_on_plan(self, result: StrategyResult) -> StrategyResult:
        """With striped streaming every rank must run rank 0's plan (same slots, same epochs)."""
        if self.device.type != "cuda":
            return result
        from flextensor_b200.parallel.striped import striping_group

        group = striping_group()
        if group is None:
            return result
        import torch.distributed as dist

        box = [result, self.layer_stats] if dist.get_rank(group) == 0 else [None, None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(box, src=src, group=group)
        plan, stats = box
        # rebind tensor ids by name (ids are positional and identical for identical models)
        if [l.label for l in stats] != [l.label for l in self.layer_stats]:
            raise RuntimeError("striped streaming needs identical offload units on every rank")
        self.layer_stats = stats
        return plan

    # ---------------------------------------------------------------- plan -> runtime
    def _build_from_result(self, result: StrategyResult) -> None:
        order = [l.label for l in self.layer_stats]
        load = {k: [t.tensor_id for t in v] for k, v in result.strategy_map.items() if v}
        t2c = (result.block_data.transfer_to_compute_map if result.block_data is not None
               else calculate_transfer_to_compute_map(self.layer_stats, result.strategy_map))
        l2b = result.block_data.label_to_block_id if result.block_data is not None else {}
        self._build_runtime(order, load, t2c, l2b)
        self.state = self.export_state()

    def _build_runtime(self, order: list[str], load: dict[str, list[int]], t2c: dict[str, str],
                       l2b: dict[str, int]) -> None:
        streamed = {t for ts in load.values() for t in ts}
        with torch.no_grad():
            for tid in list(self.host):
                if tid not in streamed:
                    self._to_device(tid)
        self.unmapped_bytes = sum(tensor_nbytes(self.params_by_tid[t].data) for t in self.resident)
        idx = {l: i for i, l in enumerate(order)}
        if self.loader_type == "strategy":
            for tid in streamed:  # the per-tensor loader streams from pinned host copies
                if self.host[tid].device == self.device:
                    self._held_ptr_to_tid.pop(self.host[tid].data_ptr(), None)
                    self._to_host(tid)
            if self.device.type == "cuda":
                torch.cuda.empty_cache()
            self.loader = TensorStrategyLoader(self.device, order, load, {k: t2c[k] for k in load}, dict(self.host),
                                               self.params_by_tid)
            self.loader.bind(self.params_by_tid)
            self.phase = TMPhase.INFERENCE
            return
        host_blocks: dict[str, HostBlock] = {}
        # One pinned arena for every packed block (a per-block pinned allocation would be rounded
        # up to a power of two by the caching host allocator).
        from flextensor_b200.core.host_store import alloc_host_bytes, packed_layout

        stripe = getattr(self, "_stripe", None)
        if stripe is not None:
            from flextensor_b200.core.host_store import pack_tensors_stripe, stripe_range

            _, rank, world = stripe
            spans = {}
            for label in order:
                if load.get(label):
                    tot = packed_layout([tensor_nbytes(self.host[t]) for t in load[label]])[1]
                    b0, b1 = stripe_range(tot, rank, world)
                    spans[label] = (b1 - b0 + 255) // 256 * 256
            arena = alloc_host_bytes(max(sum(spans.values()), 256), self.pinned_memory)
            off = 0
            with torch.no_grad():
                for label in order:
                    if label not in spans:
                        continue
                    items = [(t, self.id_to_name[t], self.host[t]) for t in load[label]]
                    host_blocks[label] = pack_tensors_stripe(
                        label, items, rank, world, pinned=self.pinned_memory,
                        buffer=arena[off:off + spans[label]])
                    off += spans[label]
                    for t, _, h in items:  # drop the device source; the stripe + slot hold it now
                        self.host[t] = torch.empty(h.shape, dtype=h.dtype, device="meta")
        arena, arena_off = None, 0
        if self.shm_store is None and stripe is None:
            need = sum(packed_layout([tensor_nbytes(self.host[t]) for t in load[l]])[1]
                       for l in order if load.get(l))
            if need:
                arena = alloc_host_bytes(need, self.pinned_memory)
        for label in order:
            tids = load.get(label)
            if not tids or label in host_blocks:
                continue
            items = [(t, self.id_to_name[t], self.host[t]) for t in tids]
            if arena is not None:
                sz = packed_layout([tensor_nbytes(h) for _, _, h in items])[1]
                blk = pack_tensors(label, items, buffer=arena[arena_off:arena_off + sz], pinned=self.pinned_memory,
                                   release_sources=self._release_host)
                arena_off += sz
                host_blocks[label] = blk
                self._rebind_to_block(blk)
                continue
            buf = (self.shm_store.block_buffer(label, items, must_exist=self.load_from_shm)
                   if self.shm_store is not None else None)
            if buf is not None and self.load_from_shm:
                from flextensor_b200.core.host_store import PackedEntry, packed_layout

                offs, _ = packed_layout([tensor_nbytes(h) for _, _, h in items])
                blk = HostBlock(label, buf, [PackedEntry(t, n, o, tensor_nbytes(h), h.dtype, tuple(h.shape))
                                             for (t, n, h), o in zip(items, offs)])
            else:
                blk = pack_tensors(label, items, buffer=buf, pinned=self.pinned_memory,
                                   release_sources=self._release_host)
                self._rebind_to_block(blk)
            host_blocks[label] = blk
        slot_of = {l: l2b.get(l, i % max(2, self.blocks)) for i, l in enumerate(host_blocks)}
        slot_bytes: dict[int, int] = {}
        for l, b in slot_of.items():
            slot_bytes[b] = max(slot_bytes.get(b, 0), host_blocks[l].nbytes)
        preload = [t for t in host_blocks if idx[t2c[t]] <= idx[t]]
        plan = SlotPlan(order=order, transfer_slot=slot_of, t2c={t: t2c[t] for t in host_blocks},
                        slot_bytes=slot_bytes, host_blocks=host_blocks, preload=preload)
        engine = None
        if self.device.type == "cuda":
            from flextensor_b200.parallel.striped import StripedTransferEngine, striping_group

            group = striping_group()
            if group is not None and self.loader_type != "strategy":
                engine = StripedTransferEngine(self.device, slot_bytes, group, timing=self.timing is not None)
        if engine is None:
            engine = make_engine(self.device, max(slot_bytes, default=0) + 1,
                                 timing=self.timing is not None, external_events=self.offload_timing == "cuda_graph")
        from flextensor_b200.runtime.prefetch_policy import PiecewisePrefetchPolicy

        self.loader = BlockLoader(self.device, plan, engine, timing=self.timing,
                                  prefetch_policy=PiecewisePrefetchPolicy.from_mode(self.piecewise_prefetch))
        self.loader.bind(self.params_by_tid, setter=self._set_param)
        if self.device.type == "cuda":
            # the per-tensor sources that were packed are free now: device-held weights go back
            # to the device allocator, per-tensor pinned copies to the pinned host cache
            torch.cuda.empty_cache()
            if self.pinned_memory and hasattr(torch._C, "_host_emptyCache"):
                torch._C._host_emptyCache()
        self.loader.preload()
        self.phase = TMPhase.INFERENCE

    def _set_param(self, tid: int, t: torch.Tensor) -> None:
        """Point parameter ``tid`` at ``t``; a ``meta`` parameter (SHM follower) is replaced by a new one."""
        p = self.params_by_tid[tid]
        if not p.is_meta:
            p.data = t
            return
        newp = nn.Parameter(t, requires_grad=False)
        from flextensor_b200.core.visitor import carry_inner_fields

        carry_inner_fields(p, newp)  # loader metadata (weight_loader, output_dim, ...) stays
        name = self.id_to_name[tid]
        for n, q in list(self.model.named_parameters(remove_duplicate=False)):
            if q is p:
                mod_path, _, leaf = n.rpartition(".")
                mod = self.model.get_submodule(mod_path) if mod_path else self.model
                setattr(mod, leaf, newp)
        self.params_by_tid[tid] = newp
        _ = name

    def _release_host(self, tid: int) -> None:
        old = self.host.get(tid)
        if old is not None:
            self._host_ptr_to_tid.pop(old.data_ptr(), None)
            self._held_ptr_to_tid.pop(old.data_ptr(), None)

    def _rebind_to_block(self, blk: HostBlock) -> None:
        """Point each packed tensor's host entry and parameter at its bytes in ``blk``.

        The per-tensor source (a pinned host copy or a device-held weight) then has no
        reference left and is freed; one in-place ``cudaHostRegister`` is undone first."""
        for e in blk.entries:
            old = self.host.get(e.tensor_id)
            v = blk.view(e)
            if old is not None and old.device.type == "cpu" and old.data_ptr() != v.data_ptr():
                self.pinner.registry.release(old.data_ptr())
            self.host[e.tensor_id] = v
            p = self.params_by_tid[e.tensor_id]
            if not p.is_meta:
                p.data = v

    # ================================================================== state / profile
    def export_state(self) -> TensorManagerState:
        r = self.strategy_result
        if self.loader is None:
            raise RuntimeError("no inference plan yet")
        load = {}
        if r is not None:
            load = {k: list(v) for k, v in r.strategy_map.items() if v}
        elif self.state is not None:
            load = self.state.load_strategy
        bd = r.block_data if r is not None else None
        if isinstance(self.loader, BlockLoader):
            alloc: dict[int, list[str]] = {}
            for l in self.loader.order:
                if l in self.loader.plan.transfer_slot:
                    alloc.setdefault(self.loader.plan.transfer_slot[l], []).append(l)
            l2b = dict(self.loader.plan.transfer_slot)
            bsz = {b: int(n) for b, n in self.loader.plan.slot_bytes.items()}
            lsz = {l: int(b.nbytes) for l, b in self.loader.plan.host_blocks.items()}
            t2c = dict(self.loader.plan.t2c)
        else:
            alloc, l2b, bsz = {}, {}, {}
            lsz = {k: sum(t.size_bytes for t in v) for k, v in load.items()}
            t2c = dict(self.loader.t2c)
        if bd is not None and not t2c:
            t2c = dict(bd.transfer_to_compute_map)
        view_ids = sorted(t for ts in load.values() for t in (x.tensor_id for x in ts))
        dt, lay = {}, {}
        for tid in view_ids:
            p = self.params_by_tid[tid]
            nm = self.id_to_name[tid]
            dt[nm] = str(p.dtype).replace("torch.", "")
            lay[nm] = {"shape": list(p.shape), "stride": list(p.stride())}
        return TensorManagerState(
            loader_type=self.loader_type,
            tensor_id_to_name_map=dict(self.id_to_name),
            allocation_ordered=alloc,
            label_to_size_map=lsz,
            block_sizes=bsz,
            load_strategy=load,
            release_strategy={},
            label_to_block_id=l2b,
            stats=list(self.layer_stats),
            transfer_to_compute_map=t2c,
            view_tensors_ids=view_ids,
            view_tensors_names=[self.id_to_name[t] for t in view_ids],
            gpu_tensors_names=sorted(self.id_to_name[t] for t in self.resident),
            shm_block_name_map=(self.shm_store.block_name_map() if self.shm_store is not None else None),
            managed_tensor_dtypes=dt,
            managed_tensor_layouts=lay,
        )

    def save_profile(self, profile_directory: str) -> None:
        import pathlib

        st = self.state or self.export_state()
        TensorManagerState.save_to_file(pathlib.Path(profile_directory) / PROFILE_FILENAME, st)

    def load_state(self, profile_directory: str) -> TensorManagerState:
        import pathlib

        return TensorManagerState.load_from_file(pathlib.Path(profile_directory) / PROFILE_FILENAME)

    def load_profile(self, profile_directory: str, model: nn.Module) -> None:
        self.restore_state(self.load_state(profile_directory), model)

    # ------------------------------------------------------------------ state adoption
    def plan_state_adoption(self, model: nn.Module, state: TensorManagerState, *,
                            host_reserve_bytes: int = 4 << 30, gpu_reserve_bytes: int = 1 << 30):
        """Read-only plan for moving ``model``'s storages to where ``state`` wants them.

        Capacity is what is free now minus the reserves (host: psutil available; GPU: free
        plus torch's cached-but-unused bytes). Raises RuntimeError when no order fits."""
        import psutil

        from flextensor_b200.core.placement import (MemoryCapacity, capture_model_state, plan_state_transition,
                                                    target_from_profile)

        if state.loader_type != self.loader_type:
            raise ValueError(f"Saved state uses loader_type='{state.loader_type}' but TensorManager is configured "
                             f"with loader_type='{self.loader_type}'. Re-profile or use a matching transfer mode.")
        for nm, v in (("host_reserve_bytes", host_reserve_bytes), ("gpu_reserve_bytes", gpu_reserve_bytes)):
            if type(v) is not int or v < 0:
                raise ValueError(f"{nm} must be a non-negative integer")
        if self.device.type != "cuda":
            raise ValueError("state adoption plans placement onto a CUDA device")
        free, _ = torch.cuda.mem_get_info(self.device)
        cached = torch.cuda.memory_reserved(self.device) - torch.cuda.memory_allocated(self.device)
        cap = MemoryCapacity(host_bytes=max(0, psutil.virtual_memory().available - host_reserve_bytes),
                             gpu_bytes=max(0, free + cached - gpu_reserve_bytes))
        pinning = "none" if not self.pinned_memory else (
            "in_place" if self.pinner.mode == "host_register" else "copy")
        current = capture_model_state(model)
        target, spec = target_from_profile(current, state, target_device=f"cuda:{self.device.index}",
                                           pinning=pinning, use_shm=self.shm_store is not None)
        return plan_state_transition(current, target, transition=spec, capacity=cap)

    def execute_state_adoption(self, model: nn.Module, plan) -> None:
        """Carry out a plan from :meth:`plan_state_adoption` (before any graph capture)."""
        from flextensor_b200.core.placement import execute_transition

        with torch.no_grad():
            execute_transition(model, plan, pin=self.pinner.pin if self.pinned_memory else None)

    def restore_adopted_state(self, model: nn.Module, state: TensorManagerState) -> None:
        """Build the saved plan's loader on a model whose placement was already adopted."""
        self.restore_state(state, model, adopted=True)

    def restore_state(self, state: TensorManagerState, model: nn.Module | None = None, *,
                      adopted: bool = False) -> None:
        """Adopt a saved plan: rebind ids by name, then build the loader directly (no profiling).

        ``adopted``: tensors the plan keeps resident are not sent through the host first."""
        if model is not None and model is not self.model:
            self.set_model(model)
        name_to_tid = self.name_to_id
        missing = [t.name for ts in state.load_strategy.values() for t in ts if t.name not in name_to_tid]
        if missing:
            raise ValueError(f"Saved state mismatch: {len(missing)} streamed tensors not in the model "
                             f"(e.g. {missing[:3]}). Re-profile the model.")
        self.layer_stats = [
            LayerStatistics(label=s.label, duration=s.duration, tensors=[
                TensorStatistics(tensor_id=name_to_tid[t.name], name=t.name, size_bytes=t.size_bytes,
                                 load_time_ms=t.load_time_ms) for t in s.tensors if t.name in name_to_tid])
            for s in state.stats]
        load = {k: [name_to_tid[t.name] for t in v] for k, v in state.load_strategy.items() if v}
        self.strategy_result = StrategyResult(strategy_map={
            k: [TensorStatistics(tensor_id=name_to_tid[t.name], name=t.name, size_bytes=t.size_bytes,
                                 load_time_ms=t.load_time_ms) for t in v] for k, v in state.load_strategy.items()})
        self._state_restored_from_profile = True
        if self.phase == TMPhase.NONE:
            streamed = {t for ts in load.values() for t in ts}
            keep = {t for t in self.owner if t not in streamed} if adopted else None
            self.initialize_warmup(keep_on_device=keep)
        self._build_runtime([s.label for s in state.stats], load, dict(state.transfer_to_compute_map),
                            dict(state.label_to_block_id))
        self.state = state
        if self.enable_diagnostics:
            from flextensor_b200.runtime.diagnostics import log_plan

            log_plan(self)

    # ================================================================== misc API
    def get_gpu_memory_usage(self) -> GPUMemoryUsage:
        blocks = self.loader.blocks_bytes if self.loader is not None else 0
        unmapped = sum(tensor_nbytes(self.params_by_tid[t].data) for t in self.resident)
        return GPUMemoryUsage(blocks_bytes=int(blocks), unmapped_tensors_bytes=int(unmapped),
                              total_bytes=int(blocks + unmapped))

    def collect_offload_timing(self):
        return self.timing.report() if self.timing is not None else None

    def reset_offload_timing(self) -> None:
        if self.timing is not None:
            self.timing.reset()

    def sync_prev_onload(self) -> None:
        if self.loader is not None:
            self.loader.sync_prev_onload()

    def join_after_forward(self) -> None:
        if self.loader is not None:
            self.loader.join_after_forward()

    def release_memory(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def shutdown(self, *, preserve_model: bool = True) -> None:
        """Tear down the loader; with ``preserve_model`` every parameter ends up on the host."""
        self._drop_getters()
        with torch.no_grad():
            if self.loader is not None:
                if preserve_model:
                    self.loader.host_views(self.params_by_tid)
                    for tid, p in self.params_by_tid.items():
                        if p.device.type != "cpu":
                            p.data = p.data.to("cpu")
                        else:
                            p.data = p.data.clone()
                self.loader.close()
                self.loader = None
            elif preserve_model and self.model is not None:
                for p in self.params_by_tid.values():
                    if p.device.type != "cpu":
                        p.data = p.data.to("cpu")
            if preserve_model and self.model is not None:
                for _, b in self.model.named_buffers():
                    if b.device.type != "cpu":
                        b.data = b.data.to("cpu")
        self.pinner.release_all()
        if self.shm_store is not None:
            self.shm_store.close(unlink=not self.load_from_shm)
        self.host.clear()
        self._host_ptr_to_tid.clear()
        self._held_ptr_to_tid.clear()
        self.phase = TMPhase.NONE
