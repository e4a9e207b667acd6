"""OffloadManager: per-name orchestrator and the module-level public API.

Lifecycle (reference: ``src/flextensor/offload_manager.py:441-2800``)::

    NOT_INITIALIZED --offload()--> DISCOVERY --discovery_iters--> PROFILING
                    --profiling_iters--> INFERENCE

* ``offload()`` selects units, patches each unit's ``forward`` to run inside
  ``TensorManager.trap(label)`` and installs a post-forward hook on the root
  module that counts forwards and advances the phase.
* The model object keeps its identity through every phase (parameters are
  re-pointed in place), so the returned object IS the caller's model;
  ``OffloadModelProxy`` exists for callers that want an explicit wrapper.
* Managers are per-name, thread-affine singletons (``get_offload_manager``).
* Every public transition runs under an error boundary that logs phase,
  iteration, device memory and host RSS before re-raising.
"""

from __future__ import annotations

import contextlib
import functools
import logging
from dataclasses import dataclass
import os
import threading
from collections.abc import Callable
from enum import Enum
from typing import Any

import torch
from torch import nn

from flextensor_b200.config import OffloadConfig, resolve_load_strategy
from flextensor_b200.core.state import TensorManagerState
from flextensor_b200.runtime.tensor_manager import TensorManager, TMPhase
from flextensor_b200.runtime.timing import OffloadTimingReport
from flextensor_b200.runtime.units import Unit, select_units
from flextensor_b200.types import GPUMemoryUsage

LOGGER = logging.getLogger(__name__)
DEFAULT_MANAGER_NAME = "default"


class OffloadPhase(Enum):
    NOT_INITIALIZED = "not_initialized"
    DISCOVERY = "discovery"
    PROFILING = "profiling"
    INFERENCE = "inference"


@dataclass(frozen=True)
class StrategyReplanStatus:
    """Snapshot of the strategy-replan lifecycle (reading it changes nothing).

    ``state``: ``"idle"`` before any request, ``"in_progress"`` while the warm / measure tail
    rides the caller's forwards, ``"done"`` once it finished (rebuilt or refused),
    ``"failed"`` if the rebuild raised (inference is unsafe afterwards). ``can_request``:
    whether ``request_strategy_replan()`` may be called now. ``applied``: ``None`` before and
    during a request, ``True`` after a rebuild, ``False`` after a refusal or failure.
    Mirrors ``src/flextensor/compile/replan_status.py:15``."""

    state: str = "idle"
    can_request: bool = True
    applied: bool | None = None


_ONE_SHOT = ("skip_discovery", "offload_timing", "piecewise_prefetch", "profile_mode", "transfer_mode")


def _diagnostic_snapshot(label: str, om: OffloadManager | None) -> None:
    try:
        import psutil

        rss = psutil.Process().memory_info().rss
    except Exception:  # noqa: BLE001
        rss = -1
    parts = [f"[{label}] pid={os.getpid()} host_rss={rss / 2**30:.2f}GiB"]
    if om is not None:
        parts.append(f"manager={om.name!r} phase={om.phase.value} iteration={om.iteration}")
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            try:
                free, total = torch.cuda.mem_get_info(i)
                parts.append(f"gpu{i}: alloc={torch.cuda.memory_allocated(i) / 2**30:.2f} "
                             f"reserved={torch.cuda.memory_reserved(i) / 2**30:.2f} total={total / 2**30:.1f}GiB")
            except Exception:  # noqa: BLE001
                pass
    LOGGER.error(" ".join(parts))


def _error_boundary(fn):
    @functools.wraps(fn)
    def wrapper(self, *a, **kw):
        try:
            return fn(self, *a, **kw)
        except Exception:
            _diagnostic_snapshot(fn.__name__, self)
            raise

    return wrapper


class OffloadModelProxy:
    """Transparent wrapper delegating every attribute and call to the managed model."""

    def __init__(self, model: nn.Module, manager: "OffloadManager"):
        object.__setattr__(self, "_ft_model", model)
        object.__setattr__(self, "_ft_manager", manager)

    @property
    def offload_manager(self) -> "OffloadManager":
        return object.__getattribute__(self, "_ft_manager")

    def __call__(self, *a, **kw):
        return object.__getattribute__(self, "_ft_model")(*a, **kw)

    def forward(self, *a, **kw):
        return object.__getattribute__(self, "_ft_model")(*a, **kw)

    def __getattr__(self, item):
        return getattr(object.__getattribute__(self, "_ft_model"), item)

    def __setattr__(self, key, value):
        setattr(object.__getattribute__(self, "_ft_model"), key, value)


class OffloadManager:
    def __init__(self, name: str = DEFAULT_MANAGER_NAME):
        self.name = name
        self.config = OffloadConfig()
        self._tm: TensorManager | None = None
        self.phase = OffloadPhase.NOT_INITIALIZED
        self.iteration = 0
        self.model: nn.Module | None = None
        self.units: list[Unit] = []
        self._orig_forwards: dict[str, Any] = {}
        self._hook = None
        self._pending_state: TensorManagerState | None = None
        self._compile_fn = None
        self._compiled: dict[str, Callable] = {}
        from flextensor_b200.runtime.compiled import CompiledOffload

        self._compiled_offload = CompiledOffload(self)
        self._skip_discovery_honored: bool | None = None
        self._manual_blocks = False
        self._replan_status = StrategyReplanStatus()
        self._tail: dict | None = None  # armed replan tail: {"warm": n, "measure": n, "seen": k}
        self._manual_update_state = False
        self._owner_thread = threading.get_ident()
        self._carrier = None

    # ------------------------------------------------------------------ config
    @property
    def compiled_offload_manager_id(self) -> int:
        from flextensor_b200.runtime import custom_ops

        return custom_ops.register_manager(self)

    def set_config(self, config: OffloadConfig) -> None:
        if self._tm is not None:
            for f in _ONE_SHOT:
                if getattr(config, f) != getattr(self.config, f):
                    if f == "skip_discovery":
                        raise RuntimeError("skip_discovery cannot change after offload(); call release() first")
                    LOGGER.warning("%s changed after the TensorManager was built; release() and re-offload() "
                                   "to apply it", f)
        self.config = config

    def init(self, config: OffloadConfig | None = None) -> None:
        if config is not None:
            self.set_config(config)
        if self._tm is None:
            self._tm = self._make_tm()

    def _make_tm(self) -> TensorManager:
        c = self.config
        if c.enable_instrumentation:
            from flextensor_b200.instrumentation import get_registry

            get_registry().enabled = True
        shm_store = None
        if c.shm_enabled:
            from flextensor_b200.shm.store import ShmWeightStore

            shm_store = ShmWeightStore(c.shm_namespace, pinned=c.pinned_memory)
        dev = torch.device("cuda", c.gpu_device) if torch.cuda.is_available() else torch.device("cpu")
        return TensorManager(
            dev, resolve_load_strategy(c), loader_type=c.transfer_mode, blocks=c.num_blocks,
            pinned_memory=c.pinned_memory, pinned_memory_mode=c.pinned_memory_mode, profile_mode=c.profile_mode,
            max_gpu_mem_fraction=c.max_gpu_mem_fraction, hold_device_weights=c.hold_device_weights,
            offload_timing=c.offload_timing,
            enable_diagnostics=c.enable_diagnostics, shm_store=shm_store, piecewise_prefetch=c.piecewise_prefetch)

    def get_tensor_manager(self) -> TensorManager | None:
        return self._tm

    @property
    def skip_discovery_honored(self) -> bool | None:
        return self._skip_discovery_honored

    @property
    def iters_before_inference(self) -> int:
        if self.phase == OffloadPhase.INFERENCE:
            return 0
        prof = max(1, self.config.profiling_iters)
        warm = self._compiled_offload.extra_forwards_before_inference()
        if self.phase == OffloadPhase.PROFILING:
            return max(0, prof - self._profile_iter()) + warm
        disc = 0 if self._skip_discovery_honored else self.config.discovery_iters
        return disc + prof + warm

    def _profile_iter(self) -> int:
        return self.iteration - (0 if self._skip_discovery_honored else self.config.discovery_iters)

    @property
    def eager_profiling_iters(self) -> int:
        return max(1, self.config.profiling_iters)

    # ------------------------------------------------------------------ patching
    def _check_thread(self) -> None:
        if threading.get_ident() != self._owner_thread:
            raise RuntimeError(f"OffloadManager {self.name!r} is thread-affine; use one manager per thread")

    def _patch(self, unit: Unit) -> None:
        mod = unit.module
        label = unit.label
        orig = mod.forward
        self._orig_forwards[label] = orig
        tm_ref = self

        @torch.compiler.disable
        def patched_forward(*args, **kwargs):
            tm = tm_ref._tm
            fn = tm_ref._compiled.get(label, orig)
            if tm is None:
                return fn(*args, **kwargs)
            with tm.trap(label):
                return fn(*args, **kwargs)

        def op_forward(*args, **kwargs):
            # external_compile in INFERENCE: trap boundaries are opaque custom ops, so a
            # caller's torch.compile of the unit keeps the prefetch schedule in its graph
            tm = tm_ref._tm
            if tm is None or tm_ref.phase != OffloadPhase.INFERENCE:
                return patched_forward(*args, **kwargs)
            mid = tm_ref.compiled_offload_manager_id
            carrier = tm_ref._carrier
            torch.ops.flextensor_b200.pre_compute(carrier, label, mid)
            out = orig(*args, **kwargs)
            torch.ops.flextensor_b200.post_compute(carrier, label, mid)
            return out

        mod.forward = op_forward if self.config.external_compile else patched_forward

    def _unpatch(self) -> None:
        for u in self.units:
            if "forward" in u.module.__dict__:
                del u.module.__dict__["forward"]
        self._orig_forwards.clear()
        self._compiled.clear()
        if self._hook is not None:
            self._hook.remove()
            self._hook = None

    def _post_forward(self, module, args, output):
        if self._tm is not None:
            self._tm.join_after_forward()
        if not self._manual_update_state:
            self.update_state()
        self._compiled_offload.on_forward_end()
        if self._tail is not None and self.phase == OffloadPhase.INFERENCE:
            self._advance_tail()
        return None

    # ------------------------------------------------------------------ replan tail
    def _advance_tail(self) -> None:
        """Warm -> measure -> rebuild, one step per completed forward (see request_strategy_replan)."""
        t = self._tail
        t["seen"] += 1
        tm = self._tm
        if t["seen"] == t["warm"]:  # warm-up done: measure from a clean slate
            if tm.timing is None:
                from flextensor_b200.runtime.timing import OffloadTimingCollector

                tm.timing = OffloadTimingCollector(tm.device, "eager")
                t["temporary_timing"] = True
            tm.loader.timing = tm.timing
            tm.reset_offload_timing()
        if t["seen"] < t["warm"] + t["measure"]:
            return
        self._tail = None
        try:
            applied = self._replan_from_timing()
            self._replan_status = StrategyReplanStatus("done", True, applied)
        except Exception:
            self._replan_status = StrategyReplanStatus("failed", False, False)
            raise
        finally:
            if t.get("temporary_timing"):
                tm.timing = None
                if tm.loader is not None:
                    tm.loader.timing = None

    # ------------------------------------------------------------------ offload
    @_error_boundary
    def offload(self, model: nn.Module, config: OffloadConfig | None = None,
                compile_fn: Callable[[nn.Module], nn.Module] | None = None) -> nn.Module:
        self._check_thread()
        if config is not None:
            self.set_config(config)
        c = self.config
        if getattr(model, "_orig_mod", None) is not None or type(model).__name__ == "OptimizedModule":
            raise ValueError("offload() needs the eager model; apply torch.compile per unit via compile_fn")
        if self.model is not None and self.model is not model:
            raise RuntimeError(f"manager {self.name!r} already manages another model; release() it first")
        self._compile_fn = compile_fn
        self._compiled_offload.resolve(c, compile_fn)
        if not c.enabled:
            dev = torch.device("cuda", c.gpu_device) if torch.cuda.is_available() else torch.device("cpu")
            self.model = model.to(dev)
            self.phase = OffloadPhase.INFERENCE
            return model
        self.init()
        tm = self._tm
        self.model = model
        tm.set_model(model)
        self.units = select_units(model, c.include_patterns, c.exclude_patterns)
        if not self.units and not self._manual_blocks:
            LOGGER.warning("no module matched include_patterns=%s; nothing is offloaded", c.include_patterns)
        tm.set_units(self.units)
        for u in self.units:
            self._patch(u)
        self._hook = model.register_forward_hook(self._post_forward, prepend=True)
        if self._pending_state is not None:
            st, self._pending_state = self._pending_state, None
            adopt, self._pending_adopt = getattr(self, "_pending_adopt", False), False
            if adopt:
                # model already loaded (e.g. by a serving engine): move only what the plan
                # moves, in a capacity-safe order, then build the loader without profiling
                plan = tm.plan_state_adoption(model, st)
                tm.execute_state_adoption(model, plan)
                tm.restore_adopted_state(model, st)
            else:
                tm.initialize_warmup()
                tm.restore_state(st, model)
            self._enter_inference()
            return model
        tm.initialize_warmup()
        self.phase = OffloadPhase.DISCOVERY
        self.iteration = 0
        if c.skip_discovery and self.units:
            self._skip_discovery_honored = True
            tm.static_discovery()
            self._to_profiling()
        else:
            if c.skip_discovery:
                LOGGER.warning("skip_discovery=True but no module was patched; running discovery")
            self._skip_discovery_honored = False if c.skip_discovery else None
            if c.discovery_iters == 0:
                self._to_profiling()
        return model

    @_error_boundary
    def offload_from_state(self, model: nn.Module, state: TensorManagerState, config: OffloadConfig | None = None,
                           *, allow_strategy_replan: bool = True, adopt: bool = False) -> nn.Module:
        """Apply a saved plan without discovery or profiling.

        ``adopt=True``: ``model`` is already placed (typically all on the GPU); its storages
        are migrated to the plan's placement in a capacity-checked order instead of first
        moving every offloadable tensor to the host."""
        if config is not None:
            self.set_config(config)
        if state.loader_type != self.config.transfer_mode:
            raise ValueError(f"state loader_type {state.loader_type!r} != config transfer_mode "
                             f"{self.config.transfer_mode!r}")
        self._pending_state = state
        self._pending_adopt = adopt
        return self.offload(model)

    @_error_boundary
    def offload_static(self, model: nn.Module, config: OffloadConfig | None = None, *,
                       durations_ms: dict[str, float] | None = None) -> nn.Module:
        """Plan and build the runtime with no discovery or profiling forward passes.

        For models that cannot run a plain forward outside their engine (serving engines that
        need attention metadata per call). Traps are the selected units and each trap reads
        exactly its unit's parameters. Trap durations come from ``durations_ms`` or, by
        default, from a conservative estimate: every unit computes for as long as its own
        weights take to copy host->device (measured), so a plan that hides each transfer
        behind one trap's compute is feasible by construction. A real profile can replace
        the estimate later (``request_strategy_replan`` / a saved profile)."""
        c = (config or self.config).model_copy(update={"skip_discovery": True})
        model = self.offload(model, c)
        tm = self._tm
        if self.phase != OffloadPhase.PROFILING:
            return model  # disabled, or nothing matched
        est = tm.estimate_unit_durations() if durations_ms is None else dict(durations_ms)
        for label in tm.labels:
            if label in est:
                tm.collector.record_duration(label, float(est[label]))
        tm.initialize_inference()
        self._enter_inference()
        return model

    def offload_block(self, name: str):
        """Manual trap: ``with om.offload_block("blk"): ...`` (discovered by tensor reads)."""
        if self._skip_discovery_honored:
            raise RuntimeError("offload_block() cannot be used when skip_discovery is honored")
        self._manual_blocks = True
        if self._tm is None:
            self.init()
        return self._tm.trap(name)

    # ------------------------------------------------------------------ phase machine
    def _to_profiling(self) -> None:
        self._tm.initialize_profile()
        self.phase = OffloadPhase.PROFILING
        self._compiled_offload.on_enter_profiling()

    def _enter_inference(self) -> None:
        self.phase = OffloadPhase.INFERENCE
        if self.config.external_compile:
            from flextensor_b200.runtime import custom_ops

            self._carrier = custom_ops.carrier_for(self._tm.device)
        self._compiled_offload.on_enter_inference()
        self._dump_instrumentation()

    def _dump_instrumentation(self) -> None:
        c = self.config
        if not c.enable_instrumentation or not c.instrumentation_output_dir or self._tm is None:
            return
        from flextensor_b200.instrumentation import dump_to_directory

        try:
            stats = self._tm.get_memory_transfer_stats()
            dump_to_directory(c.instrumentation_output_dir, extra={
                "memory_transfer_stats": {str(k): v for k, v in (stats or {}).items()}})
        except Exception:  # noqa: BLE001 - a failed dump never blocks inference
            LOGGER.warning("instrumentation dump failed; continuing", exc_info=True)

    @_error_boundary
    def update_state(self, *, replay_generation: int = -1) -> None:
        if self.phase in (OffloadPhase.NOT_INITIALIZED, OffloadPhase.INFERENCE):
            return
        tm = self._tm
        if tm is not None and tm.is_profiling_suspended() and self.phase == OffloadPhase.PROFILING:
            return
        self.iteration += 1
        if self.phase == OffloadPhase.DISCOVERY and self.iteration >= self.config.discovery_iters:
            self._to_profiling()
            return
        if self.phase == OffloadPhase.PROFILING and self._profile_iter() >= max(1, self.config.profiling_iters):
            tm.initialize_inference()
            self._enter_inference()

    # ------------------------------------------------------------------ profiles
    def _profile_dir(self, d: str | None) -> str:
        d = d or self.config.profile_storage_dir
        if not d:
            raise ValueError("no profile directory given and config.profile_storage_dir is unset")
        return d

    def save_profile(self, profile_directory: str | None = None) -> None:
        if self.config.profile_read_only:
            LOGGER.warning("profile_read_only=True; not saving")
            return
        if self._tm is None or self.phase != OffloadPhase.INFERENCE:
            raise RuntimeError("save_profile() needs the INFERENCE phase")
        self._tm.save_profile(self._profile_dir(profile_directory))

    def load_profile(self, profile_directory: str | None = None, model: nn.Module | None = None) -> None:
        st = TensorManagerState.load_from_file(os.path.join(self._profile_dir(profile_directory), "profile.json"))
        if self.phase == OffloadPhase.NOT_INITIALIZED or model is None and self.model is None:
            self._pending_state = st
            return
        self._tm.restore_state(st, model or self.model)
        self._enter_inference()

    def export_state(self) -> TensorManagerState:
        return self._tm.export_state()

    # ------------------------------------------------------------------ runtime queries
    def get_gpu_memory_usage(self) -> GPUMemoryUsage:
        if self._tm is None:
            return GPUMemoryUsage(0, 0, 0)
        return self._tm.get_gpu_memory_usage()

    def collect_offload_timing(self) -> OffloadTimingReport | None:
        return self._tm.collect_offload_timing() if self._tm is not None else None

    def reset_offload_timing(self) -> None:
        if self._tm is not None:
            self._tm.reset_offload_timing()

    def update_offload_timing(self, *, replay_generation: int = -1) -> bool:
        return self.collect_offload_timing() is not None

    def sync_prev_onload(self) -> None:
        if self._tm is not None:
            self._tm.sync_prev_onload()

    def join_after_forward(self) -> None:
        if self._tm is not None:
            self._tm.join_after_forward()

    def offload_units(self) -> tuple[tuple[str, nn.Module], ...]:
        return tuple((u.label, u.module) for u in self.units)

    def resident_units(self) -> tuple[tuple[str, nn.Module], ...]:
        if self._tm is None or self._tm.loader is None:
            return ()
        streamed_owners = set()
        plan = getattr(self._tm.loader, "plan", None)
        if plan is not None:
            streamed_owners = set(plan.t2c.values())
        else:
            streamed_owners = set(self._tm.loader.c2t)
        return tuple((u.label, u.module) for u in self.units if u.label not in streamed_owners)

    def get_layer_label_by_idx(self) -> list[str]:
        return [u.label for u in self.units]

    @property
    def strategy_replan_status(self) -> StrategyReplanStatus:
        return self._replan_status

    @_error_boundary
    def request_strategy_replan(self, *, manual_update_state: bool = False, warmup_forwards: int = 1,
                                measure_forwards: int = 3) -> int:
        """Re-plan from measured inference compute times.

        Arms a tail that rides the caller's next forwards: ``warmup_forwards`` forwards are
        discarded, the next ``measure_forwards`` are timed per trap (offload timing is enabled
        for them if it is off), and after the last one the strategy is recomputed from those
        compute budgets and the loader rebuilt. Returns the number of forwards until the
        rebuild (``StrategyReplanStatus`` tracks progress)."""
        if self.phase != OffloadPhase.INFERENCE or self._tm is None or self._tm.loader is None:
            raise RuntimeError("request_strategy_replan() needs a manager in the INFERENCE phase")
        if not self._replan_status.can_request:
            raise RuntimeError(f"a replan cannot be requested now (state={self._replan_status.state!r})")
        if warmup_forwards < 1 or measure_forwards < 1:
            raise ValueError("warmup_forwards and measure_forwards must be >= 1")
        self._manual_update_state = manual_update_state
        self._tail = {"warm": warmup_forwards, "measure": measure_forwards, "seen": 0}
        self._replan_status = StrategyReplanStatus("in_progress", False, None)
        return warmup_forwards + measure_forwards

    def _replan_from_timing(self) -> bool:
        tm = self._tm
        rep = tm.collect_offload_timing()
        if rep is None or not rep.per_trap:
            LOGGER.warning("strategy replan refused: no per-trap timing was collected")
            return False
        budgets = rep.compute_budgets_by_profile_label()
        from flextensor_b200.core.stats import LayerStatistics

        tm.layer_stats = [LayerStatistics(label=l.label, tensors=l.tensors, duration=budgets.get(l.label, l.duration))
                          for l in tm.layer_stats]
        tm.loader.host_views(tm.params_by_tid)
        for tids in (tm.unit_tids.values()):
            for t in tids:
                if t not in tm.resident:
                    tm.host[t] = tm.params_by_tid[t].data
        tm.loader.close()
        result = tm.strategy.compute(tm.layer_stats, tm.memory_stats, tm._gpu_budget())
        tm.strategy_result = result
        tm._build_from_result(result)
        return True

    def clear_profiling_durations(self) -> None:
        if self._tm is not None:
            self._tm.clear_profiling_durations()

    def suspend_profiling(self) -> None:
        if self._tm is not None:
            self._tm.suspend_profiling()

    def resume_profiling(self) -> None:
        if self._tm is not None:
            self._tm.resume_profiling()

    def pause_profiling(self):
        if self._tm is None:
            return contextlib.nullcontext()
        return self._tm.pause_profiling()

    # ------------------------------------------------------------------ release
    def release(self, *, preserve_model: bool = True) -> None:
        tm, self._tm = self._tm, None
        try:
            if tm is not None:
                tm.release_memory()
                tm.shutdown(preserve_model=preserve_model)
        finally:
            self._compiled_offload.teardown()
            self._unpatch()
            self.phase = OffloadPhase.NOT_INITIALIZED
            self.iteration = 0
            self.model = None
            self.units = []
            self._pending_state = None
            self._skip_discovery_honored = None
            self._manual_blocks = False


class _UnitCore(nn.Module):
    """Holds a unit's original bound forward so a per-unit compiler never re-enters the trap."""

    def __init__(self, fwd):
        super().__init__()
        self._fwd = fwd

    def forward(self, *a, **kw):
        return self._fwd(*a, **kw)


# ============================================================================ registry + module API

_registry: dict[tuple[int, str], OffloadManager] = {}
_reg_lock = threading.Lock()


def get_offload_manager(name: str = DEFAULT_MANAGER_NAME) -> OffloadManager:
    key = (threading.get_ident(), name)
    with _reg_lock:
        om = _registry.get(key)
        if om is None:
            om = OffloadManager(name)
            _registry[key] = om
        return om


def init(config: OffloadConfig | None = None, name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).init(config)


def offload(model: nn.Module, config: OffloadConfig | None = None, name: str = DEFAULT_MANAGER_NAME,
            compile_fn: Callable[[nn.Module], nn.Module] | None = None) -> nn.Module:
    return get_offload_manager(name).offload(model, config, compile_fn=compile_fn)


def set_config(config: OffloadConfig, name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).set_config(config)


def save_profile(profile_directory: str | None = None, name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).save_profile(profile_directory)


def load_profile(profile_directory: str | None = None, model: nn.Module | None = None,
                 name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).load_profile(profile_directory, model)


def offload_from_state(model: nn.Module, state: TensorManagerState, config: OffloadConfig | None = None,
                       name: str = DEFAULT_MANAGER_NAME, *, allow_strategy_replan: bool = True) -> nn.Module:
    return get_offload_manager(name).offload_from_state(model, state, config=config,
                                                        allow_strategy_replan=allow_strategy_replan)


def offload_from_profile(model: nn.Module, profile_directory: str, config: OffloadConfig | None = None,
                         name: str = DEFAULT_MANAGER_NAME,
                         compile_fn: Callable[[nn.Module], nn.Module] | None = None) -> nn.Module:
    init(config=config, name=name)
    load_profile(profile_directory, model=None, name=name)
    return offload(model, config=config, name=name, compile_fn=compile_fn)


def offload_block(block_name: str, name: str = DEFAULT_MANAGER_NAME) -> Any:
    return get_offload_manager(name).offload_block(block_name)


def release(name: str = DEFAULT_MANAGER_NAME, *, preserve_model: bool = True) -> None:
    get_offload_manager(name).release(preserve_model=preserve_model)


def get_gpu_memory_usage(name: str = DEFAULT_MANAGER_NAME) -> GPUMemoryUsage:
    return get_offload_manager(name).get_gpu_memory_usage()


def reset_offload_timing(name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).reset_offload_timing()


def collect_offload_timing(name: str = DEFAULT_MANAGER_NAME) -> OffloadTimingReport | None:
    return get_offload_manager(name).collect_offload_timing()


def update_offload_timing(name: str = DEFAULT_MANAGER_NAME, *, replay_generation: int = -1) -> bool:
    return get_offload_manager(name).update_offload_timing(replay_generation=replay_generation)


def offload_units(name: str = DEFAULT_MANAGER_NAME) -> tuple[tuple[str, nn.Module], ...]:
    return get_offload_manager(name).offload_units()


def resident_units(name: str = DEFAULT_MANAGER_NAME) -> tuple[tuple[str, nn.Module], ...]:
    return get_offload_manager(name).resident_units()


def request_strategy_replan(name: str = DEFAULT_MANAGER_NAME, *, manual_update_state: bool = False) -> int:
    return get_offload_manager(name).request_strategy_replan(manual_update_state=manual_update_state)


def update_state(name: str = DEFAULT_MANAGER_NAME, *, replay_generation: int = -1) -> None:
    get_offload_manager(name).update_state(replay_generation=replay_generation)


def clear_profiling_durations(name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).clear_profiling_durations()


def suspend_profiling(name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).suspend_profiling()


def resume_profiling(name: str = DEFAULT_MANAGER_NAME) -> None:
    get_offload_manager(name).resume_profiling()


def pause_profiling(name: str = DEFAULT_MANAGER_NAME) -> Any:
    return get_offload_manager(name).pause_profiling()
