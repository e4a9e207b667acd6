"""Compiled offload: per-unit ``torch.compile`` (or any ``compile_fn``) with the offload schedule
kept intact, and the plan built from COMPILED compute times.

Parity with ``src/flextensor/compile/lifecycle.py:76-656`` and
``src/flextensor/compiled_offload.py:196-298`` (behaviour, not structure). One
:class:`CompiledOffload` per manager decides the path from ``compile_fn`` and the config:

* ``compile_fn`` with ``profile_mode="view"`` -> **compiled view-profile**: every unit is compiled
  when PROFILING starts, the first ``PROFILE_COMPILE_WARMUP_FORWARDS`` forwards run unmeasured
  (profiling suspended while each unit's lazy compile settles), then ``profiling_iters`` forwards
  are measured under the compiled code, so the strategy is built from compiled timings and
  needs no replan;
* ``compile_fn`` with another profile mode -> **eager profile, compiled inference, replan tail**:
  units are compiled on entering INFERENCE and a tail rides the caller's next forwards --
  ``COMPILED_WARMUP_FORWARDS`` unmeasured (compilation), ``profiling_iters`` timed -- after which
  the strategy is rebuilt from the compiled compute times (``strategy_replan_status`` reports it);
* ``external_compile`` without ``compile_fn`` -> unit boundaries are opaque custom ops
  (``runtime/custom_ops.py``) so the caller may compile the units itself; it then calls
  ``request_strategy_replan()``.

Compiled offload needs a block transfer mode (the custom ops drive the block loader); a
``transfer_mode="strategy"`` config is rejected before any live state is torn down.

Dynamo keeps one cache entry per guard set of a code object, and all units of one class share
their ``forward`` code: N identical blocks compiled separately need N entries, far more than
dynamo's default per-code limit of 8, after which the remaining blocks silently fall back to
eager. :func:`bump_dynamo_limits` raises the limits to cover every unit (restored on teardown).
"""

from __future__ import annotations

import logging
from typing import Callable

from torch import nn

from flextensor_b200.config import BLOCK_TRANSFER_MODES

LOGGER = logging.getLogger(__name__)

COMPILED_WARMUP_FORWARDS = 3
PROFILE_COMPILE_WARMUP_FORWARDS = 3
_DYNAMO_LIMIT_KEYS = ("cache_size_limit", "recompile_limit", "accumulated_cache_size_limit",
                      "accumulated_recompile_limit")


def bump_dynamo_limits(n_units: int, per_unit: int = 4) -> dict[str, int]:
    """Raise dynamo's per-code-object and accumulated cache limits so ``n_units`` units that
    share one forward code object each keep their compiled entries (``per_unit`` entries of
    headroom each for shape / dtype specialisations). Returns the previous values."""
    try:
        import torch._dynamo.config as dcfg
    except Exception:  # noqa: BLE001 - no dynamo: nothing to raise
        return {}
    need = max(8, n_units * per_unit)
    old: dict[str, int] = {}
    for key in _DYNAMO_LIMIT_KEYS:
        if hasattr(dcfg, key):
            cur = getattr(dcfg, key)
            if isinstance(cur, int) and cur < need * (8 if key.startswith("accumulated") else 1):
                old[key] = cur
                setattr(dcfg, key, need * (8 if key.startswith("accumulated") else 1))
    if old:
        LOGGER.info("compiled offload: dynamo limits raised for %d units: %s", n_units,
                    {k: getattr(dcfg, k) for k in old})
    return old


def restore_dynamo_limits(old: dict[str, int]) -> None:
    if not old:
        return
    import torch._dynamo.config as dcfg

    for k, v in old.items():
        setattr(dcfg, k, v)


class CompiledOffload:
    """Compile lifecycle of one :class:`~flextensor_b200.runtime.manager.OffloadManager`.

    ``mode``: ``off`` | ``view_profile`` | ``inference_tail`` | ``external``."""

    def __init__(self, manager):
        self._om = manager
        self.mode = "off"
        self.compile_fn: Callable[[nn.Module], nn.Module] | None = None
        self.profile_warm_remaining = 0
        self._suspended = False
        self._dynamo_old: dict[str, int] = {}

    # ---------------------------------------------------------------- activation
    def resolve(self, config, compile_fn) -> str:
        """Pick the path; validates before tearing down what a previous offload left."""
        if compile_fn is not None or config.external_compile:
            if config.transfer_mode not in BLOCK_TRANSFER_MODES:
                raise ValueError(
                    "compiled offload requires a block transfer_mode (allocation_block_transfer or "
                    f"raw_block_transfer); got transfer_mode={config.transfer_mode!r}")
        self.teardown()
        self.compile_fn = compile_fn
        if compile_fn is not None:
            self.mode = "view_profile" if config.profile_mode == "view" else "inference_tail"
        elif config.external_compile:
            self.mode = "external"
        else:
            self.mode = "off"
        return self.mode

    @property
    def active(self) -> bool:
        return self.mode != "off"

    def extra_forwards_before_inference(self) -> int:
        """Unmeasured compile-warmup forwards still owed before INFERENCE (view profile)."""
        if self.mode != "view_profile":
            return 0
        if self._om.phase.name in ("DISCOVERY", "NOT_INITIALIZED"):
            return PROFILE_COMPILE_WARMUP_FORWARDS
        return self.profile_warm_remaining

    # ---------------------------------------------------------------- phase hooks
    def _compile_units(self) -> None:
        om = self._om
        if self.compile_fn is None or om._compiled:
            return
        from flextensor_b200.runtime.manager import _UnitCore

        self._dynamo_old = bump_dynamo_limits(len(om.units))
        for u in om.units:
            core = _UnitCore(om._orig_forwards[u.label])
            om._compiled[u.label] = self.compile_fn(core)

    def on_enter_profiling(self) -> None:
        if self.mode != "view_profile":
            return
        self._compile_units()
        tm = self._om._tm
        if tm is not None and not self._suspended:
            tm.suspend_profiling()
            self._suspended = True
        self.profile_warm_remaining = PROFILE_COMPILE_WARMUP_FORWARDS
        LOGGER.info("compiled view-profile: %d compile-warmup forwards, then %d measured forwards",
                    PROFILE_COMPILE_WARMUP_FORWARDS, self._om.config.profiling_iters)

    def on_forward_end(self) -> None:
        """After the manager's state update: count down the unmeasured compile warm-up."""
        om = self._om
        if self.mode != "view_profile" or self.profile_warm_remaining <= 0:
            return
        if om.phase.name != "PROFILING":
            return
        self.profile_warm_remaining -= 1
        if self.profile_warm_remaining == 0 and self._suspended:
            om._tm.clear_profiling_durations()
            om._tm.resume_profiling()
            self._suspended = False

    def on_enter_inference(self) -> None:
        if self.mode == "view_profile":
            self._compile_units()  # already compiled when profiling started (restored plans: now)
        elif self.mode == "inference_tail":
            self._compile_units()
            om = self._om
            if om._tm is not None and om._tm.loader is not None and om._replan_status.can_request:
                om.request_strategy_replan(warmup_forwards=COMPILED_WARMUP_FORWARDS,
                                           measure_forwards=max(1, om.config.profiling_iters))

    def teardown(self) -> None:
        om = self._om
        if self._suspended and om._tm is not None:
            try:
                om._tm.resume_profiling()
            except RuntimeError:
                pass
        self._suspended = False
        self.profile_warm_remaining = 0
        restore_dynamo_limits(self._dynamo_old)
        self._dynamo_old = {}
        self.compile_fn = None
        self.mode = "off"
