"""FlexTensor worker for vLLM (V1 engine).

``load_model``: read the OffloadConfig (``FT_*`` environment / ``FT_CONFIG_FILE``); when
enabled, install :class:`FlexTensorBootstrapOffloader` so decoder layers are built and loaded
into host memory, let vLLM load the model, then hand it to the FlexTensor runtime:

* with a saved profile (``profile_storage_dir`` holding ``profile.json``) the plan is applied
  directly;
* otherwise the plan is computed without forward passes (``OffloadManager.offload_static``:
  per-layer durations estimated from the measured host->device time of each layer's bytes)
  under ``max_gpu_mem_fraction`` when set.

Units are patched in place, so vLLM keeps calling its own model object. vLLM then sizes the
KV cache with the ring slots already allocated. Selection of compile/graph behaviour follows
vLLM's: under vLLM's compile mode the trap boundaries are the opaque custom ops
``flextensor_b200::pre_compute`` / ``post_compute`` (``external_compile``); CUDA-graph
replays use device-event timing (``offload_timing="cuda_graph"`` when timing is on).
With ``FT_SHM_ENABLED=1`` (plus a read-only saved profile and ``FT_SHM_NAMESPACE``), vLLM's local
data-parallel replicas share one host copy of the weights (``contrib/vllm/shared.py``).
Parity: ``src/flextensor/contrib/vllm/v2/worker.py:235-616``. Rejected like the reference:
expert parallelism / EPLB, and the shared-memory path outside its validated topology.
"""

from __future__ import annotations

import logging
import os

import torch

from flextensor_b200.config import _register_env_var, load_config
from flextensor_b200.contrib.vllm.offloader import FlexTensorBootstrapOffloader
from flextensor_b200.contrib.vllm.patterns import resolve_vllm_patterns

LOGGER = logging.getLogger("vllm.flextensor_b200.worker")
MANAGER_NAME = "vllm"
_register_env_var("FT_VLLM_USE_V2_WORKER")
_register_env_var("FT_VLLM_REPLAN_AFTER")
_register_env_var("FT_VLLM_FUSED_TP")

from vllm.v1.worker.gpu_worker import Worker  # noqa: E402

from flextensor_b200.contrib.vllm import loader as _loader  # noqa: E402,F401 - registers load_format "flextensor"
from flextensor_b200.contrib.vllm import shared as _shared  # noqa: E402,F401 - registers "flextensor_shm"

_selector = os.environ.get("FT_VLLM_USE_V2_WORKER", "1")
if _selector not in ("0", "1"):
    raise ValueError(f"FT_VLLM_USE_V2_WORKER must be '0' (legacy) or '1' (v2), got {_selector!r}")
if _selector == "0":
    LOGGER.warning("FT_VLLM_USE_V2_WORKER=0: there is no separate legacy worker in flextensor_b200; the "
                   "state-takeover worker serves both settings")


class FlexTensorWorkerError(RuntimeError):
    pass


def ensure_drafter_on_device(model_runner, device) -> bool:
    """Speculative decoding: vLLM keeps the drafter at ``model_runner.drafter.model``. Its layers
    pass through the bootstrap offloader too (host-staged) but FlexTensor takes over only the main
    model, so the drafter must go back to the device, and BEFORE the takeover: a drafter module
    that shares a tensor with the main model (e.g. ``embed_tokens``) would otherwise move after
    FlexTensor recorded that tensor. Returns whether a drafter was moved."""
    drafter = getattr(model_runner, "drafter", None)
    if drafter is None:
        return False
    model = getattr(drafter, "model", None)
    if model is None or not callable(getattr(model, "to", None)):
        LOGGER.warning("speculative drafter without a movable .model (%s): it stays where vLLM put it",
                       type(drafter).__name__)
        return False
    model.to(device)
    return True


def _validate(vllm_config, cfg) -> None:
    par = vllm_config.parallel_config
    if getattr(par, "enable_expert_parallel", False) or getattr(par, "enable_eplb", False):
        raise FlexTensorWorkerError("expert parallelism / EPLB is not supported with FlexTensor offloading")
    if cfg.shm_enabled and (par.tensor_parallel_size > 1 or par.pipeline_parallel_size > 1):
        raise FlexTensorWorkerError("the shared-memory weight store needs tensor_parallel_size == "
                                    "pipeline_parallel_size == 1")
    if cfg.transfer_mode == "strategy":
        raise FlexTensorWorkerError("the vLLM worker needs a block transfer_mode")


class FlexTensorOffloadWorker(Worker):
    """Production profile refresh: the first plan comes from estimated layer times (or a saved
    profile); after ``FT_VLLM_REPLAN_AFTER`` model steps (default 64, 0 = never) the worker asks
    the manager for a strategy replan, whose warm / measure tail times the next real batches
    per trap and rebuilds the plan from those compute times; the refreshed plan is saved to
    ``profile_storage_dir`` when one is configured and writable."""

    _ft_steps = 0
    _ft_replan_after = None

    def execute_model(self, scheduler_output):
        out = super().execute_model(scheduler_output)
        om = getattr(self, "_ft_manager", None)
        if om is None:
            return out
        if self._ft_replan_after is None:
            self._ft_replan_after = int(os.environ.get("FT_VLLM_REPLAN_AFTER", "64"))
        self._ft_steps += 1
        st = om.strategy_replan_status
        if self._ft_replan_after and self._ft_steps == self._ft_replan_after and st.can_request:
            try:
                om.request_strategy_replan()
                LOGGER.info("FlexTensor: profile refresh armed after %d steps", self._ft_steps)
            except Exception:  # noqa: BLE001 - a refresh is an optimisation, never fatal
                LOGGER.warning("FlexTensor: profile refresh could not start", exc_info=True)
        elif st.state == "done" and st.applied and not getattr(self, "_ft_saved", False):
            self._ft_saved = True
            cfg = om.config
            if cfg.profile_storage_dir and not cfg.profile_read_only:
                try:
                    om.save_profile(cfg.profile_storage_dir)
                except Exception:  # noqa: BLE001
                    LOGGER.warning("FlexTensor: saving the refreshed profile failed", exc_info=True)
        return out

    def _maybe_fuse_tp(self) -> None:
        """``FT_VLLM_FUSED_TP=1``: fused GEMM + all-reduce for the row-parallel layers (eager mode)."""
        if os.environ.get("FT_VLLM_FUSED_TP", "0") != "1":
            return
        par = self.vllm_config.parallel_config
        if par.tensor_parallel_size <= 1:
            return
        from vllm.config import CUDAGraphMode

        comp = self.vllm_config.compilation_config
        if comp.cudagraph_mode is not None and comp.cudagraph_mode != CUDAGraphMode.NONE:
            LOGGER.warning("FT_VLLM_FUSED_TP needs eager execution (enforce_eager); keeping vLLM's all-reduce")
            return
        from vllm.distributed.parallel_state import get_tp_group

        from flextensor_b200.contrib.vllm.tp_patch import patch_row_parallel

        max_rows = self.vllm_config.scheduler_config.max_num_batched_tokens
        patch_row_parallel(self.model_runner.get_model(), max_rows, get_tp_group().cpu_group)

    def _load_shared(self, cfg, *args, **kwargs) -> None:
        """Data-parallel replicas sharing one host copy of the weights (``contrib/vllm/shared.py``):
        vLLM loads through the ``flextensor_shm`` format, which restores the model from the saved
        profile through a shared session (creator loads the checkpoint, followers attach)."""
        import atexit

        from vllm.model_executor.offloader.base import NoopOffloader, get_offloader, set_offloader

        import flextensor_b200 as ft
        from flextensor_b200.contrib.vllm.shared import SHM_LOAD_FORMAT, SharedLoad, active_shared_load
        from flextensor_b200.shared_offload import SharedOffloadSession

        prev = get_offloader()
        if not isinstance(prev, NoopOffloader):
            raise FlexTensorWorkerError(f"another vLLM offloader is active: {type(prev).__name__}")
        session = SharedOffloadSession(cfg.shm_namespace, wait_timeout=cfg.shm_wait_timeout)
        lc = self.vllm_config.load_config
        ctx = SharedLoad(session=session, config=cfg, profile_directory=cfg.profile_storage_dir, device=self.device,
                         underlying_format=lc.load_format, manager_name=MANAGER_NAME)
        boot = FlexTensorBootstrapOffloader()
        set_offloader(boot)
        orig = lc.load_format
        try:
            lc.load_format = SHM_LOAD_FORMAT
            try:
                with active_shared_load(ctx):
                    super().load_model(*args, **kwargs)
            finally:
                lc.load_format = orig
            if ctx.model is None or ctx.model is not self.model_runner.get_model():
                raise FlexTensorWorkerError("the shared load did not hand its model to the model runner")
            om = ft.get_offload_manager(MANAGER_NAME)
            boot.manager = om
            self._ft_manager = om
            self._ft_session = session
            atexit.register(session.close)
            LOGGER.info("FlexTensor shared host weights: role=%s namespace=%s", ctx.role, cfg.shm_namespace)
        except BaseException:
            try:
                session.close()
            finally:
                set_offloader(prev)
            raise

    def load_model(self, *args, **kwargs) -> None:
        if self.device.index is None:
            raise FlexTensorWorkerError(f"worker device needs an explicit index, got {self.device}")
        cfg = load_config(gpu_device=self.device.index)
        if not cfg.enabled:
            super().load_model(*args, **kwargs)
            self._maybe_fuse_tp()
            return
        if kwargs.get("load_dummy_weights"):
            raise FlexTensorWorkerError("load_dummy_weights=True is not supported")
        _validate(self.vllm_config, cfg)
        from flextensor_b200.contrib.vllm.graph_join import install_segment_join

        install_segment_join()  # copy stream joined at every eager break of a graph capture
        inc, exc = resolve_vllm_patterns(cfg)
        from vllm.config import CompilationMode, CUDAGraphMode

        comp = self.vllm_config.compilation_config
        external_compile = comp.mode == CompilationMode.VLLM_COMPILE
        graphs = comp.cudagraph_mode is not None and comp.cudagraph_mode != CUDAGraphMode.NONE
        timing = cfg.offload_timing
        if timing != "off":
            timing = "cuda_graph" if graphs else "eager"
        cfg = cfg.model_copy(update={"include_patterns": inc, "exclude_patterns": exc,
                                     "external_compile": external_compile, "offload_timing": timing})

        if cfg.shm_enabled:
            from flextensor_b200.contrib.vllm.shared import validate_shared_topology

            validate_shared_topology(self.vllm_config, cfg)
            self._load_shared(cfg, *args, **kwargs)
            return

        from vllm.model_executor.offloader.base import NoopOffloader, get_offloader, set_offloader

        prev = get_offloader()
        if not isinstance(prev, NoopOffloader):
            raise FlexTensorWorkerError(f"another vLLM offloader is active: {type(prev).__name__}")
        boot = FlexTensorBootstrapOffloader()
        set_offloader(boot)
        import flextensor_b200 as ft

        om = ft.get_offload_manager(MANAGER_NAME)
        try:
            super().load_model(*args, **kwargs)
            raw = self.model_runner.get_model()
            ensure_drafter_on_device(self.model_runner, self.device)
            before = torch.cuda.memory_allocated(self.device)
            prof = cfg.profile_storage_dir
            if prof and os.path.exists(os.path.join(prof, "profile.json")):
                om.set_config(cfg)
                om.load_profile(prof)
                om.offload(raw, cfg)
            else:
                om.offload_static(raw, cfg)
            boot.manager = om
            self._ft_manager = om
            self.model_runner.model_memory_usage += torch.cuda.memory_allocated(self.device) - before
            self._maybe_fuse_tp()
            LOGGER.info("FlexTensor took over %s: %.2f GB staged on host, ring slots %.2f GB",
                        type(raw).__name__, boot.staged_bytes / 1e9,
                        om.get_gpu_memory_usage().blocks_bytes / 1e9)
        except Exception:
            try:
                om.release()
            finally:
                set_offloader(prev)
            raise
