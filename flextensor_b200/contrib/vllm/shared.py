"""Data-parallel vLLM replicas on one node sharing a single host copy of the offloaded weights.

vLLM's local data parallelism (``data_parallel_backend="mp"``) runs one engine process per
replica. With ``FT_SHM_ENABLED=1``, a saved profile (``FT_PROFILE_STORAGE_DIR`` with
``FT_PROFILE_READ_ONLY=1``) and an explicit ``FT_SHM_NAMESPACE``, the FlexTensor worker loads
the model through the ``flextensor_shm`` load format. That load goes through one
:class:`~flextensor_b200.shared_offload.SharedOffloadSession` per namespace:

* the first replica to start (the creator) loads the checkpoint with the configured format and
  publishes the resident tensors and the streamed weight blocks in POSIX shared memory;
* every other replica (a follower) builds the model on the meta device and materialises the
  resident tensors from the shared store. Its streamed weights are views of the same shared
  blocks: N replicas hold one host copy, not N. A follower runs only the attention layers'
  post-load hooks, and checks that they kept every registered tensor on its shared storage.

The supported topology is validated up front and fails closed, like the reference
(``src/flextensor/contrib/vllm/v2/worker.py:90-133``, ``v2/loader.py``): one node, TP = PP = 1,
no context parallelism, the unconverted generation model without quantization, LoRA or
speculative decoding, no expert parallelism, and checkpoint format ``auto``.
"""

from __future__ import annotations

import contextlib
import contextvars
import logging
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
from torch import nn

LOGGER = logging.getLogger("vllm.flextensor_b200.shared")
SHM_LOAD_FORMAT = "flextensor_shm"


class SharedTopologyError(RuntimeError):
    pass


def _fmt_name(load_format: Any) -> str:
    v = getattr(load_format, "value", load_format)
    return v if isinstance(v, str) else str(v)


def validate_shared_topology(vllm_config: Any, cfg: Any) -> None:
    """Raise :class:`SharedTopologyError` unless this engine can share its host weights."""
    if not cfg.profile_storage_dir or not cfg.profile_read_only:
        raise SharedTopologyError("shared host weights need FT_PROFILE_STORAGE_DIR and FT_PROFILE_READ_ONLY=1")
    if not cfg.shm_namespace:
        raise SharedTopologyError("shared host weights need an explicit FT_SHM_NAMESPACE")
    mc = vllm_config.model_config
    if getattr(mc, "runner_type", "generate") != "generate" or getattr(mc, "convert_type", "none") != "none":
        raise SharedTopologyError("shared host weights need the native, unconverted generation model")
    for what, value in (("quantization", getattr(mc, "quantization", None)),
                        ("LoRA", getattr(vllm_config, "lora_config", None)),
                        ("speculative decoding", getattr(vllm_config, "speculative_config", None))):
        if value is not None:
            raise SharedTopologyError(f"shared host weights do not support {what}")
    par = vllm_config.parallel_config
    sizes = {k: getattr(par, k, 1) for k in ("tensor_parallel_size", "pipeline_parallel_size",
                                             "prefill_context_parallel_size", "decode_context_parallel_size")}
    bad = {k: v for k, v in sizes.items() if v != 1}
    if bad:
        raise SharedTopologyError(f"shared host weights need TP = PP = PCP = DCP = 1, got {bad}")
    if getattr(par, "data_parallel_backend", "mp") != "mp" or getattr(par, "nnodes", 1) != 1:
        raise SharedTopologyError("shared host weights need single-node data parallelism (backend 'mp')")
    if getattr(par, "data_parallel_external_lb", False) or getattr(par, "data_parallel_hybrid_lb", False):
        raise SharedTopologyError("shared host weights do not support external or hybrid DP load balancing")
    if any(getattr(par, k, False) for k in ("enable_expert_parallel", "enable_eplb", "enable_ep_weight_filter")):
        raise SharedTopologyError("shared host weights do not support expert parallelism or EPLB")
    fmt = _fmt_name(getattr(getattr(vllm_config, "load_config", None), "load_format", "auto"))
    if fmt != "auto":
        raise SharedTopologyError(f"shared host weights need load_format 'auto', got {fmt!r}")


@dataclass
class SharedLoad:
    """What the worker hands to the ``flextensor_shm`` loader for one load."""

    session: Any                 # SharedOffloadSession
    config: Any                  # OffloadConfig
    profile_directory: str
    device: torch.device
    underlying_format: Any       # the checkpoint format the creator loads with
    manager_name: str = "vllm"
    role: str | None = None      # "creator" / "follower", set by the load
    model: nn.Module | None = field(default=None, repr=False)


_ACTIVE: contextvars.ContextVar[SharedLoad | None] = contextvars.ContextVar("ft_vllm_shared_load", default=None)


@contextlib.contextmanager
def active_shared_load(ctx: SharedLoad):
    if _ACTIVE.get() is not None:
        raise RuntimeError("a shared vLLM model load is already in progress in this context")
    token = _ACTIVE.set(ctx)
    try:
        yield ctx
    finally:
        _ACTIVE.reset(token)


def storage_snapshot(model: nn.Module) -> dict[tuple[str, str], tuple[torch.Tensor, int]]:
    """Every registered parameter / buffer with the address of its storage."""
    snap = {("param", n): (p, p.untyped_storage().data_ptr()) for n, p in model.named_parameters(remove_duplicate=False)}
    snap.update({("buffer", n): (b, b.untyped_storage().data_ptr())
                 for n, b in model.named_buffers(remove_duplicate=False)})
    return snap


def check_storage_unchanged(model: nn.Module, snap: dict[tuple[str, str], tuple[torch.Tensor, int]]) -> None:
    """A follower's post-load hooks must leave every registered tensor on its shared storage."""
    now = {("param", n): p for n, p in model.named_parameters(remove_duplicate=False)}
    now.update({("buffer", n): b for n, b in model.named_buffers(remove_duplicate=False)})
    problems = []
    for key, (t, ptr) in snap.items():
        cur = now.get(key)
        if cur is None:
            problems.append(f"{key[0]} {key[1]} removed")
        elif cur is not t:
            problems.append(f"{key[0]} {key[1]} replaced")
        elif cur.untyped_storage().data_ptr() != ptr:
            problems.append(f"{key[0]} {key[1]} moved to new storage")
    if problems:
        raise RuntimeError(f"follower post-load processing left the shared storage: {problems[:10]}")


def shared_load(ctx: SharedLoad, load_checkpoint: Callable[[], nn.Module], build_meta: Callable[[], nn.Module],
                follower_post_load: Callable[[nn.Module], None]) -> nn.Module:
    """Creator: ``load_checkpoint()``; follower: ``build_meta()`` (no concrete tensor allowed),
    materialised from the shared store, then ``follower_post_load`` under a storage check."""

    def creator():
        m = load_checkpoint()
        ctx.role = "creator"
        LOGGER.info("FlexTensor shared load: creator, checkpoint loaded")
        return m

    def follower():
        m = build_meta()
        concrete = [n for n, t in list(m.named_parameters()) + list(m.named_buffers()) if not t.is_meta]
        if concrete:
            raise RuntimeError(f"the follower's model skeleton holds concrete tensors: {concrete[:10]}")
        ctx.role = "follower"
        LOGGER.info("FlexTensor shared load: follower, checkpoint skipped")
        return m.eval()

    model = ctx.session.offload_from_profile(ctx.profile_directory, config=ctx.config, name=ctx.manager_name,
                                             creator_model_factory=creator, follower_model_factory=follower,
                                             materialize_device=ctx.device)
    if ctx.role == "follower":
        snap = storage_snapshot(model)
        follower_post_load(model)
        check_storage_unchanged(model, snap)
        LOGGER.info("FlexTensor shared load: follower post-load kept %d tensors on shared storage", len(snap))
    elif ctx.role != "creator":
        raise RuntimeError("the shared session returned without choosing a creator or follower role")
    ctx.model = model
    return model


def _attention_post_load(model: nn.Module, dtype: torch.dtype) -> None:
    from vllm.model_executor.layers.attention_layer_base import AttentionLayerBase

    for mod in model.modules():
        if isinstance(mod, AttentionLayerBase) and hasattr(mod, "process_weights_after_loading"):
            mod.process_weights_after_loading(dtype)


def _register() -> type | None:
    try:
        from vllm.model_executor.model_loader import DefaultModelLoader, get_model_loader, register_model_loader
    except Exception:  # noqa: BLE001 - vLLM absent
        return None

    @register_model_loader(SHM_LOAD_FORMAT)
    class FlexTensorSharedLoader(DefaultModelLoader):
        """``load_format="flextensor_shm"``: restore the model through the worker's shared session."""

        def load_model(self, vllm_config, model_config, prefix: str = "") -> nn.Module:
            from vllm.model_executor.model_loader.utils import initialize_model
            from vllm.utils.torch_utils import set_default_torch_dtype

            ctx = _ACTIVE.get()
            if ctx is None:
                raise RuntimeError("the flextensor_shm load format is set by the FlexTensor worker only")
            if ctx.model is not None:
                raise RuntimeError("this shared load already produced a model")
            if _fmt_name(ctx.underlying_format) == SHM_LOAD_FORMAT:
                raise RuntimeError("the shared loader cannot wrap itself")

            def load_checkpoint():
                fmt = self.load_config.load_format
                self.load_config.load_format = ctx.underlying_format
                try:
                    return get_model_loader(self.load_config).load_model(vllm_config=vllm_config,
                                                                         model_config=model_config, prefix=prefix)
                finally:
                    self.load_config.load_format = fmt

            def build_meta():
                with set_default_torch_dtype(model_config.dtype), torch.device("meta"):
                    return initialize_model(vllm_config=vllm_config, model_config=model_config, prefix=prefix)

            def follower_post_load(model):
                with ctx.device:
                    _attention_post_load(model, model_config.dtype)

            return shared_load(ctx, load_checkpoint, build_meta, follower_post_load)

    return FlexTensorSharedLoader


FlexTensorSharedLoader = _register()
