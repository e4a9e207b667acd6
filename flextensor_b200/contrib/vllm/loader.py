"""Host-first model loading for offloaded vLLM models (``--load-format flextensor``).

vLLM normally builds the model on the GPU and loads the checkpoint into it there. A model that
only fits because FlexTensor will stream most of its weights cannot be built that way. This
loader works in two phases:

1. Build the model on the host and stream the checkpoint into it. vLLM's post-load weight
   processing (``process_weights_after_loading``: FP8 / online quantization repacking, MLA
   weight absorption, ...) is held back, because several of those kernels are CUDA-only.
2. Move one processing unit at a time to the GPU: the smallest ``<list>.<index>`` block that
   holds a module with post-load processing, e.g. ``model.layers.7``, so dependent projections
   such as MLA's ``kv_b_proj`` are processed together. Run the held-back processing there with
   vLLM's own routine, optionally JIT the unit's DeepGEMM kernels while it is resident, and move
   it back. Modules with processing outside any unit (e.g. a quantized ``lm_head``) get the same
   treatment one by one.

At most one unit is on the device at a time. If FlexTensor is disabled for this worker
(``FT_ENABLED`` unset or 0), the processed model is moved to the GPU at the end, so the stock
vLLM worker can serve it.

Reference behaviour: ``src/flextensor/contrib/vllm/loader.py:91-304`` (``FlexTensorModelLoader``).
"""

from __future__ import annotations

import contextlib
import logging
import re
from collections.abc import Iterator

import torch
from torch import nn

LOGGER = logging.getLogger("vllm.flextensor_b200.loader")

_UNIT_RE = re.compile(r"^(.*?\.?[A-Za-z_]\w*\.\d+)(?:\.|$)")


def _has_post_load(module: nn.Module) -> bool:
    qm = getattr(module, "quant_method", None)
    if qm is not None and hasattr(qm, "process_weights_after_loading"):
        return True
    return _is_attention_with_post_load(module)


def _is_attention_with_post_load(module: nn.Module) -> bool:
    if not hasattr(module, "process_weights_after_loading"):
        return False
    try:
        from vllm.model_executor.layers.attention_layer_base import AttentionLayerBase
    except Exception:  # noqa: BLE001 - vLLM absent: only duck-typed attention layers
        return type(module).__name__.endswith("Attention")
    return isinstance(module, AttentionLayerBase)


def unit_name(module_name: str) -> str | None:
    """The processing unit of a module: the prefix ending at the first indexed container
    element (``model.layers.3.self_attn.qkv_proj`` -> ``model.layers.3``), else None."""
    m = _UNIT_RE.match(module_name)
    return m.group(1) if m else None


def processing_units(model: nn.Module) -> tuple[dict[str, nn.Module], list[tuple[str, nn.Module]]]:
    """Units (in model order) that contain a module with post-load processing, and the
    processing modules that lie outside every unit."""
    units: dict[str, nn.Module] = {}
    loose: list[tuple[str, nn.Module]] = []
    for name, mod in model.named_modules():
        if not name or not _has_post_load(mod):
            continue
        u = unit_name(name)
        if u is None:
            loose.append((name, mod))
        elif u not in units:
            units[u] = model.get_submodule(u)
    inside = tuple(u + "." for u in units)
    loose = [(n, m) for n, m in loose if not n.startswith(inside)]
    return units, loose


@contextlib.contextmanager
def hold_post_load_hooks(model: nn.Module) -> Iterator[int]:
    """While loading on the host, every quantization method's ``process_weights_after_loading``
    is a no-op (vLLM may call it as checkpoint shards complete); the methods come back on exit.
    Yields how many method objects were held."""
    held: list[tuple[object, object]] = []  # (method object, its own attribute or a sentinel)
    seen: set[int] = set()
    missing = object()
    for mod in model.modules():
        qm = getattr(mod, "quant_method", None)
        if qm is None or not hasattr(qm, "process_weights_after_loading") or id(qm) in seen:
            continue
        seen.add(id(qm))
        held.append((qm, getattr(qm, "__dict__", {}).get("process_weights_after_loading", missing)))
        qm.process_weights_after_loading = lambda layer: None
    try:
        yield len(held)
    finally:
        for qm, own in held:
            if own is missing:
                del qm.process_weights_after_loading
            else:
                qm.process_weights_after_loading = own


def plain_parameters(module: nn.Module) -> int:
    """Swap vLLM's loader-time parameter subclasses for plain ``nn.Parameter`` (their loading
    metadata is spent, and keeping the subclass can send quantization helpers recursing through
    ``__torch_function__``). Returns how many were swapped."""
    n = 0
    for mod in module.modules():
        for pname, p in list(mod.named_parameters(recurse=False)):
            if type(p) is nn.Parameter:
                continue
            setattr(mod, pname, nn.Parameter(p.detach(), requires_grad=p.requires_grad))
            n += 1
    return n


def _deep_gemm_warmup(module: nn.Module, max_tokens: int) -> None:
    """JIT the unit's DeepGEMM kernels while its weights are on the GPU (vLLM's post-load warmup
    would otherwise meet host-resident weights); failures only defer the JIT to first use."""
    try:
        import vllm.envs as envs
        from vllm.utils.deep_gemm import is_deep_gemm_supported

        if envs.VLLM_DEEP_GEMM_WARMUP == "skip" or not is_deep_gemm_supported():
            return
        from vllm.model_executor.warmup import deep_gemm_warmup as dgw

        dgw.deepgemm_fp8_gemm_nt_warmup(module, max_tokens)
        dgw.deepgemm_grouped_fp8_gemm_nt_contiguous_warmup(module, max_tokens)
    except Exception as e:  # noqa: BLE001
        LOGGER.debug("DeepGEMM warmup skipped for a unit: %s", e)


def _process_on(module: nn.Module, model_config, device: torch.device, max_tokens: int) -> None:
    from vllm.model_executor.model_loader.utils import process_weights_after_loading

    module.to(device)
    try:
        plain_parameters(module)
        process_weights_after_loading(module, model_config, device)
        _deep_gemm_warmup(module, max_tokens)
    finally:
        module.to("cpu")


def _register() -> type | None:
    try:
        from vllm.model_executor.model_loader import DefaultModelLoader, register_model_loader
    except Exception:  # noqa: BLE001 - vLLM absent: nothing to register
        return None

    @register_model_loader("flextensor")
    class FlexTensorModelLoader(DefaultModelLoader):
        """``load_format="flextensor"``: host build + load, then per-unit GPU post-processing."""

        def _prepare_weights(self, *args, **kwargs):
            fmt = self.load_config.load_format
            if fmt == "flextensor":  # the files are whatever the checkpoint holds
                self.load_config.load_format = "auto"
            try:
                return super()._prepare_weights(*args, **kwargs)
            finally:
                self.load_config.load_format = fmt

        def load_model(self, vllm_config, model_config, prefix: str = "") -> nn.Module:
            from vllm.model_executor.model_loader.utils import initialize_model
            from vllm.platforms import current_platform
            from vllm.utils.torch_utils import set_default_torch_dtype

            gpu = torch.device(vllm_config.device_config.device)
            cpu = torch.device("cpu")
            platform_type = current_platform.device_type
            prev_default = torch.get_default_device()
            try:
                # some model code allocates on the platform's device type: host it all
                current_platform.device_type = "cpu"
                torch.set_default_device(cpu)
                with set_default_torch_dtype(model_config.dtype):
                    model = initialize_model(vllm_config=vllm_config, model_config=model_config, prefix=prefix)
                    with hold_post_load_hooks(model) as held:
                        self.load_weights(model, model_config)
            finally:
                current_platform.device_type = platform_type
                torch.set_default_device(prev_default)
            units, loose = processing_units(model)
            LOGGER.info("FlexTensor loader: %d held-back method(s); post-processing %d unit(s) and %d "
                        "loose module(s) on %s one at a time", held, len(units), len(loose), gpu)
            max_tokens = vllm_config.scheduler_config.max_num_batched_tokens
            for name, mod in list(units.items()) + loose:
                try:
                    _process_on(mod, model_config, gpu, max_tokens)
                except Exception:
                    LOGGER.error("FlexTensor loader: post-processing %s failed", name)
                    raise
                torch.cuda.empty_cache()
            from flextensor_b200.config import load_config

            if not load_config(gpu_device=gpu.index or 0).enabled:
                model.to(gpu)  # nothing will stream the host weights: serve from the device
            return model.eval()

    return FlexTensorModelLoader


FlexTensorModelLoader = _register()
