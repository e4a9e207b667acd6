"""Diffusers pipelines: offload each denoiser of a pipeline under its own named manager.

Wan2.2 A14B pipelines carry two transformers (high-noise ``transformer`` and low-noise
``transformer_2``); each gets its own OffloadManager so each learns its own schedule and the
pair's ring slots are sized independently. Everything else in the pipeline (VAE, text
encoder) is moved to the GPU. Works on any object with a ``components`` dict of modules
(diffusers ``DiffusionPipeline``) or plain attributes.

    pipe = offload_pipeline(pipe, OffloadConfig(include_patterns=WAN_INCLUDE_PATTERNS))
    pipe(...)                      # discovery + profiling passes, then inference
    release_pipeline(pipe)

Mirrors ``examples/diffusers/quickstart/wan_t2v.py:37-65`` of the reference.
"""

from __future__ import annotations

from typing import Any

import torch

import flextensor_b200 as ft

WAN_INCLUDE_PATTERNS = ["rope", "patch_embedding", "condition_embedder", "blocks.*", "norm_out", "proj_out"]
DEFAULT_COMPONENTS = ("transformer", "transformer_2")


def _components(pipe: Any) -> dict[str, Any]:
    comps = getattr(pipe, "components", None)
    if isinstance(comps, dict):
        return comps
    return {k: v for k, v in vars(pipe).items() if isinstance(v, torch.nn.Module)}


def manager_name(component: str) -> str:
    return component.replace("_", "")


def offload_pipeline(pipe: Any, config: ft.OffloadConfig, components: tuple[str, ...] = DEFAULT_COMPONENTS,
                     device: str | torch.device | None = None, compile_fn=None) -> Any:
    """Offload ``components`` (each under manager ``manager_name(component)``); move the rest to
    ``device`` (default: the config's GPU)."""
    dev = torch.device(device) if device is not None else (
        torch.device("cuda", config.gpu_device) if torch.cuda.is_available() else torch.device("cpu"))
    comps = _components(pipe)
    for name, mod in comps.items():
        if isinstance(mod, torch.nn.Module) and name not in components:
            mod.to(dev)
    for name in components:
        mod = comps.get(name)
        if mod is None:
            continue
        wrapped = ft.offload(mod, config=config, name=manager_name(name), compile_fn=compile_fn)
        setattr(pipe, name, wrapped)
        if isinstance(getattr(pipe, "components", None), dict) and name in pipe.components:
            try:
                pipe.components[name] = wrapped
            except TypeError:
                pass
    return pipe


def save_pipeline_profiles(pipe: Any, directory: str, components: tuple[str, ...] = DEFAULT_COMPONENTS) -> None:
    """One ``profile.json`` per offloaded component under ``directory/<component>``."""
    import os

    for name in components:
        om = ft.get_offload_manager(manager_name(name))
        if om.get_tensor_manager() is not None:
            om.save_profile(os.path.join(directory, name))


def offload_pipeline_from_profiles(pipe: Any, directory: str, config: ft.OffloadConfig,
                                   components: tuple[str, ...] = DEFAULT_COMPONENTS, device=None) -> Any:
    """Skip discovery/profiling: apply the saved per-component plans."""
    import os

    dev = torch.device(device) if device is not None else (
        torch.device("cuda", config.gpu_device) if torch.cuda.is_available() else torch.device("cpu"))
    comps = _components(pipe)
    for name, mod in comps.items():
        if isinstance(mod, torch.nn.Module) and name not in components:
            mod.to(dev)
    for name in components:
        mod = comps.get(name)
        if mod is None:
            continue
        setattr(pipe, name, ft.offload_from_profile(mod, os.path.join(directory, name), config=config,
                                                    name=manager_name(name)))
    return pipe


def release_pipeline(pipe: Any, components: tuple[str, ...] = DEFAULT_COMPONENTS) -> None:
    for name in components:
        ft.release(manager_name(name))
