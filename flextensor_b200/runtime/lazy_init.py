"""Profile-driven lazy model construction (``src/flextensor/lazy_model_init.py:22-604``).

``load_model_from_profile`` builds the model with parameters on the ``meta``
device, then materialises from a safetensors file: tensors the profile keeps
resident (``gpu_tensors_names``) are loaded straight onto the device, streamed
tensors are loaded into host memory (the TensorManager packs them into host
blocks later). Only keys the model owns are read.
"""

from __future__ import annotations

import torch
from torch import nn


def load_specific_keys(path: str, keys: list[str], device: str | torch.device = "cpu",
                       strict: bool = False) -> dict[str, torch.Tensor]:
    from safetensors import safe_open

    out: dict[str, torch.Tensor] = {}
    with safe_open(path, framework="pt", device=str(device)) as f:
        have = set(f.keys())
        missing = [k for k in keys if k not in have]
        if missing and strict:
            raise KeyError(f"{len(missing)} profile keys missing from {path}: {missing[:5]}")
        for k in keys:
            if k in have:
                out[k] = f.get_tensor(k)
    return out


def create_split_device_model(model_class: type[nn.Module], model_args: tuple = (), model_kwargs: dict | None = None,
                              param_device: str = "meta", buffer_device: str = "cpu") -> nn.Module:
    with torch.device(param_device):
        model = model_class(*model_args, **(model_kwargs or {}))
    for mod in model.modules():
        for name, b in list(mod._buffers.items()):
            if b is not None and b.device.type == "meta":
                mod._buffers[name] = torch.zeros(b.shape, dtype=b.dtype, device=buffer_device)
    return model


def _assign(model: nn.Module, name: str, tensor: torch.Tensor) -> None:
    mod_path, _, leaf = name.rpartition(".")
    mod = model.get_submodule(mod_path) if mod_path else model
    old = getattr(mod, leaf)
    if isinstance(old, nn.Parameter):
        setattr(mod, leaf, nn.Parameter(tensor.to(old.dtype), requires_grad=False))
    else:
        mod._buffers[leaf] = tensor


def load_model_from_profile(tensor_manager, profile_directory: str, model_class: type[nn.Module],
                            model_args: tuple = (), safetensor_path: str | None = None,
                            model_kwargs: dict | None = None, buffer_device: str | None = None,
                            diagnose: bool = False, strict: bool = False) -> nn.Module:
    if safetensor_path is None:
        raise ValueError("safetensor_path is required")
    dev = buffer_device or str(tensor_manager.device)
    state = tensor_manager.load_state(profile_directory)
    model = create_split_device_model(model_class, model_args, model_kwargs, "meta", dev).eval()
    names = [n for n, _ in model.named_parameters()]
    gpu_names = set(state.gpu_tensors_names)
    on_gpu = load_specific_keys(safetensor_path, [n for n in names if n in gpu_names], dev, strict)
    on_host = load_specific_keys(safetensor_path, [n for n in names if n not in gpu_names], "cpu", strict)
    for n, t in {**on_gpu, **on_host}.items():
        _assign(model, n, t)
    if diagnose:
        still_meta = [n for n, p in model.named_parameters() if p.device.type == "meta"]
        if still_meta:
            raise RuntimeError(f"parameters left on meta after load: {still_meta[:5]}")
    return model
