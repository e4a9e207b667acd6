"""Profile-driven lazy model construction (``src/flextensor/lazy_model_init.py:22-604``).

``load_model_from_profile`` builds the model with parameters on the ``meta``
device, then materialises from a safetensors file: tensors the profile keeps
resident (``gpu_tensors_names``) are loaded straight onto the device, streamed
tensors are loaded into host memory (the TensorManager packs them into host
blocks later), persistent buffers found in the file onto the buffer device. Only keys the
model owns are read.

Nested parameter links (a registered parameter carrying an attribute that points at another
registered tensor, e.g. ``linear.weight.scale is linear.scale`` in quantized layers, or a flag
such as ``weight.is_packed``) live in the parameter objects' ``__dict__``, not in the state
dict, so materialising new ``Parameter`` objects would drop them. :class:`LinkTracker` records
them on the meta model (by target name) and puts them back on the loaded tensors.
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
    _materialize_buffers(model, buffer_device)
    return model


def _materialize_buffers(model: nn.Module, buffer_device: str) -> None:
    for mod in model.modules():
        for name, b in list(mod._buffers.items()):
            if b is not None and b.device.type == "meta":
                mod._buffers[name] = torch.zeros(b.shape, dtype=b.dtype, device=buffer_device)


class LinkTracker:
    """The attributes that registered parameters and buffers of a model carry, by owner name.

    ``links[(owner, attr)] = target`` for an attribute holding another registered tensor of the
    model (stored by name, restored to whatever tensor sits under that name after loading);
    ``plain[(owner, attr)] = value`` for non-tensor attributes (copied as they are). Private
    attributes (leading ``_``) are not tracked."""

    def __init__(self) -> None:
        self.links: dict[tuple[str, str], str] = {}
        self.plain: dict[tuple[str, str], object] = {}
        self.ties: dict[str, str] = {}  # alias name -> the name a shared parameter loads under

    @staticmethod
    def _named(model: nn.Module) -> dict[str, torch.Tensor]:
        named = dict(model.named_parameters(remove_duplicate=False))
        named.update(dict(model.named_buffers(remove_duplicate=False)))
        return named

    @classmethod
    def capture(cls, model: nn.Module) -> "LinkTracker":
        t = cls()
        named = cls._named(model)
        by_id: dict[int, str] = {}
        for n, x in named.items():
            first = by_id.setdefault(id(x), n)
            if first != n:
                t.ties[n] = first
        for owner, x in named.items():
            if owner in t.ties:
                continue
            for attr, v in list(getattr(x, "__dict__", {}).items()):
                if attr.startswith("_"):
                    continue
                if isinstance(v, torch.Tensor):
                    target = by_id.get(id(v))
                    if target is not None:
                        t.links[(owner, attr)] = target
                else:
                    t.plain[(owner, attr)] = v
        return t

    def restore(self, model: nn.Module) -> int:
        """Re-attach every tracked attribute to the tensors now registered in ``model``;
        returns how many were set. A name that no longer exists raises KeyError. Tied
        parameters (one tensor under several names) are re-tied first."""
        n = 0
        for alias, canon in self.ties.items():
            mod_path, _, leaf = alias.rpartition(".")
            mod = model.get_submodule(mod_path) if mod_path else model
            target = self._named(model)[canon]
            if isinstance(target, nn.Parameter):
                setattr(mod, leaf, target)
            else:
                mod._buffers[leaf] = target
            n += 1
        named = self._named(model)
        for (owner, attr), v in self.plain.items():
            setattr(named[owner], attr, v)
            n += 1
        for (owner, attr), target in self.links.items():
            setattr(named[owner], attr, named[target])
            n += 1
        return n

    def __len__(self) -> int:
        return len(self.links) + len(self.plain) + len(self.ties)


def create_split_device_model_with_tracking(model_class: type[nn.Module], model_args: tuple = (),
                                            model_kwargs: dict | None = None, param_device: str = "meta",
                                            buffer_device: str = "cpu") -> tuple[nn.Module, LinkTracker]:
    """:func:`create_split_device_model` plus the model's nested parameter links; call
    ``tracker.restore(model)`` after the weights are loaded (new tensor objects)."""
    with torch.device(param_device):
        model = model_class(*model_args, **(model_kwargs or {}))
    tracker = LinkTracker.capture(model)  # before the buffers become new tensors
    _materialize_buffers(model, buffer_device)
    tracker.restore(model)
    return model, tracker


def _non_persistent(model: nn.Module, name: str) -> set[str]:
    mod_path = name.rpartition(".")[0]
    mod = model.get_submodule(mod_path) if mod_path else model
    return set(getattr(mod, "_non_persistent_buffers_set", ()))


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
    model, tracker = create_split_device_model_with_tracking(model_class, model_args, model_kwargs, "meta", dev)
    model.eval()
    names = [n for n, _ in model.named_parameters()]
    gpu_names = set(state.gpu_tensors_names)
    on_gpu = load_specific_keys(safetensor_path, [n for n in names if n in gpu_names], dev, strict)
    on_host = load_specific_keys(safetensor_path, [n for n in names if n not in gpu_names], "cpu", strict)
    for n, t in {**on_gpu, **on_host}.items():
        _assign(model, n, t)
    # persistent buffers saved with the weights (running statistics, quantization zero points)
    persistent = [n for n, _ in model.named_buffers()
                  if n.rpartition(".")[2] not in _non_persistent(model, n)]
    for n, t in load_specific_keys(safetensor_path, persistent, dev, False).items():
        _assign(model, n, t)
    tracker.restore(model)
    if diagnose:
        still_meta = [n for n, p in model.named_parameters() if p.device.type == "meta"]
        if still_meta:
            raise RuntimeError(f"parameters left on meta after load: {still_meta[:5]}")
    return model
