"""Offload-unit selection ("traps") and tensor identity.

A unit is the outermost module matched by ``include_patterns``
(``src/flextensor/offload_manager.py:2701-2792``, ``src/flextensor/tensor_discovery.py:538-569``):

* name patterns that match a module path select modules (``*`` = one segment);
* name patterns that only match parameter paths are parameter filters: the
  module pattern is the pattern minus its last segment, and only matching
  parameters of the unit are offloaded;
* ``class:`` patterns select modules by class;
* ``exclude_patterns`` (``*`` recursive) drop modules and parameters; a
  ``class:`` exclude cascades to every descendant parameter.

Container modules without their own ``forward`` (``ModuleList``/``ModuleDict``/
``Sequential`` is kept, it has a forward) are replaced by their children so
a pattern like ``*`` on a model whose blocks live in a ``ModuleList`` still
yields one unit per block.

Tensor ids are positions in ``named_parameters()`` order (duplicates removed),
so the same model built in another process gets the same ids; ``profile.json``
still rebinds by name.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import nn

from flextensor_b200.utils.patterns import (
    get_class_matched_module_paths,
    matches_any_class_pattern,
    matches_any_pattern,
    partition_patterns,
)


@dataclass
class Unit:
    label: str
    module: nn.Module
    params: list[tuple[str, nn.Parameter]] = field(default_factory=list)
    """(full dotted name, parameter) of the unit's offloadable parameters."""
    kept: list[tuple[str, nn.Parameter]] = field(default_factory=list)
    """Parameters of the unit filtered out by parameter patterns / excludes (stay resident)."""


def _is_container(m: nn.Module) -> bool:
    return isinstance(m, (nn.ModuleList, nn.ModuleDict))


def named_model_tensors(model: nn.Module) -> list[tuple[str, nn.Parameter]]:
    return list(model.named_parameters(remove_duplicate=True))


def tensor_id_map(model: nn.Module) -> tuple[dict[int, str], dict[str, int]]:
    names = [n for n, _ in named_model_tensors(model)]
    return dict(enumerate(names)), {n: i for i, n in enumerate(names)}


def select_units(model: nn.Module, include_patterns: list[str], exclude_patterns: list[str]) -> list[Unit]:
    """Units in module-registration order (the usual execution order)."""
    inc = partition_patterns(include_patterns)
    exc = partition_patterns(exclude_patterns)
    modules = dict(model.named_modules())
    mod_paths = [p for p in modules if p]
    param_paths = [n for n, _ in model.named_parameters()]

    module_pats: list[str] = []
    param_filters: list[str] = []
    for pat in inc.name_patterns:
        if any(matches_any_pattern(p, [pat], recursive_star=False) for p in mod_paths):
            module_pats.append(pat)
        elif any(matches_any_pattern(p, [pat], recursive_star=True) for p in param_paths):
            parent = pat.rsplit(".", 1)[0] if "." in pat else ""
            if parent:
                module_pats.append(parent)
            param_filters.append(pat)

    picked: set[str] = {p for p in mod_paths if matches_any_pattern(p, module_pats, recursive_star=False)}
    picked |= get_class_matched_module_paths(model, inc.class_patterns)

    # containers -> children
    changed = True
    while changed:
        changed = False
        for p in list(picked):
            if _is_container(modules[p]):
                picked.discard(p)
                picked |= {f"{p}.{c}" for c, _ in modules[p].named_children()}
                changed = True

    # excludes on modules
    exc_mod = {p for p in picked if matches_any_pattern(p, exc.name_patterns, recursive_star=True)}
    exc_mod |= {p for p in picked if matches_any_class_pattern(type(modules[p]), exc.class_patterns)}
    picked -= exc_mod

    # outermost only
    ordered = [p for p in mod_paths if p in picked]
    outer = [p for p in ordered if not any(p.startswith(q + ".") for q in picked if q != p)]

    class_excluded_roots = get_class_matched_module_paths(model, exc.class_patterns)
    units = []
    seen_param_ids: set[int] = set()
    for path in outer:
        mod = modules[path]
        u = Unit(label=path, module=mod)
        for local, prm in mod.named_parameters(remove_duplicate=True):
            full = f"{path}.{local}"
            if id(prm) in seen_param_ids:
                continue
            seen_param_ids.add(id(prm))
            keep = True
            if param_filters and matches_any_pattern(path, [f.rsplit(".", 1)[0] for f in param_filters],
                                                     recursive_star=False):
                keep = matches_any_pattern(full, param_filters, recursive_star=True)
            parts = full.split(".")
            prefixes = [".".join(parts[:i]) for i in range(1, len(parts) + 1)]
            if any(matches_any_pattern(pp, exc.name_patterns, recursive_star=True) for pp in prefixes):
                keep = False
            if any(full.startswith(r + ".") for r in class_excluded_roots):
                keep = False
            (u.params if keep else u.kept).append((full, prm))
        units.append(u)
    return units


def param_owner_label(units: list[Unit]) -> dict[int, str]:
    """id(parameter) -> unit label for offloadable parameters."""
    return {id(p): u.label for u in units for _, p in u.params}


def storage_bytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()
