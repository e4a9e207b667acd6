"""Trap boundaries as opaque custom ops, so compiled graphs keep the prefetch schedule.

``flextensor_b200::pre_compute(Tensor(a!) carrier, str unit, int manager_id)``
and ``post_compute`` call the manager's loader ``enter``/``exit`` (same
contract as ``src/flextensor/custom_ops.py:267-328``). The carrier is declared
mutated so a compiler can neither drop nor reorder the calls relative to the
unit's compute; its values are never written. With ``external_compile`` the
patched unit forward is::

    pre_compute(carrier, unit, id); y = orig_forward(...); post_compute(carrier, unit, id)

and a caller can ``torch.compile`` each unit. Per-unit compiled timings
(CUDA events around the boundaries) are collected while profiling is enabled.
"""

from __future__ import annotations

import itertools
import weakref
from dataclasses import dataclass, field

import torch
from torch.library import Library

_LIB = Library("flextensor_b200", "FRAGMENT")
_LIB.define("pre_compute(Tensor(a!) carrier, str offload_unit_name, int manager_id) -> ()")
_LIB.define("post_compute(Tensor(a!) carrier, str offload_unit_name, int manager_id) -> ()")


@dataclass
class _State:
    manager: weakref.ref | None = None
    profiling: bool = False
    starts: dict = field(default_factory=dict)
    events: list = field(default_factory=list)


_STATES: dict[int, _State] = {}
_ids = itertools.count(1)


def register_manager(manager) -> int:
    mid = getattr(manager, "_custom_op_id", None)
    if mid is None:
        mid = next(_ids)
        manager._custom_op_id = mid
        _STATES[mid] = _State(manager=weakref.ref(manager))
    return mid


def _loader(mid: int):
    st = _STATES.get(mid)
    if st is None or st.manager is None:
        return None, st
    om = st.manager()
    tm = om.get_tensor_manager() if om is not None else None
    return (tm.loader if tm is not None else None), st


def _pre_impl(carrier: torch.Tensor, offload_unit_name: str, manager_id: int) -> None:
    loader, st = _loader(manager_id)
    if loader is not None:
        loader.enter(offload_unit_name)
    if st is not None and st.profiling and carrier.is_cuda:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        st.starts[offload_unit_name] = e


def _post_impl(carrier: torch.Tensor, offload_unit_name: str, manager_id: int) -> None:
    loader, st = _loader(manager_id)
    if st is not None and st.profiling and carrier.is_cuda and offload_unit_name in st.starts:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        st.events.append((offload_unit_name, st.starts.pop(offload_unit_name), e))
    if loader is not None:
        loader.exit(offload_unit_name)


def _fake(carrier: torch.Tensor, offload_unit_name: str, manager_id: int) -> None:
    return None


_LIB.impl("pre_compute", _pre_impl, "CompositeExplicitAutograd")
_LIB.impl("post_compute", _post_impl, "CompositeExplicitAutograd")
torch.library.register_fake("flextensor_b200::pre_compute", _fake, lib=_LIB)
torch.library.register_fake("flextensor_b200::post_compute", _fake, lib=_LIB)


def enable_compiled_profiling(manager_id: int) -> None:
    st = _STATES.setdefault(manager_id, _State())
    st.profiling, st.starts, st.events = True, {}, []


def disable_compiled_profiling(manager_id: int) -> None:
    st = _STATES.get(manager_id)
    if st is not None:
        st.profiling = False
        st.starts.clear()


def collect_compiled_layer_durations(manager_id: int) -> dict[str, list[float]]:
    st = _STATES.get(manager_id)
    out: dict[str, list[float]] = {}
    if st is None:
        return out
    for name, a, b in st.events:
        b.synchronize()
        out.setdefault(name, []).append(a.elapsed_time(b))
    st.events = []
    return out


def carrier_for(device: torch.device) -> torch.Tensor:
    return torch.zeros(1, device=device)
