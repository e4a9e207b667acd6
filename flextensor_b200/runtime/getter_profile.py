"""``profile_mode="getter"``: parameter reads resolved by per-module property getters.

Parity with ``src/flextensor/tensor_manager.py:226-318`` (``extend_nn_module`` /
``_make_tensor_getter``). While profiling, every module that directly owns offloadable
parameters is given a dynamically created subclass of its own class whose properties shadow
those parameter names. The Parameter objects never change (no ``.data`` rebinding, so tied
weights, external references and identity-keyed caches see the host tensors throughout):

* inside a trap the getter returns the device copy the trap loaded for that parameter, with the
  parameter's inner fields (``weight.weight_scale``, loader metadata) carried onto the copy;
* a read outside the owning trap (a cross-unit read discovery did not see) promotes that
  parameter to the device for good, with a warning naming it and the bytes lost to offloading,
  so the profile stays runnable;
* on leaving PROFILING every module gets its original class back.
"""

from __future__ import annotations

import logging

import torch
from torch import nn

from flextensor_b200.core.visitor import carry_inner_fields

LOGGER = logging.getLogger(__name__)


class GetterProfile:
    def __init__(self, tm):
        self.tm = tm
        self.loaded: dict[int, torch.Tensor] = {}   # id(param) -> device copy for the running trap
        self._swapped: dict[nn.Module, type] = {}
        self.promoted: set[int] = set()

    def install(self) -> None:
        tm = self.tm
        offloadable = {id(tm.params_by_tid[t]): t for t in tm.owner}
        for mod in tm.model.modules():
            names = [n for n, p in mod._parameters.items() if p is not None and id(p) in offloadable]
            if not names or mod in self._swapped:
                continue
            base = type(mod)
            props = {n: property(self._getter(mod._parameters[n], offloadable[id(mod._parameters[n])]))
                     for n in names}
            sub = type(base.__name__, (base,), props)
            self._swapped[mod] = base
            mod.__class__ = sub

    def _getter(self, param: nn.Parameter, tid: int):
        gp = self
        pid = id(param)

        def get(_self):
            dev = gp.loaded.get(pid)
            if dev is not None:
                return dev
            tm = gp.tm
            if param.device != tm.device and not param.is_meta and tm.device.type != "cpu":
                if pid not in gp.promoted:
                    LOGGER.warning("cross-unit read: %s was read outside its offload unit during getter "
                                   "profiling and is now resident on %s (%.2f MiB no longer offloaded)",
                                   tm.id_to_name.get(tid, tid), tm.device, param.nbytes / 2**20)
                    gp.promoted.add(pid)
                gp.tm.promote_resident(tid)
            return param

        return get

    def load(self, tids: list[int]) -> None:
        tm = self.tm
        for t in tids:
            p = tm.params_by_tid[t]
            d = tm.host[t].to(tm.device, non_blocking=True)
            carry_inner_fields(p, d)
            self.loaded[id(p)] = d

    def unload(self, tids: list[int]) -> None:
        for t in tids:
            self.loaded.pop(id(self.tm.params_by_tid[t]), None)

    def uninstall(self) -> None:
        for mod, base in self._swapped.items():
            mod.__class__ = base
        self._swapped.clear()
        self.loaded.clear()

    @property
    def installed(self) -> bool:
        return bool(self._swapped)
