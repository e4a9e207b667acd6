"""Loader for the prebuilt native extension and thin Python wrappers around it.

The extension is imported straight from the in-tree build directory. On a
machine with a CUDA device the extension is REQUIRED: every op and the
transfer engine raise if it is missing instead of silently falling back.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import sys
import threading

import torch

from flextensor_b200.ops.build import MODULE_NAME, built_library
from flextensor_b200.instrumentation.core import instrumentable

_lock = threading.Lock()
_mod = None


class NativeExtensionMissing(RuntimeError):
    pass


def lib():
    """The loaded ``ft_b200_C`` module (raises :class:`NativeExtensionMissing` if not built)."""
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        if MODULE_NAME in sys.modules:
            _mod = sys.modules[MODULE_NAME]
            return _mod
        path = built_library()
        if path is None:
            raise NativeExtensionMissing(
                "flextensor_b200 native extension is not built; run `python -m flextensor_b200.ops.build` "
                "(or __graft_entry__.build())")
        import torch  # noqa: F401  (libtorch symbols must be loaded first)

        loader = importlib.machinery.ExtensionFileLoader(MODULE_NAME, str(path))
        spec = importlib.util.spec_from_file_location(MODULE_NAME, str(path), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        sys.modules[MODULE_NAME] = mod
        _mod = mod
        return mod


def available() -> bool:
    try:
        lib()
        return True
    except NativeExtensionMissing:
        return False


def pinned_empty(nbytes: int) -> torch.Tensor:
    """``nbytes`` uint8 CPU tensor in page-locked memory of exactly that size (no rounding)."""
    return lib().pinned_empty(int(nbytes))


def host_register(ptr: int, nbytes: int) -> None:
    lib().host_register(int(ptr), int(nbytes))


def host_unregister(ptr: int) -> None:
    lib().host_unregister(int(ptr))


def device_error(reset: bool = False) -> int:
    return lib().device_error(reset)


@instrumentable
class NativeTransferEngine:
    """C++ ring-slot engine; same interface as ``PyTransferEngine`` (string keys mapped to ints)."""

    def __init__(self, device: torch.device, n_slots: int, timing: bool = False, external_events: bool = False,
                 max_keys: int = 4096):
        self.device = torch.device(device)
        self.timing = timing
        self._keys: dict[str, int] = {}
        self._names: list[str] = []
        self._e = lib().TransferEngine(self.device.index or 0, int(n_slots), int(max_keys), bool(timing))

    def _k(self, key: str) -> int:
        k = self._keys.get(key)
        if k is None:
            k = len(self._names)
            self._keys[key] = k
            self._names.append(key)
        return k

    def begin(self) -> None:
        self._e.begin()

    def submit(self, slot: int, dst: torch.Tensor, src: torch.Tensor, key: str) -> None:
        self._e.submit(int(slot), dst, src, self._k(key))

    def wait_ready(self, key: str) -> None:
        k = self._keys.get(key)
        if k is not None:
            self._e.wait_ready(k)

    def finish_use(self, slot: int) -> None:
        self._e.finish_use(int(slot))

    def join(self) -> None:
        self._e.join()

    def synchronize(self) -> None:
        self._e.synchronize()

    def reset(self) -> None:
        self._e.synchronize()

    def take_records(self):
        from flextensor_b200.runtime.engine import TransferRecord

        out = []
        for key, nbytes, tms, wms in self._e.take_samples():
            r = TransferRecord(self._names[key], nbytes)
            r.start, r.end, r.wait_start, r.wait_end = None, None, None, None
            r.transfer_ms, r.wait_ms = tms, wms
            out.append(r)
        return out
