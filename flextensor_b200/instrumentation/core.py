"""Registry, decorator, serializer and dumper for constructor instrumentation.

Reference behaviour: ``instrumentation/decorator.py:22`` (wrap ``__init__``, bind the
arguments to the signature, record only when enabled, never let recording break the
constructor), ``registry.py:32`` (thread-safe singleton), ``serializers.py:189`` (JSON-safe
values with cycle protection), ``dumper.py:41,105`` (atomic write, timestamped directory),
``host_resources.py:12`` (psutil memory snapshot).
"""

from __future__ import annotations

import dataclasses
import enum
import functools
import inspect
import json
import logging
import os
import threading
from dataclasses import dataclass, field
from datetime import datetime
from pathlib import Path
from typing import Any, Mapping

import torch

LOGGER = logging.getLogger("flextensor_b200.instrumentation")
_MAX_DEPTH = 6
_MAX_ITEMS = 256


@dataclass
class ComponentRecord:
    class_name: str
    module_path: str
    init_timestamp: str
    args: dict[str, Any] = field(default_factory=dict)


class InstrumentationRegistry:
    """Process-wide, thread-safe store of :class:`ComponentRecord`. Disabled by default."""

    _instance: "InstrumentationRegistry | None" = None
    _create_lock = threading.Lock()

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._records: list[ComponentRecord] = []
        self._enabled = False

    @classmethod
    def get_instance(cls) -> "InstrumentationRegistry":
        inst = cls._instance
        if inst is None:
            with cls._create_lock:
                if cls._instance is None:
                    cls._instance = cls()
                inst = cls._instance
        return inst

    @property
    def enabled(self) -> bool:
        return self._enabled

    @enabled.setter
    def enabled(self, value: bool) -> None:
        self._enabled = bool(value)

    def register(self, class_name: str, module_path: str, args: dict[str, Any]) -> None:
        if not self._enabled:
            return
        rec = ComponentRecord(class_name, module_path, datetime.now().isoformat(), dict(args))
        with self._lock:
            self._records.append(rec)

    def get_records(self) -> list[ComponentRecord]:
        with self._lock:
            return list(self._records)

    def clear(self) -> None:
        with self._lock:
            self._records.clear()

    def __len__(self) -> int:
        with self._lock:
            return len(self._records)


# ----------------------------------------------------------------------------- serializer
def _tensor_summary(t: torch.Tensor) -> dict[str, Any]:
    return {"type": "Tensor", "shape": list(t.shape), "dtype": str(t.dtype), "device": str(t.device),
            "numel": int(t.numel()), "nbytes": int(t.numel() * t.element_size())}


def _ser(v: Any, seen: set[int], depth: int) -> Any:
    if v is None or isinstance(v, (bool, int, float, str)):
        return v
    if isinstance(v, enum.Enum):
        return v.value if isinstance(v.value, (int, str)) else v.name
    if isinstance(v, (torch.dtype, torch.device, torch.Size)):
        return str(v) if not isinstance(v, torch.Size) else list(v)
    if isinstance(v, torch.Tensor):
        return _tensor_summary(v)
    if isinstance(v, torch.nn.Module):
        return {"type": type(v).__name__, "module": type(v).__module__,
                "num_parameters": sum(p.numel() for p in v.parameters())}
    if isinstance(v, Path):
        return str(v)
    if depth >= _MAX_DEPTH:
        return {"type": type(v).__name__, "truncated": "depth"}
    oid = id(v)
    if oid in seen:
        return {"type": type(v).__name__, "cycle": True}
    seen = seen | {oid}
    if isinstance(v, Mapping):
        items = list(v.items())
        out = {str(k): _ser(x, seen, depth + 1) for k, x in items[:_MAX_ITEMS]}
        if len(items) > _MAX_ITEMS:
            out["__truncated__"] = len(items) - _MAX_ITEMS
        return out
    if isinstance(v, (list, tuple, set, frozenset)):
        seq = sorted(v, key=repr) if isinstance(v, (set, frozenset)) else list(v)
        out = [_ser(x, seen, depth + 1) for x in seq[:_MAX_ITEMS]]
        if len(seq) > _MAX_ITEMS:
            out.append({"truncated": len(seq) - _MAX_ITEMS})
        return out
    if hasattr(v, "model_dump") and callable(v.model_dump):  # pydantic
        try:
            return _ser(v.model_dump(), seen, depth + 1)
        except Exception:  # noqa: BLE001 - degrade to repr below
            pass
    if dataclasses.is_dataclass(v) and not isinstance(v, type):
        return {"type": type(v).__name__,
                **{f.name: _ser(getattr(v, f.name), seen, depth + 1) for f in dataclasses.fields(v)}}
    if callable(v) and not hasattr(v, "__dict__"):
        return {"type": "callable", "repr": getattr(v, "__qualname__", repr(v))}
    if inspect.isfunction(v) or inspect.ismethod(v) or inspect.isclass(v):
        return {"type": "callable", "repr": f"{getattr(v, '__module__', '?')}.{getattr(v, '__qualname__', v)}"}
    if hasattr(v, "__dict__"):
        attrs = {k: x for k, x in vars(v).items() if not k.startswith("_")}
        return {"type": type(v).__name__, **{k: _ser(x, seen, depth + 1) for k, x in list(attrs.items())[:_MAX_ITEMS]}}
    return {"type": type(v).__name__, "repr": repr(v)[:200]}


def serialize_value(value: Any) -> Any:
    try:
        return _ser(value, set(), 0)
    except Exception as e:  # noqa: BLE001 - instrumentation never raises into the caller
        return {"type": type(value).__name__, "error": str(e)}


def serialize_args(args: dict[str, Any]) -> dict[str, Any]:
    return {k: serialize_value(v) for k, v in args.items()}


# ----------------------------------------------------------------------------- decorator
def instrumentable(cls):
    """Record ``cls.__init__`` arguments (bound to the signature, defaults applied)."""
    orig = cls.__init__
    try:
        sig = inspect.signature(orig)
    except (TypeError, ValueError):
        sig = None

    @functools.wraps(orig)
    def __init__(self, *args, **kwargs):
        orig(self, *args, **kwargs)
        reg = InstrumentationRegistry.get_instance()
        if not reg.enabled or type(self) is not cls:
            return  # subclasses record themselves if decorated; no double entries
        try:
            if sig is not None:
                b = sig.bind(self, *args, **kwargs)
                b.apply_defaults()
                raw = {k: v for k, v in b.arguments.items() if k != "self"}
            else:
                raw = {"args": list(args), **kwargs}
            reg.register(cls.__name__, f"{cls.__module__}.{cls.__qualname__}", serialize_args(raw))
        except Exception:  # noqa: BLE001
            LOGGER.debug("instrumentation of %s failed", cls.__name__, exc_info=True)

    cls.__init__ = __init__
    cls.__ft_instrumented__ = True
    return cls


# ----------------------------------------------------------------------------- dumper
def capture_host_resources() -> dict[str, int]:
    import psutil

    vm, sw = psutil.virtual_memory(), psutil.swap_memory()
    return {"host_memory_total": int(vm.total), "host_memory_used": int(vm.used),
            "host_memory_available": int(vm.available), "swap_total": int(sw.total),
            "swap_used": int(sw.used), "swap_free": int(sw.free)}


def dump_to_file(output_path: str | Path, *, extra: dict[str, Any] | None = None) -> None:
    from flextensor_b200._version import __version__

    recs = InstrumentationRegistry.get_instance().get_records()
    doc: dict[str, Any] = {
        "timestamp": datetime.now().isoformat(),
        "flextensor_version": __version__,
        "components": [dataclasses.asdict(r) for r in recs],
        "host_memory": capture_host_resources(),
    }
    if extra:
        clash = set(extra) & set(doc)
        if clash:
            raise ValueError(f"extra keys collide with built-in keys: {sorted(clash)}")
        doc.update(extra)
    path = Path(output_path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    try:
        with open(tmp, "w") as f:
            json.dump(doc, f, indent=2, default=serialize_value)
        os.replace(tmp, path)
    except BaseException:
        tmp.unlink(missing_ok=True)
        raise
    LOGGER.info("instrumentation: %d components -> %s", len(recs), path)


def dump_to_directory(output_dir: str | Path, *, extra: dict[str, Any] | None = None) -> Path:
    stamp = datetime.now().strftime("%Y%m%d_%H%M%S")
    path = Path(output_dir) / stamp / f"components.{stamp}_pid{os.getpid()}.json"
    dump_to_file(path, extra=extra)
    return path
