"""Generic walk over every tensor a model can reach, with in-place replacement.

Parity with ``src/flextensor/tensor_processors.py:101-604`` (``TypeHandler`` protocol,
``ProcessingContext``, the container / object handlers and ``TensorProcessor``): a model's
tensors are not only its registered parameters and buffers. Modules keep tensors in plain
attributes, in lists / tuples / dicts / sets nested to any depth, inside plain helper objects,
and quantized checkpoints hang tensors (and loader metadata) off a weight as attributes of
the tensor object itself (``weight.weight_scale``, ``weight.weight_loader``). Whatever moves a
model between host and device must reach all of them and keep that metadata.

:class:`TensorVisitor` walks modules (each module once, so shared submodules are not
processed twice; ``torch.compile`` wrappers are unwrapped), dispatching every attribute value
through a handler chain (instance handlers, then global ones, then the built-ins):

* tensors: ``fn(tensor)``; an ``nn.Parameter`` stays an ``nn.Parameter`` (same
  ``requires_grad``); the old tensor's inner fields are carried over to the new one, with
  tensor-valued fields mapped through ``fn`` as well;
* ``list`` / ``tuple`` (namedtuples included) / ``dict`` (``OrderedDict`` kept) / ``set``:
  rebuilt only when an element changed, otherwise the same object is returned (immutable
  mappings and identity-keyed caches survive);
* plain objects with a ``__dict__`` (not modules, types or Python modules): their attributes
  are walked and written back when changed; each object is visited once (cycles are safe).

``update=False`` walks without writing anything back (mapping / discovery passes).
"""

from __future__ import annotations

import collections
import types
from typing import Any, Callable, Protocol

import torch
from torch import nn

_LEAVES = (type(None), bool, int, float, complex, str, bytes, torch.dtype, torch.device)


class TypeHandler(Protocol):
    def can_handle(self, value: Any) -> bool: ...

    def process_attribute(self, value: Any, ctx: "VisitContext") -> Any: ...


def carry_inner_fields(src: torch.Tensor, dst: torch.Tensor, fn: Callable[[torch.Tensor], torch.Tensor] | None = None
                       ) -> None:
    """Copy the instance attributes of tensor ``src`` onto ``dst`` (tensor-valued ones through
    ``fn`` when given). Class attributes and private names are not copied."""
    if src is dst:
        if fn is None:
            return
        for k, v in list(getattr(src, "__dict__", {}).items()):
            if not k.startswith("_") and isinstance(v, torch.Tensor):
                nv = fn(v)
                if nv is not v:
                    setattr(dst, k, nv)
        return
    for k, v in list(getattr(src, "__dict__", {}).items()):
        if k.startswith("_"):
            continue
        if isinstance(v, torch.Tensor) and fn is not None:
            v = fn(v)
        try:
            setattr(dst, k, v)
        except (AttributeError, TypeError):
            pass


class VisitContext:
    """One walk: the handler chain, the tensor map function and the memo of mapped tensors
    (a tensor reachable twice is mapped once and both places get the same result)."""

    def __init__(self, visitor: "TensorVisitor"):
        self.visitor = visitor
        self.handlers = visitor.handlers()
        self._memo: dict[int, torch.Tensor] = {}
        self._keep: list[Any] = []  # keeps memo keys alive for the walk

    def map_tensor(self, t: torch.Tensor) -> torch.Tensor:
        key = id(t)
        if key in self._memo:
            return self._memo[key]
        out = self.visitor.fn(t)
        if out is None:
            out = t
        if out is not t:
            if isinstance(t, nn.Parameter) and not isinstance(out, nn.Parameter):
                out = nn.Parameter(out, requires_grad=t.requires_grad)
            carry_inner_fields(t, out, self.map_tensor)
        elif self.visitor.inner_fields:
            carry_inner_fields(t, t, self.map_tensor)
        self._memo[key] = out
        self._keep.append(t)
        return out

    def dispatch(self, value: Any) -> Any:
        if isinstance(value, _LEAVES):
            return value
        for h in self.handlers:
            if h.can_handle(value):
                return h.process_attribute(value, self)
        return value


class TensorHandler:
    def can_handle(self, value: Any) -> bool:
        return isinstance(value, torch.Tensor)

    def process_attribute(self, value: torch.Tensor, ctx: VisitContext) -> torch.Tensor:
        return ctx.map_tensor(value)


class SequenceHandler:
    """list / tuple / namedtuple, rebuilt only if an element changed."""

    def __init__(self):
        self._active: set[int] = set()

    def can_handle(self, value: Any) -> bool:
        return isinstance(value, (list, tuple))

    def process_attribute(self, value, ctx: VisitContext):
        if id(value) in self._active:
            return value
        self._active.add(id(value))
        try:
            new = [ctx.dispatch(v) for v in value]
        finally:
            self._active.discard(id(value))
        if all(a is b for a, b in zip(new, value)):
            return value
        if isinstance(value, list):
            if ctx.visitor.update:
                value[:] = new  # same list object: other holders of it see the change
                return value
            return new
        if hasattr(value, "_fields"):  # namedtuple
            return type(value)(*new)
        return type(value)(new)


class DictHandler:
    """dict (OrderedDict kept; values only), rebuilt only if a value changed."""

    def __init__(self):
        self._active: set[int] = set()

    def can_handle(self, value: Any) -> bool:
        return isinstance(value, dict)

    def process_attribute(self, value: dict, ctx: VisitContext):
        if id(value) in self._active:
            return value
        self._active.add(id(value))
        try:
            new = {k: ctx.dispatch(v) for k, v in value.items()}
        finally:
            self._active.discard(id(value))
        if all(new[k] is value[k] for k in value):
            return value
        if ctx.visitor.update and type(value) in (dict, collections.OrderedDict):
            for k, v in new.items():
                value[k] = v
            return value
        out = collections.OrderedDict() if isinstance(value, collections.OrderedDict) else {}
        out.update(new)
        return out


class SetHandler:
    def can_handle(self, value: Any) -> bool:
        return isinstance(value, (set, frozenset)) and len(value) > 0

    def process_attribute(self, value, ctx: VisitContext):
        pairs = [(v, ctx.dispatch(v)) for v in value]
        if all(n is o for o, n in pairs):
            return value
        return type(value)(n for _, n in pairs)


class ObjectHandler:
    """Plain objects holding tensors (helper caches, config objects); walked once each."""

    def __init__(self):
        self._seen: set[int] = set()

    def can_handle(self, value: Any) -> bool:
        return (not isinstance(value, (type, types.ModuleType, types.FunctionType, types.MethodType,
                                       torch.Tensor, nn.Module))
                and getattr(type(value), "__dictoffset__", 0) != 0 and hasattr(value, "__dict__"))

    def process_attribute(self, value: Any, ctx: VisitContext):
        if id(value) in self._seen:
            return value
        self._seen.add(id(value))
        for k, v in list(vars(value).items()):
            nv = ctx.dispatch(v)
            if nv is not v and ctx.visitor.update:
                try:
                    setattr(value, k, nv)
                except (AttributeError, TypeError):
                    pass
        return value


def unwrap_compiled(module: nn.Module) -> nn.Module:
    """The real module behind ``torch.compile`` wrappers (``OptimizedModule._orig_mod``):
    writing the wrapper's empty ``_parameters`` back would wipe the wrapped module's."""
    seen = set()
    while type(module).__name__ == "OptimizedModule":
        if id(module) in seen:
            raise RuntimeError("cycle of torch.compile wrappers")
        seen.add(id(module))
        inner = getattr(module, "_modules", {}).get("_orig_mod")
        if inner is None:
            raise RuntimeError("torch.compile wrapper without _orig_mod: refusing to process it")
        module = inner
    return module


class TensorVisitor:
    """Map every reachable tensor of a model through ``fn`` (identity when ``fn`` returns the
    same tensor or None).

    ``params`` / ``buffers``: whether registered parameters / buffers are visited (they are
    mapped with ``.data`` replacement so the Parameter object, its identity and its inner
    fields stay); ``attributes``: plain module attributes and everything nested below them;
    ``inner_fields``: tensor-valued attributes of tensors; ``recursive``: descend into child
    modules."""

    _global_handlers: list[TypeHandler] = []

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor | None], *, params: bool = False,
                 buffers: bool = False, attributes: bool = True, inner_fields: bool = True, recursive: bool = True,
                 update: bool = True, handlers: list[TypeHandler] | None = None):
        self.fn = fn
        self.params, self.buffers, self.attributes = params, buffers, attributes
        self.inner_fields, self.recursive, self.update = inner_fields, recursive, update
        self._handlers = list(handlers or [])

    @classmethod
    def register_global_handler(cls, handler: TypeHandler) -> None:
        cls._global_handlers.insert(0, handler)

    @classmethod
    def clear_global_handlers(cls) -> None:
        cls._global_handlers.clear()

    def register_handler(self, handler: TypeHandler) -> None:
        self._handlers.insert(0, handler)

    def handlers(self) -> list[TypeHandler]:
        return [*self._handlers, *self._global_handlers, TensorHandler(), SequenceHandler(), DictHandler(),
                SetHandler(), ObjectHandler()]

    def apply(self, model: Any) -> Any:
        ctx = VisitContext(self)
        if isinstance(model, nn.Module):
            seen: set[int] = set()
            self._module(unwrap_compiled(model), ctx, seen)
            return model
        return ctx.dispatch(model)

    def _module(self, m: nn.Module, ctx: VisitContext, seen: set[int]) -> None:
        if id(m) in seen:
            return
        seen.add(id(m))
        if self.params:
            for k, p in list(m._parameters.items()):
                if p is not None:
                    self._registered(p, ctx)
        if self.buffers:
            for k, b in list(m._buffers.items()):
                if b is not None:
                    nb = ctx.map_tensor(b)
                    if nb is not b and self.update:
                        m._buffers[k] = nb
        if self.attributes:
            for k, v in list(vars(m).items()):
                if k.startswith("_") or isinstance(v, nn.Module):
                    continue
                nv = ctx.dispatch(v)
                if nv is not v and self.update:
                    setattr(m, k, nv)
        if self.recursive:
            for _, child in m.named_children():
                self._module(unwrap_compiled(child), ctx, seen)

    def _registered(self, p: nn.Parameter, ctx: VisitContext) -> None:
        """Parameters keep their object: the mapped tensor becomes ``p.data``."""
        if id(p) in ctx._memo:
            return
        out = self.fn(p)
        if out is not None and out is not p and self.update:
            with torch.no_grad():
                p.data = out.data if isinstance(out, nn.Parameter) else out
        ctx._memo[id(p)] = p
        ctx._keep.append(p)
        if self.inner_fields:
            carry_inner_fields(p, p, ctx.map_tensor)


def iter_tensors(model: Any, *, params: bool = True, buffers: bool = True, attributes: bool = True
                 ) -> list[torch.Tensor]:
    """Every distinct tensor reachable from ``model`` (read-only walk)."""
    found: dict[int, torch.Tensor] = {}

    def rec(t):
        found.setdefault(id(t), t)
        return t

    TensorVisitor(rec, params=params, buffers=buffers, attributes=attributes, update=False).apply(model)
    return list(found.values())
