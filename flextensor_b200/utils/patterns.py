"""Dot-path and class-name glob matching used to select offload units.

Semantics follow the reference's pattern contract (``src/flextensor/utils.py:162-380``,
``src/flextensor/config.py:303-375``):

* A pattern is split on ``.`` into segments; inside a segment ``*`` and ``?``
  are shell-style wildcards that never cross a dot.
* A segment that is exactly ``*`` matches one or more whole path segments when
  ``recursive_star`` is true (parameter filtering, excludes) and exactly one
  segment otherwise (module selection).
* ``class:<glob>`` patterns match either the short class name or the fully
  qualified ``module.qualname``; the glob is one segment, so ``*`` spans dots.
* ``name:<glob>`` is the explicit form of a bare ``<glob>``.

The implementation compiles every pattern once into a tuple of segment
matchers and runs a memoised segment walk, so matching a model with tens of
thousands of parameters against a handful of patterns stays linear.
"""

from __future__ import annotations

import fnmatch
import functools
import re
from collections.abc import Iterable, Iterator, Mapping
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any

CLASS_PATTERN_PREFIX = "class:"
NAME_PATTERN_PREFIX = "name:"

_STAR = object()  # sentinel: a whole segment that is exactly "*"


@functools.lru_cache(maxsize=4096)
def _segment_regex(segment: str) -> re.Pattern[str]:
    out = []
    for ch in segment:
        if ch == "*":
            out.append(".*")
        elif ch == "?":
            out.append(".")
        else:
            out.append(re.escape(ch))
    return re.compile("".join(out), re.DOTALL)


@functools.lru_cache(maxsize=4096)
def _compile(pattern: str) -> tuple[Any, ...]:
    return tuple(_STAR if seg == "*" else _segment_regex(seg) for seg in pattern.split("."))


def _walk(parts: tuple[str, ...], compiled: tuple[Any, ...], recursive_star: bool) -> bool:
    @functools.lru_cache(maxsize=None)
    def go(i: int, j: int) -> bool:
        if j == len(compiled):
            return i == len(parts)
        if i == len(parts):
            return False
        seg = compiled[j]
        if seg is _STAR:
            if recursive_star:
                # one or more segments
                return any(go(k, j + 1) for k in range(i + 1, len(parts) + 1))
            return go(i + 1, j + 1)
        return seg.fullmatch(parts[i]) is not None and go(i + 1, j + 1)

    return go(0, 0)


def matches_any_pattern(path: str, patterns: Iterable[str], *, recursive_star: bool = True) -> bool:
    """True when the dot-separated ``path`` matches at least one name pattern."""
    parts = tuple(path.split("."))
    return any(_walk(parts, _compile(p), recursive_star) for p in patterns)


def any_path_matches_pattern(paths: Iterable[str], pattern: str, *, recursive_star: bool = True) -> bool:
    """True when at least one of ``paths`` matches the single ``pattern``."""
    compiled = _compile(pattern)
    return any(_walk(tuple(p.split(".")), compiled, recursive_star) for p in paths)


@dataclass(frozen=True, slots=True)
class PartitionedPatterns:
    """Patterns split by prefix; keys are the raw pattern, values the glob body.

    Unpacks as ``names, classes = partition_patterns(...)`` (body lists).
    """

    name_bodies: Mapping[str, str] = field(default_factory=dict)
    class_bodies: Mapping[str, str] = field(default_factory=dict)

    def __post_init__(self) -> None:
        object.__setattr__(self, "name_bodies", MappingProxyType(dict(self.name_bodies)))
        object.__setattr__(self, "class_bodies", MappingProxyType(dict(self.class_bodies)))

    @property
    def name_patterns(self) -> list[str]:
        return list(self.name_bodies.values())

    @property
    def class_patterns(self) -> list[str]:
        return list(self.class_bodies.values())

    def __iter__(self) -> Iterator[list[str]]:
        yield self.name_patterns
        yield self.class_patterns


def partition_patterns(patterns: Iterable[str]) -> PartitionedPatterns:
    """Split raw patterns into name globs and class globs (prefix removed)."""
    names: dict[str, str] = {}
    classes: dict[str, str] = {}
    for raw in patterns:
        for prefix, sink in ((CLASS_PATTERN_PREFIX, classes), (NAME_PATTERN_PREFIX, names)):
            if raw.startswith(prefix):
                body = raw[len(prefix):]
                if not body.strip():
                    raise ValueError(f"pattern {raw!r} has an empty body; use {prefix}<glob> or remove the entry")
                sink[raw] = body
                break
        else:
            names[raw] = raw
    return PartitionedPatterns(name_bodies=names, class_bodies=classes)


def class_fqcn(cls: type) -> str:
    return f"{cls.__module__}.{cls.__qualname__}"


def matches_any_class_pattern(cls: type, class_patterns: Iterable[str]) -> bool:
    """True when ``cls``'s short name or fully-qualified name matches a class glob."""
    pats = list(class_patterns)
    if not pats:
        return False
    short, fq = cls.__name__, class_fqcn(cls)
    for p in pats:
        rx = _segment_regex(p)
        if rx.fullmatch(short) or rx.fullmatch(fq):
            return True
    return False


def get_module_paths(model: Any) -> list[str]:
    return [p for p, _ in model.named_modules() if p]


def get_class_matched_module_paths(model: Any, class_patterns: list[str]) -> set[str]:
    """Paths (root excluded) of modules whose class matches ``class_patterns``."""
    if not class_patterns:
        return set()
    named = getattr(model, "named_modules", None)
    if not callable(named):
        raise TypeError(f"class: patterns require a model exposing named_modules(); got {type(model).__name__}.")
    return {p for p, m in named() if p and matches_any_class_pattern(type(m), class_patterns)}


def glob_to_fnmatch(pattern: str) -> str:
    """Translate a dot glob into an ``fnmatch`` expression (used for quick prefilters)."""
    return fnmatch.translate(pattern)


def validate_pattern_list(value: Any) -> Any:
    """Normalise and validate an include/exclude list (see ``OffloadConfig``).

    Rejects non-string entries, empty entries or bodies, and ``:`` prefixes
    other than ``class:``/``name:``; strips surrounding whitespace.
    """
    from collections.abc import Sequence

    if not isinstance(value, Sequence) or isinstance(value, (str, bytes)):
        return value
    out: list[str] = []
    for i, entry in enumerate(value):
        if not isinstance(entry, str):
            raise ValueError(f"pattern entries must be strings; got {type(entry).__name__} at index {i}: {entry!r}")
        entry = entry.strip()
        if not entry:
            raise ValueError(f"pattern entry at index {i} is empty or whitespace-only; remove it")
        for prefix in (CLASS_PATTERN_PREFIX, NAME_PATTERN_PREFIX):
            if entry.startswith(prefix):
                body = entry[len(prefix):].strip()
                if not body:
                    raise ValueError(
                        f"pattern {entry!r} at index {i} has an empty body; use {prefix}<glob> or remove the entry"
                    )
                entry = prefix + body
                break
        else:
            if ":" in entry:
                raise ValueError(
                    f"pattern {entry!r} at index {i} contains ':' but doesn't start with "
                    f"{CLASS_PATTERN_PREFIX!r} or {NAME_PATTERN_PREFIX!r}; did you mean {CLASS_PATTERN_PREFIX}<glob>?"
                )
        out.append(entry)
    return out
