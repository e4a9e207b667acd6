"""``OffloadConfig`` and its loaders.

The field set, defaults, validators and the ``FT_*`` environment contract are
part of the public API and are kept identical to the reference
(``src/flextensor/config.py:55-525`` for fields/validators, ``:831-848`` for strict
env validation, ``:900-1059`` for ``load_config*``):

* precedence: config file < ``FT_*`` environment < keyword arguments;
* env-only loading defaults ``enabled=False``;
* unknown ``FT_*`` variables raise, with a did-you-mean hint;
* files may be INI (``[flextensor]`` section), JSON or YAML.
"""

from __future__ import annotations

import configparser
import difflib
import json
import logging
import os
import sys
import types
from collections.abc import Mapping
from pathlib import Path
from typing import Annotated, Any, Literal, Self, Union, get_args, get_origin

import yaml
from pydantic import BaseModel, Field, WithJsonSchema, field_validator, model_validator

from flextensor_b200.planner.protocol import Strategy
from flextensor_b200.utils.patterns import validate_pattern_list

logger = logging.getLogger(__name__)

PinnedMemoryMode = Literal["torch", "host_register"]
ProfileMode = Literal["torch_function", "getter", "view"]
OffloadTimingMode = Literal["off", "eager", "cuda_graph"]
PiecewisePrefetchMode = Literal["off", "warn", "error"]
BLOCK_TRANSFER_MODES = frozenset({"allocation_block_transfer", "raw_block_transfer"})
OFFLOAD_TRANSFER_MODES = frozenset({"strategy", *BLOCK_TRANSFER_MODES})

_REGISTERED_ENV_VARS: set[str] = set()

# Removed fields: name -> (version removed, migration hint).
_REMOVED_FIELDS: dict[str, tuple[str, str]] = {
    "release_tensors": ("v0.2.0", "GPU tensors are now always released after layer execution."),
    "enable_direct_mode": ("v0.2.0", "Direct mode is now always enabled."),
    "enable_tracing": ("v0.2.0", "Use TensorManager(_use_trace_tensor=True) for tracing."),
    "rearrange_transfers": ("v0.2.0", "Transfer rearrangement is now auto-enabled when gap layers are detected."),
    "compute_transfer_gap": ("v0.2.0", "Use TensorManager(_compute_transfer_gap=N) to override."),
    "enable_untraced_tensor_discovery": (
        "v0.2.0",
        "Untraced tensor discovery is now always enabled. "
        "Use TensorManager(_enable_untraced_tensor_discovery=False) to override.",
    ),
    "enable_module_tracker": ("v0.2.0", "ModuleTracker is now always enabled for manual traps."),
    "warmup_iters": ("v0.4.0", "Use discovery_iters instead."),
    "profile_iters": ("v0.4.0", "Use profiling_iters instead."),
}


class OffloadConfig(BaseModel):
    """Configuration of one offload manager (28 fields, reference-compatible)."""

    enabled: bool = Field(default=True)
    """Enable offloading; ``False`` preloads the whole model to the device."""
    gpu_device: int = Field(default=0, ge=0)
    """CUDA device index."""
    pinned_memory: bool = Field(default=True)
    """Keep host copies page-locked so H2D copies are asynchronous."""
    pinned_memory_mode: PinnedMemoryMode = Field(default="torch")
    """``torch``: copy into a fresh pinned allocation; ``host_register``: cudaHostRegister in place."""
    shm_enabled: bool = Field(default=False)
    """Store offloaded weights in POSIX shared memory shared by local workers."""
    shm_namespace: str | None = Field(default=None)
    """Base name of the shared-memory segments (required with ``shm_enabled``)."""
    shm_wait_timeout: float = Field(default=0.0, ge=0.0)
    """Follower wait bound in seconds (0 = only creator-heartbeat liveness)."""
    discovery_iters: int = Field(default=1, ge=0)
    """Forwards spent discovering which tensors each trap uses."""
    skip_discovery: bool = Field(default=False)
    """Derive trap->tensor maps statically from patched modules instead of running discovery."""
    profiling_iters: int = Field(default=10, ge=0)
    """Forwards spent timing each trap before planning."""
    external_compile: bool = Field(default=False)
    """Arm the custom-op loader path so the caller can torch.compile units after INFERENCE."""
    transfer_budget_scale: float = Field(default=1.0, gt=0.0)
    """Multiplier on each trap's transfer time budget (<1 adds safety margin)."""
    transfer_mode: str = Field(default="allocation_block_transfer")
    """``allocation_block_transfer`` | ``raw_block_transfer`` | ``strategy``."""
    num_blocks: int = Field(default=4, ge=2)
    """Maximum number of GPU ring slots."""
    min_blocks: int = Field(default=4, ge=2)
    """Minimum number of ring slots tried by the assignment search."""
    max_gpu_mem_fraction: float | None = Field(default=None, gt=0.0, le=1.0)
    """Memory mode: cap weights+slots to this fraction of device memory. ``None`` = latency mode."""
    profile_storage_dir: str | None = Field(default=None)
    """Directory for ``profile.json`` persistence."""
    profile_read_only: bool = Field(default=False)
    """Only load profiles; never write them."""
    load_strategy: Annotated[Strategy, WithJsonSchema({"type": "object"})] | None = Field(default=None)
    """Explicit planner; ``None`` selects ``AdaptiveStrategy``."""
    enable_instrumentation: bool = Field(default=False)
    """Record component constructor arguments and dump them at INFERENCE."""
    instrumentation_output_dir: str = Field(default=".flextensor/instrumentation")
    """Where instrumentation dumps go."""
    offload_timing: OffloadTimingMode = Field(default="off")
    """Per-trap transfer/compute/wait timing during inference (``eager`` or ``cuda_graph`` events)."""
    piecewise_prefetch: PiecewisePrefetchMode = Field(default="warn")
    """What to do when a piecewise graph join puts an outstanding H2D on the critical path."""
    include_patterns: list[str] = Field(default_factory=lambda: ["*"])
    """Modules/parameters to offload (``<glob>``, ``name:<glob>``, ``class:<glob>``)."""
    exclude_patterns: list[str] = Field(default_factory=list)
    """Modules/parameters kept resident; applied after ``include_patterns``."""
    enable_diagnostics: bool = Field(default=False)
    """Log per-trap duration statistics and the block table after planning."""
    profile_mode: ProfileMode = Field(default="view")
    """Profiling mechanism: ``view`` (slot views), ``getter`` (property getters) or ``torch_function``."""

    # ---- fields beyond the reference schema
    hold_device_weights: bool = Field(default=True)
    """Unit weights that already sit on the compute device stay there through discovery and
    profiling and are packed device -> pinned arena once the plan exists (no per-tensor host copy).
    ``False`` moves them to pinned host memory at warm-up, which frees device memory for the
    profiling passes."""

    model_config = {"arbitrary_types_allowed": True, "use_attribute_docstrings": True}

    @field_validator("include_patterns", "exclude_patterns", mode="before")
    @classmethod
    def _validate_pattern_entries(cls, v: Any) -> Any:
        return validate_pattern_list(v)

    @model_validator(mode="before")
    @classmethod
    def _reject_removed_fields(cls, data: Any) -> Any:
        if isinstance(data, dict):
            for name, (version, msg) in _REMOVED_FIELDS.items():
                if name in data:
                    raise ValueError(
                        f"'{name}' was removed in {version}. {msg} Remove '{name}' from your OffloadConfig() call."
                    )
        return data

    @model_validator(mode="after")
    def _validate_block_range(self) -> Self:
        if self.num_blocks < self.min_blocks:
            raise ValueError(f"num_blocks ({self.num_blocks}) must be >= min_blocks ({self.min_blocks})")
        return self

    @model_validator(mode="after")
    def _validate_shm_namespace(self) -> Self:
        if self.shm_enabled and sys.platform == "win32":
            raise ValueError("Shared memory (SHM) is not supported on Windows")
        if self.shm_enabled and (self.shm_namespace is None or not self.shm_namespace.strip()):
            raise ValueError("shm_namespace must be non-empty when shm_enabled=True")
        return self

    @model_validator(mode="after")
    def _validate_profile_mode(self) -> Self:
        if self.transfer_mode not in OFFLOAD_TRANSFER_MODES:
            raise ValueError(
                f"transfer_mode={self.transfer_mode!r} is not one of {sorted(OFFLOAD_TRANSFER_MODES)}"
            )
        if self.profile_mode == "torch_function" and self.transfer_mode in BLOCK_TRANSFER_MODES:
            raise ValueError(
                f"profile_mode='torch_function' is incompatible with transfer_mode={self.transfer_mode!r}. "
                "Use profile_mode='getter' or 'view', or set transfer_mode='strategy'."
            )
        if self.external_compile and self.transfer_mode not in BLOCK_TRANSFER_MODES:
            raise ValueError(
                "external_compile=True requires a block transfer_mode (allocation_block_transfer or "
                f"raw_block_transfer); got transfer_mode={self.transfer_mode!r}."
            )
        if self.offload_timing != "off" and self.transfer_mode not in BLOCK_TRANSFER_MODES:
            raise ValueError(
                f"offload_timing={self.offload_timing!r} requires a block transfer_mode "
                f"(allocation_block_transfer or raw_block_transfer); got transfer_mode={self.transfer_mode!r}."
            )
        return self

    def model_copy(self, *, update: Mapping[str, Any] | None = None, deep: bool = False) -> Self:
        """Validated copy that keeps explicit-field tracking."""
        if not update:
            return super().model_copy(deep=deep)
        upd = self._reject_removed_fields(dict(update))  # type: ignore[operator]
        copied = super().model_copy(update=upd, deep=deep)
        out = type(self).model_validate(dict(copied))
        object.__setattr__(out, "__pydantic_fields_set__", set(copied.model_fields_set))
        return out


def resolve_load_strategy(config: OffloadConfig) -> Strategy:
    """The explicit ``load_strategy`` or a fresh ``AdaptiveStrategy`` built from the config."""
    if config.load_strategy is not None:
        return config.load_strategy
    from flextensor_b200.planner.adaptive import AdaptiveStrategy

    return AdaptiveStrategy(
        scale=config.transfer_budget_scale,
        loader_type=config.transfer_mode,
        n_blocks=config.num_blocks,
        min_blocks=config.min_blocks,
    )


def config_field_was_set(config: Any, field_name: str) -> bool:
    fs = getattr(config, "model_fields_set", None)
    return isinstance(fs, (set, frozenset)) and field_name in fs


# --------------------------------------------------------------------------- env / file loading


def _scalar_kind(annotation: object) -> type:
    """Map a field annotation onto the coercion kind used for env/INI strings."""
    if annotation is None:
        return str
    origin = get_origin(annotation)
    if origin is Union or origin is types.UnionType:
        arms = [a for a in get_args(annotation) if a is not type(None)]
        if not arms:
            return str
        first = arms[0]
        if get_origin(first) is Union:
            return object
        if get_origin(first) is list:
            return list
        if isinstance(first, type) and first in (bool, int, float, str):
            return first
        return object
    if origin is list:
        return list
    if origin is Literal:
        members = get_args(annotation)
        t = type(members[0]) if members else str
        return t if t in (bool, int, float, str) else str
    if isinstance(annotation, type) and annotation in (bool, int, float, str):
        return annotation
    return object


def _field_kinds() -> dict[str, type]:
    return {name: _scalar_kind(f.annotation) for name, f in OffloadConfig.model_fields.items()}


_TRUE = {"true", "1", "yes", "y", "on"}
_FALSE = {"false", "0", "no", "n", "off"}


def _coerce(value: str, kind: type) -> Any:
    low = value.lower()
    if low in ("none", "null") or value == "":
        return None
    if kind is bool:
        if low in _TRUE:
            return True
        if low in _FALSE:
            return False
        raise ValueError(f"Cannot parse '{value}' as boolean")
    if kind is int:
        return int(value)
    if kind is float:
        return float(value)
    return value


def _split_list(value: str) -> list[str]:
    return [p.strip() for p in value.split(",") if p.strip()]


def _load_ini(path: Path, kinds: dict[str, type]) -> dict[str, Any]:
    parser = configparser.ConfigParser()
    parser.read(path)
    if "flextensor" not in parser:
        raise ValueError("INI file must contain [flextensor] section")
    sec = parser["flextensor"]
    out: dict[str, Any] = {}
    for name, kind in kinds.items():
        if name not in sec or kind is object:
            continue
        out[name] = _split_list(sec[name]) if kind is list else _coerce(sec[name], kind)
    for name in _REMOVED_FIELDS:
        if name in sec:
            out[name] = sec[name]
    return out


def _from_mapping(data: dict[str, Any], kinds: dict[str, type]) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for name, value in data.items():
        if name in _REMOVED_FIELDS:
            out[name] = value
            continue
        kind = kinds.get(name)
        if kind is None or kind is object:
            continue
        if kind is not list and isinstance(value, str) and kind is not str:
            out[name] = _coerce(value, kind)
        else:
            out[name] = value
    return out


def _load_file(path: Path, kinds: dict[str, type]) -> dict[str, Any]:
    suffix = path.suffix.lower()
    if suffix in (".conf", ".ini"):
        return _load_ini(path, kinds)
    if suffix == ".json":
        with path.open() as f:
            return _from_mapping(json.load(f), kinds)
    if suffix in (".yaml", ".yml"):
        with path.open() as f:
            data = yaml.safe_load(f)
        return {} if data is None else _from_mapping(data, kinds)
    raise ValueError(f"Unsupported config file format: {suffix}. Use .conf, .ini, .json, .yaml, or .yml")


def _register_env_var(name: str) -> None:
    """Declare an extra ``FT_*`` variable (integration flags) so strict env validation accepts it."""
    _REGISTERED_ENV_VARS.add(name)


def _known_env(prefix: str, kinds: dict[str, type], config_file_env_var: str) -> set[str]:
    known = {f"{prefix}{n.upper()}" for n in kinds}
    known |= {f"{prefix}{n.upper()}" for n in _REMOVED_FIELDS}
    known.add(f"{prefix}CONFIG_FILE")
    if config_file_env_var and config_file_env_var.startswith(prefix):
        known.add(config_file_env_var)
    known |= {n for n in _REGISTERED_ENV_VARS if n.startswith(prefix)}
    return known


def _validate_env(prefix: str, kinds: dict[str, type], config_file_env_var: str) -> None:
    if not prefix:
        return
    known = _known_env(prefix, kinds, config_file_env_var)
    errors = []
    for name in sorted(n for n in os.environ if n.startswith(prefix) and n not in known):
        msg = f"Unrecognized environment variable with {prefix} prefix: {name}"
        hint = difflib.get_close_matches(name, sorted(known), n=1, cutoff=0.75)
        if hint:
            msg += f". Did you mean: {hint[0]}?"
        errors.append(msg)
    if errors:
        raise ValueError("\n".join(errors))


def _load_env(prefix: str, kinds: dict[str, type], config_file_env_var: str) -> dict[str, Any]:
    _validate_env(prefix, kinds, config_file_env_var)
    for name, (version, msg) in _REMOVED_FIELDS.items():
        var = f"{prefix}{name.upper()}"
        if os.environ.get(var) is not None:
            logger.warning("Environment variable '%s' is ignored: '%s' was removed in %s. %s", var, name, version, msg)
    out: dict[str, Any] = {}
    for name, kind in kinds.items():
        if kind is object:
            continue
        var = f"{prefix}{name.upper()}"
        raw = os.environ.get(var)
        if raw is None:
            continue
        try:
            out[name] = _split_list(raw) if kind is list else _coerce(raw, kind)
        except (ValueError, TypeError) as exc:
            raise ValueError(f"Failed to convert {var}={raw}: {exc}") from exc
    return out


def load_config(
    config_path: str | Path | None = None,
    env_prefix: str = "FT_",
    use_env: bool = True,
    config_file_env_var: str = "FT_CONFIG_FILE",
    **kwargs: Any,
) -> OffloadConfig:
    """Build an ``OffloadConfig`` from file < env < kwargs (env-only defaults ``enabled=False``)."""
    kinds = _field_kinds()
    data: dict[str, Any] = {}
    path_str = config_path or (os.environ.get(config_file_env_var) if config_file_env_var else None)
    if path_str is not None:
        path = Path(path_str)
        if not path.exists():
            raise FileNotFoundError(f"Config file not found: {path}")
        data = _load_file(path, kinds)
    elif use_env:
        data["enabled"] = False
    if use_env:
        data.update(_load_env(env_prefix, kinds, config_file_env_var))
    data.update(kwargs)
    return OffloadConfig(**data)


def load_config_from_file(
    config_path: str | Path | None = None,
    env_var: str = "FT_CONFIG_FILE",
    **kwargs: Any,
) -> OffloadConfig:
    """Load from a config file only (no environment overrides)."""
    if config_path is None and os.environ.get(env_var) is None:
        raise FileNotFoundError(f"No config file specified. Provide config_path or set {env_var} environment variable.")
    return load_config(config_path=config_path, use_env=False, config_file_env_var=env_var, **kwargs)


def load_config_from_env(prefix: str = "FT_", **kwargs: Any) -> OffloadConfig:
    """Load from ``{prefix}{FIELD}`` environment variables only (``enabled`` defaults to False)."""
    return load_config(config_path=None, env_prefix=prefix, use_env=True, config_file_env_var="", **kwargs)
