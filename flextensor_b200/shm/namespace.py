"""SHM namespace scheme (names are an interop contract; ``src/flextensor/shm/namespace.py:17-133``).

``ft_<sha256[:8]>`` over model path + patterns + budget + manager name;
rank suffix ``_tp{t}_pp{p}[_ep{e}]``; blocks ``{ns}_w{i}``, ``{ns}_prof``,
``{ns}_crd``, tensor store ``{ns}_t``.
"""

from __future__ import annotations

import hashlib
import json
import pathlib
from typing import Any

SHM_PROTOCOL_VERSION: int = 4
DEFAULT_MANAGER_NAME = "default"


def compute_shm_namespace(model_path: str, config, extra_keys: dict[str, Any] | None = None,
                          manager_name: str = DEFAULT_MANAGER_NAME) -> str:
    if config.shm_namespace is not None:
        return config.shm_namespace
    budget = None
    if config.max_gpu_mem_fraction is not None:
        budget = f"fraction:{config.max_gpu_mem_fraction}"
    h: dict[str, Any] = {
        "model_path": str(pathlib.Path(model_path).resolve()),
        "include_patterns": sorted(config.include_patterns),
        "exclude_patterns": sorted(config.exclude_patterns),
        "max_gpu_mem_bytes": budget,
        "manager_name": manager_name,
    }
    if config.load_strategy is not None:
        h["strategy"] = type(config.load_strategy).__name__
    if extra_keys:
        h["extra"] = {k: str(v) for k, v in sorted(extra_keys.items())}
    canon = json.dumps(h, sort_keys=True, separators=(",", ":"))
    return "ft_" + hashlib.sha256(canon.encode()).hexdigest()[:8]


def apply_rank_suffix(base_namespace: str, tp_rank: int, pp_rank: int, ep_rank: int | None = None) -> str:
    s = f"{base_namespace}_tp{tp_rank}_pp{pp_rank}"
    return s if ep_rank is None else f"{s}_ep{ep_rank}"


def weight_block_name(namespace: str, block_index: int) -> str:
    return f"{namespace}_w{block_index}"


def profile_block_name(namespace: str) -> str:
    return f"{namespace}_prof"


def coord_block_name(namespace: str) -> str:
    return f"{namespace}_crd"


def tensor_store_name(namespace: str) -> str:
    return f"{namespace}_t"


def heartbeat_block_name(namespace: str) -> str:
    return f"{namespace}_hb"


def session_namespace(base: str, name: str) -> str:
    """Per-manager namespace inside a ``SharedOffloadSession``: ``ft_<sha256(base\\0name)[:12]>``."""
    return "ft_" + hashlib.sha256(f"{base}\0{name}".encode()).hexdigest()[:12]
