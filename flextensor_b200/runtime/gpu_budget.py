"""GPU memory budget for memory-mode planning (``src/flextensor/gpu_budget.py:38-230``).

budget = total_device_bytes x fraction, capped by what the process can still
obtain (free + cached-but-unused), floored at 256 MiB, minus bytes the planner
cannot see (resident non-unit parameters and buffers already on the device).
"""

from __future__ import annotations

import torch

MIN_BUDGET = 256 * 1024 * 1024


def available_bytes(device: torch.device) -> tuple[int, int]:
    """(total, obtainable) bytes on ``device``."""
    if device.type != "cuda":
        import psutil

        vm = psutil.virtual_memory()
        return int(vm.total), int(vm.available)
    free, total = torch.cuda.mem_get_info(device)
    cached_unused = torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    return int(total), int(free + max(0, cached_unused))


def resolve_gpu_budget(device: torch.device, fraction: float, strategy_invisible_bytes: int = 0,
                       reclaimable_bytes: int = 0) -> int:
    """``reclaimable_bytes``: unit weights still held on the device that the plan may stream
    (they are freed once packed), so they count as obtainable."""
    if not (0.0 < fraction <= 1.0):
        raise ValueError(f"max_gpu_mem_fraction must be in (0, 1], got {fraction}")
    total, obtainable = available_bytes(torch.device(device))
    budget = min(int(total * fraction), obtainable + int(strategy_invisible_bytes) + int(reclaimable_bytes))
    budget = max(budget, MIN_BUDGET)
    return max(MIN_BUDGET, budget - int(strategy_invisible_bytes))


def reserve_strategy_invisible_gpu_budget(budget: int, invisible: int) -> int:
    return max(MIN_BUDGET, int(budget) - int(invisible))
