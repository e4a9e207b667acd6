"""Placement strategies: which tensors to stream, during which trap, in which slot.

Class names and constructor signatures are the reference's public API
(``src/flextensor/strategy/{simple,knapsack,global_strategy,budget_fill}.py``);
the algorithms are this package's own:

* Per-pair fill (``KnapsackStrategy``/``KnapsackBlockStrategy``): for trap j the
  H2D window is trap j-1's compute time x ``scale``; the bytes that fit
  (via the transfer interpolator) are filled by an exact subset-sum over
  quantised sizes (Python big-int bitsets), so the largest subset of j's
  tensors that still hides behind j-1 is streamed.
* Memory mode (``max_gpu_mem_bytes`` set): the window scale is raised by
  bisection until the plan's peak fits the budget.
* ``GlobalOffloadStrategy``: gap-aware windows (a trap with nothing to transfer
  lends its compute time to the next transfer) plus a chosen slot-assignment
  policy, with scale bisection in memory mode.
* ``GlobalTensorSelectionStrategy``/``BudgetFill*DE``: scipy differential
  evolution over per-tensor (or per-layer fraction) choices, seeded with the
  greedy plan, scored with the shared evaluator.
* ``BudgetFillGreedyStrategy``: memory-first ranked-prefix scan (tensors whose
  transfer fits the window first, then by size) until peak <= budget.
"""

from __future__ import annotations

import logging
import math
import warnings

import numpy as np

from flextensor_b200.core.stats import LayerStatistics, TensorStatistics
from flextensor_b200.planner.blocks import OptimizedRoundRobinAssignment, StrictRoundRobinAssignment
from flextensor_b200.planner.common import (
    MB,
    build_block_data,
    byte_budget,
    eligible,
    estimated_overhead,
    evaluate_strategy_result,
    interpolator_for,
    peak_memory,
    require_layers,
    validate_memory_params,
)
from flextensor_b200.planner.protocol import StrategyComputeError, StrategyResult

logger = logging.getLogger(__name__)

_QUANTA = 4096


def subset_fill(tensors: list[TensorStatistics], capacity: float) -> list[TensorStatistics]:
    """Largest-bytes subset with total <= capacity (exact on a 1/4096-of-capacity grid)."""
    if capacity <= 0 or not tensors:
        return []
    total = sum(t.size_bytes for t in tensors)
    if total <= capacity:
        return list(tensors)
    unit = max(1.0, capacity / _QUANTA)
    cap_q = int(capacity // unit)
    sizes = [max(1, math.ceil(t.size_bytes / unit)) for t in tensors]
    mask = (1 << (cap_q + 1)) - 1
    reach = [1]
    for s in sizes:
        reach.append((reach[-1] | (reach[-1] << s)) & mask)
    best = reach[-1].bit_length() - 1
    chosen: list[TensorStatistics] = []
    cur = best
    for i in range(len(tensors) - 1, -1, -1):
        if not (reach[i] >> cur) & 1:
            chosen.append(tensors[i])
            cur -= sizes[i]
    chosen.reverse()
    return chosen


def _single_windows(layer_stats: list[LayerStatistics], scale: float) -> list[float]:
    return [0.0] + [layer_stats[i - 1].duration * scale for i in range(1, len(layer_stats))]


def _per_pair_plan(
    layer_stats: list[LayerStatistics],
    interp,
    scale: float,
    threshold_mb: float,
    cyclic: bool,
    group_size: int = 1,
) -> dict[str, list[TensorStatistics]]:
    """strategy_map where trap i-1 streams a knapsack-filled subset of trap i's tensors."""
    n = len(layer_stats)
    plan: dict[str, list[TensorStatistics]] = {}
    g = max(1, group_size)
    for j in range(1, n):
        src = layer_stats[j - 1]
        if j % g and g > 1:
            pass
        window = src.duration * scale
        cand = eligible(layer_stats[j].tensors, threshold_mb)
        pick = subset_fill(cand, byte_budget(interp, window, cand))
        if pick:
            plan[src.label] = pick
    if cyclic and n >= 2:
        cand = eligible(layer_stats[0].tensors, threshold_mb)
        pick = subset_fill(cand, byte_budget(interp, layer_stats[-1].duration * scale, cand))
        if pick:
            plan[layer_stats[-1].label] = pick
    return plan


def _gap_plan(layer_stats, interp, scale, threshold_mb, assign_all: bool = False):
    """Gap-aware: traps that stream nothing donate their time to the next transfer."""
    plan: dict[str, list[TensorStatistics]] = {}
    n = len(layer_stats)
    window_start = 0
    window = 0.0
    for j in range(1, n):
        window += layer_stats[j - 1].duration * scale
        cand = eligible(layer_stats[j].tensors, threshold_mb)
        pick = list(cand) if assign_all else subset_fill(cand, byte_budget(interp, window, cand))
        if pick:
            plan[layer_stats[window_start].label] = pick
            window_start = j
            window = 0.0
        else:
            # this trap streams nothing; the pending window keeps growing but the
            # transfer must be issued at the window's first trap
            pass
    return plan


def _bisect_scale(make_plan, layer_stats, budget: int, lo: float, hi: float = 64.0, iters: int = 24):
    """Smallest scale >= lo whose plan fits ``budget`` (plans grow with scale)."""
    best = make_plan(lo)
    if peak_memory(best, layer_stats) <= budget:
        return best
    top = make_plan(hi)
    if peak_memory(top, layer_stats) > budget:
        return top
    a, b = lo, hi
    best = top
    for _ in range(iters):
        mid = math.sqrt(a * b)
        r = make_plan(mid)
        if peak_memory(r, layer_stats) <= budget:
            best, b = r, mid
        else:
            a = mid
    return best


# --------------------------------------------------------------------------- simple


class GreedyStrategy:
    """Offload each trap's tensors while cumulative compute time covers their transfer."""

    def __init__(self, threshold_mb: float = 0.1, n_blocks: int = 4, scale: float = 1.0):
        validate_memory_params(scale)
        self.threshold_mb, self.n_blocks, self.scale = threshold_mb, n_blocks, scale

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        if not layer_stats:
            return StrategyResult(strategy_map={}, block_data=None)
        interp = interpolator_for(layer_stats, memory_stats)
        plan: dict[str, list[TensorStatistics]] = {}
        credit = 0.0
        for j in range(1, len(layer_stats)):
            credit += layer_stats[j - 1].duration * self.scale
            cand = sorted(eligible(layer_stats[j].tensors, self.threshold_mb), key=lambda t: -t.size_bytes)
            take = []
            for t in cand:
                cost = interp.bytes_to_duration(t.size_bytes) if interp else t.load_time_ms
                if cost <= credit:
                    take.append(t)
                    credit -= cost
            if take:
                plan[layer_stats[j - 1].label] = take
            credit = min(credit, layer_stats[j - 1].duration * self.scale)
        return StrategyResult(plan, build_block_data(plan, layer_stats, self.n_blocks))


class NthLayerStrategy:
    """Stream every ``nth_layer``-th trap entirely (during the trap before it)."""

    def __init__(self, nth_layer: int, threshold_mb: float = 0.1, n_blocks: int = 4, cyclic: bool = False):
        if nth_layer < 1:
            raise ValueError("nth_layer must be >= 1")
        self.nth_layer, self.threshold_mb, self.n_blocks = nth_layer, threshold_mb, n_blocks
        self.cyclic = cyclic

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        if not layer_stats:
            return StrategyResult(strategy_map={}, block_data=None)
        plan = {}
        for j in range(1, len(layer_stats)):
            if j % self.nth_layer == 0:
                cand = eligible(layer_stats[j].tensors, self.threshold_mb)
                if cand:
                    plan[layer_stats[j - 1].label] = cand
        if self.cyclic and len(layer_stats) >= 2:
            # trap 0 streams during the previous forward's last trap (wrap-around)
            cand = eligible(layer_stats[0].tensors, self.threshold_mb)
            if cand:
                plan[layer_stats[-1].label] = cand
        return StrategyResult(plan, build_block_data(plan, layer_stats, self.n_blocks))


# --------------------------------------------------------------------------- knapsack family


class KnapsackStrategy:
    """Per-pair subset-sum fill for the per-tensor (non-block) loader; cyclic by default.
    ``n_blocks`` is accepted for the reference's signature: the per-tensor loader has no ring."""

    def __init__(self, scale: float = 1.0, cyclic: bool = True, group_size: int = 1, threshold_mb: float = 0.1,
                 n_blocks: int = 4):
        validate_memory_params(scale)
        self.scale, self.cyclic, self.group_size = scale, cyclic, group_size
        self.threshold_mb, self.n_blocks = threshold_mb, n_blocks

    def _plan(self, layer_stats, interp, scale):
        return _per_pair_plan(layer_stats, interp, scale, self.threshold_mb, self.cyclic, self.group_size)

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        if len(layer_stats) < 2:
            return StrategyResult(strategy_map={}, block_data=None)
        interp = interpolator_for(layer_stats, memory_stats)
        if max_gpu_mem_bytes is None:
            return StrategyResult(self._plan(layer_stats, interp, self.scale), None)
        return _bisect_scale(lambda s: StrategyResult(self._plan(layer_stats, interp, s), None),
                             layer_stats, max_gpu_mem_bytes, self.scale)


class KnapsackBlockStrategy:
    """Per-pair subset-sum fill with GPU ring slots (block loaders)."""

    def __init__(self, scale: float = 1.0, group_size: int = 1, threshold_mb: float = 0.1, n_blocks: int = 4):
        validate_memory_params(scale)
        self.scale, self.group_size, self.threshold_mb, self.n_blocks = scale, group_size, threshold_mb, n_blocks

    def _result(self, layer_stats, interp, scale) -> StrategyResult:
        plan = _per_pair_plan(layer_stats, interp, scale, self.threshold_mb, False, self.group_size)
        return StrategyResult(plan, build_block_data(plan, layer_stats, self.n_blocks))

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        require_layers(layer_stats)
        interp = interpolator_for(layer_stats, memory_stats)
        if interp is None:
            raise StrategyComputeError("KnapsackBlock needs memory transfer statistics")
        if max_gpu_mem_bytes is None:
            return self._result(layer_stats, interp, self.scale)
        return _bisect_scale(lambda s: self._result(layer_stats, interp, s), layer_stats, max_gpu_mem_bytes,
                             self.scale)


class AdaptiveKnapsackStrategy:
    """Knapsack planner picking block or per-tensor form from ``loader_type``."""

    def __init__(self, scale: float = 1.0, loader_type: str = "strategy", cyclic: bool = True, group_size: int = 1,
                 threshold_mb: float = 0.1):
        self.loader_type = loader_type
        if loader_type == "strategy":
            self._inner = KnapsackStrategy(scale=scale, cyclic=cyclic, group_size=group_size,
                                           threshold_mb=threshold_mb)
        else:
            self._inner = KnapsackBlockStrategy(scale=scale, group_size=group_size, threshold_mb=threshold_mb)

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        return self._inner.compute(layer_stats, memory_stats, max_gpu_mem_bytes)


# --------------------------------------------------------------------------- global family


class GlobalOffloadStrategy:
    """Gap-aware windows + slot-assignment policy; scale bisection in memory mode."""

    def __init__(self, n_blocks: int = 4, scale: float = 1.0, threshold_mb: float = 0.1,
                 min_blocks: int | None = None, max_blocks: int | None = None, assignment_strategy=None):
        validate_memory_params(scale)
        self.n_blocks, self.scale, self.threshold_mb = n_blocks, scale, threshold_mb
        self.assignment = assignment_strategy or OptimizedRoundRobinAssignment(
            min_blocks=min_blocks or 2, max_blocks=max_blocks or n_blocks)

    def _result(self, layer_stats, interp, scale):
        plan = _gap_plan(layer_stats, interp, scale, self.threshold_mb)
        return StrategyResult(plan, build_block_data(plan, layer_stats, self.n_blocks, self.assignment))

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        require_layers(layer_stats)
        interp = interpolator_for(layer_stats, memory_stats)
        if interp is None:
            raise StrategyComputeError("GlobalOffload needs memory transfer statistics")
        if max_gpu_mem_bytes is None:
            return self._result(layer_stats, interp, self.scale)
        return _bisect_scale(lambda s: self._result(layer_stats, interp, s), layer_stats, max_gpu_mem_bytes,
                             self.scale)


def _de_select(cands: list[tuple[str, TensorStatistics]], layer_stats, interp, n_blocks, assignment, budget,
               seed_mask: np.ndarray | list[np.ndarray] | None, pop_size: int, epoch: int, max_early_stop: int,
               seed: int | None, memory_first: bool, optimizer: str = "DE", seed_ratio: float = 0.0):
    """Search over per-candidate offload binaries (x_i > 0.5 streams candidate i); returns the best
    StrategyResult found, never worse (by the same cost) than the first seed plan.

    ``optimizer``: ``DE`` -- differential evolution over a population whose first
    ``max(1, seed_ratio * pop)`` members start from the seed plans (``seed_mask``: one mask or a
    list of them, e.g. knapsack plans at several scales); ``SA`` (alias ``DA``) -- dual annealing
    (generalised simulated annealing, local search off: the cost is piecewise constant) started
    from the first seed plan. Both stop after ``epoch`` iterations, or once ``max_early_stop``
    iterations (DE generations; SA minima reported) brought no improvement."""
    from scipy.optimize import differential_evolution, dual_annealing

    if not cands:
        return StrategyResult({}, build_block_data({}, layer_stats, n_blocks, assignment))
    total_model = sum(t.size_bytes for l in layer_stats for t in l.tensors) or 1
    masks = [] if seed_mask is None else ([seed_mask] if isinstance(seed_mask, np.ndarray) else list(seed_mask))

    def build(x: np.ndarray) -> StrategyResult:
        plan: dict[str, list[TensorStatistics]] = {}
        for keep, (label, t) in zip(x > 0.5, cands):
            if keep:
                plan.setdefault(label, []).append(t)
        return StrategyResult(plan, build_block_data(plan, layer_stats, n_blocks, assignment))

    def cost(x: np.ndarray) -> float:
        r = build(x)
        peak = peak_memory(r, layer_stats)
        over = estimated_overhead(r.strategy_map, layer_stats, interp) if interp else 0.0
        off = sum(t.size_bytes for ts in r.strategy_map.values() for t in ts) / total_model
        pen = 0.0 if budget is None else max(0.0, peak - budget) / total_model * 100.0
        if memory_first:
            return pen * 10 + off + over
        return pen * 10 + over * 10 - off * 0.1

    best = {"f": np.inf, "stale": 0}
    patience = max(1, int(max_early_stop))

    def improved(f: float) -> bool:
        """Record ``f``; True once ``patience`` consecutive reports brought no improvement."""
        if f < best["f"] - 1e-12:
            best["f"], best["stale"] = f, 0
        else:
            best["stale"] += 1
        return best["stale"] >= patience

    rng = np.random.default_rng(seed)
    bounds = [(0.0, 1.0)] * len(cands)
    if optimizer == "DE":
        n_pop = max(5, pop_size)
        init = rng.random((n_pop, len(cands)))
        n_seeded = min(n_pop, max(1 if masks else 0, int(round(seed_ratio * n_pop))))
        for i in range(n_seeded):
            m = masks[i % len(masks)]
            jitter = rng.uniform(0.0, 0.3, len(cands)) if i >= len(masks) else 0.0
            init[i] = np.clip(np.where(m, 0.9, 0.1) + np.where(m, -jitter, jitter), 0.0, 1.0)

        def de_cb(intermediate_result):
            if improved(float(intermediate_result.fun)):
                raise StopIteration

        res = differential_evolution(cost, bounds=bounds, maxiter=max(1, epoch), init=init, seed=seed,
                                     polish=False, tol=1e-6, updating="deferred", callback=de_cb)
        x = res.x
    elif optimizer in ("SA", "DA"):
        x0 = np.where(masks[0], 0.9, 0.1) if masks else rng.random(len(cands))

        def sa_cb(xk, f, context):
            return improved(float(f))

        res = dual_annealing(cost, bounds=bounds, maxiter=max(1, epoch), seed=seed, x0=x0, no_local_search=True,
                             callback=sa_cb)
        x = res.x
    else:
        raise ValueError(f"optimizer must be 'DE' or 'SA', got {optimizer!r}")
    if masks:
        x0 = np.where(masks[0], 1.0, 0.0)
        if cost(x0) < cost(x):
            x = x0
    return build(x)


class GlobalTensorSelectionStrategy:
    """DE over per-tensor offload choices (seeded with the knapsack plan)."""

    def __init__(self, scale: float = 1.0, scale_ub: float | None = None, n_blocks: int = 4,
                 min_blocks: int | None = None, max_blocks: int | None = None, threshold_mb: float = 0.1,
                 pop_size: int = 50, epoch: int = 200, max_early_stop: int = 25, optimizer: str = "DE",
                 seed_ratio: float = 0.25, seed: int | None = None, assignment_strategy=None):
        if optimizer not in ("DE", "SA", "DA"):
            raise ValueError("optimizer must be 'DE' (differential evolution) or 'SA' (dual annealing; alias 'DA')")
        self.scale, self.scale_ub, self.n_blocks, self.threshold_mb = scale, scale_ub, n_blocks, threshold_mb
        self.pop_size, self.epoch, self.max_early_stop, self.seed = pop_size, epoch, max_early_stop, seed
        self.optimizer, self.seed_ratio = optimizer, seed_ratio
        self.assignment = assignment_strategy or OptimizedRoundRobinAssignment(
            min_blocks=min_blocks or 2, max_blocks=max_blocks or n_blocks)

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        require_layers(layer_stats)
        interp = interpolator_for(layer_stats, memory_stats)
        cands = [(layer_stats[j - 1].label, t) for j in range(1, len(layer_stats))
                 for t in eligible(layer_stats[j].tensors, self.threshold_mb)]
        # seed plans: the knapsack plan at the base scale and, up to scale_ub, at larger scales
        scales = [self.scale]
        if self.scale_ub is not None and self.scale_ub > self.scale:
            scales += list(np.linspace(self.scale, self.scale_ub, 4)[1:])
        masks = []
        for sc in scales:
            base = KnapsackBlockStrategy(float(sc), threshold_mb=self.threshold_mb, n_blocks=self.n_blocks).compute(
                layer_stats, memory_stats, max_gpu_mem_bytes)
            chosen = {t.tensor_id for ts in base.strategy_map.values() for t in ts}
            masks.append(np.array([t.tensor_id in chosen for _, t in cands], dtype=bool))
        return _de_select(cands, layer_stats, interp, self.n_blocks, self.assignment, max_gpu_mem_bytes, masks,
                          self.pop_size, self.epoch, self.max_early_stop, self.seed, memory_first=False,
                          optimizer=self.optimizer, seed_ratio=self.seed_ratio)


# --------------------------------------------------------------------------- budget-fill family


def _ranked_candidates(layer_stats, interp, scale, threshold_mb):
    """(transfer label, tensor) pairs ranked: transfer fits its window first, then larger first."""
    out = []
    for j in range(1, len(layer_stats)):
        window = layer_stats[j - 1].duration * scale
        for t in eligible(layer_stats[j].tensors, threshold_mb):
            ms = interp.bytes_to_duration(t.size_bytes) if interp else t.load_time_ms
            out.append((ms <= window, t.size_bytes, j, layer_stats[j - 1].label, t))
    out.sort(key=lambda c: (not c[0], -c[1], c[2]))
    return [(c[3], c[4]) for c in out]


def _budget_unreachable(name: str, budget: int, peak: int) -> None:
    warnings.warn(f"{name}: GPU budget {budget / 1024**3:.2f} GB is unreachable "
                  f"(best-effort peak {peak / 1024**3:.2f} GB)", UserWarning, stacklevel=3)


class BudgetFillGreedyStrategy:
    """Shortest ranked prefix whose plan fits ``max_gpu_mem_bytes``."""

    def __init__(self, n_blocks: int = 0, *, threshold_mb: float = 1.0, scale: float = 1.0,
                 assignment_strategy=None) -> None:
        validate_memory_params(scale)
        self.n_blocks, self.threshold_mb, self.scale = n_blocks, threshold_mb, scale
        self.assignment = assignment_strategy or StrictRoundRobinAssignment()

    def _build(self, prefix, layer_stats):
        plan: dict[str, list[TensorStatistics]] = {}
        for label, t in prefix:
            plan.setdefault(label, []).append(t)
        order = {l.label: i for i, l in enumerate(layer_stats)}
        plan = dict(sorted(plan.items(), key=lambda kv: order[kv[0]]))
        return StrategyResult(plan, build_block_data(plan, layer_stats, self.n_blocks, self.assignment))

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        require_layers(layer_stats)
        if max_gpu_mem_bytes is None:
            raise StrategyComputeError("BudgetFill strategies need max_gpu_mem_bytes")
        interp = interpolator_for(layer_stats, memory_stats)
        ranked = _ranked_candidates(layer_stats, interp, self.scale, self.threshold_mb)
        best = None
        for k in range(0, len(ranked) + 1):
            r = self._build(ranked[:k], layer_stats)
            if peak_memory(r, layer_stats) <= max_gpu_mem_bytes:
                return r
            if best is None or peak_memory(r, layer_stats) < peak_memory(best, layer_stats):
                best = r
        _budget_unreachable(type(self).__name__, max_gpu_mem_bytes, peak_memory(best, layer_stats))
        return best


class BudgetFillTensorDEStrategy:
    """Memory-first DE over per-tensor binaries."""

    def __init__(self, n_blocks: int = 0, *, threshold_mb: float = 1.0, scale: float = 1.0,
                 assignment_strategy=None, pop_size: int = 30, epoch: int = 80, max_early_stop: int = 25,
                 seed: int | None = None) -> None:
        self.n_blocks, self.threshold_mb, self.scale = n_blocks, threshold_mb, scale
        self.assignment = assignment_strategy or StrictRoundRobinAssignment()
        self.pop_size, self.epoch, self.max_early_stop, self.seed = pop_size, epoch, max_early_stop, seed

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        greedy = BudgetFillGreedyStrategy(self.n_blocks, threshold_mb=self.threshold_mb, scale=self.scale,
                                          assignment_strategy=self.assignment)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            base = greedy.compute(layer_stats, memory_stats, max_gpu_mem_bytes)
        interp = interpolator_for(layer_stats, memory_stats)
        chosen = {t.tensor_id for ts in base.strategy_map.values() for t in ts}
        cands = [(layer_stats[j - 1].label, t) for j in range(1, len(layer_stats))
                 for t in eligible(layer_stats[j].tensors, self.threshold_mb)]
        mask = np.array([t.tensor_id in chosen for _, t in cands], dtype=bool)
        r = _de_select(cands, layer_stats, interp, self.n_blocks, self.assignment, max_gpu_mem_bytes, mask,
                       self.pop_size, self.epoch, self.max_early_stop, self.seed, memory_first=True)
        sb = evaluate_strategy_result(base, layer_stats, "g", interp, max_gpu_mem_bytes)
        sr = evaluate_strategy_result(r, layer_stats, "de", interp, max_gpu_mem_bytes)
        return r if (sr.is_valid and _offloaded(r) < _offloaded(base)) or not sb.is_valid and sr < sb else base


def _offloaded(r: StrategyResult) -> int:
    return sum(t.size_bytes for ts in r.strategy_map.values() for t in ts)


class BudgetFillLayerDEStrategy:
    """Memory-first DE over per-layer offload fractions (largest tensors first within a layer)."""

    def __init__(self, n_blocks: int = 0, *, threshold_mb: float = 1.0, scale: float = 1.0,
                 assignment_strategy=None, pop_size: int = 20, epoch: int = 60, max_early_stop: int = 20,
                 seed: int | None = None) -> None:
        self.n_blocks, self.threshold_mb, self.scale = n_blocks, threshold_mb, scale
        self.assignment = assignment_strategy or StrictRoundRobinAssignment()
        self.pop_size, self.epoch, self.max_early_stop, self.seed = pop_size, epoch, max_early_stop, seed

    def _build(self, fr: np.ndarray, layer_stats) -> StrategyResult:
        plan: dict[str, list[TensorStatistics]] = {}
        for j in range(1, len(layer_stats)):
            cand = sorted(eligible(layer_stats[j].tensors, self.threshold_mb), key=lambda t: -t.size_bytes)
            tot = sum(t.size_bytes for t in cand)
            goal = fr[j - 1] * tot
            acc, take = 0, []
            for t in cand:
                if acc >= goal - 1e-9:
                    break
                take.append(t)
                acc += t.size_bytes
            if take:
                plan[layer_stats[j - 1].label] = take
        return StrategyResult(plan, build_block_data(plan, layer_stats, self.n_blocks, self.assignment))

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        require_layers(layer_stats)
        if max_gpu_mem_bytes is None:
            raise StrategyComputeError("BudgetFill strategies need max_gpu_mem_bytes")
        from scipy.optimize import differential_evolution

        total_model = sum(t.size_bytes for l in layer_stats for t in l.tensors) or 1
        interp = interpolator_for(layer_stats, memory_stats)

        def cost(fr):
            r = self._build(fr, layer_stats)
            peak = peak_memory(r, layer_stats)
            pen = max(0.0, peak - max_gpu_mem_bytes) / total_model * 1000.0
            over = estimated_overhead(r.strategy_map, layer_stats, interp) if interp else 0.0
            return pen + _offloaded(r) / total_model + over

        n = len(layer_stats) - 1
        rng = np.random.default_rng(self.seed)
        init = rng.random((max(5, self.pop_size), n))
        init[0] = 1.0  # stream everything eligible
        # the greedy budget fill at this scale, as per-layer fractions
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            greedy = BudgetFillGreedyStrategy(self.n_blocks, threshold_mb=self.threshold_mb, scale=self.scale,
                                              assignment_strategy=self.assignment).compute(
                layer_stats, memory_stats, max_gpu_mem_bytes)
        for j in range(1, len(layer_stats)):
            tot = sum(t.size_bytes for t in eligible(layer_stats[j].tensors, self.threshold_mb))
            got = sum(t.size_bytes for t in greedy.strategy_map.get(layer_stats[j - 1].label, ()))
            init[1, j - 1] = min(1.0, got / tot) if tot else 0.0
        state = {"f": np.inf, "stale": 0}

        def stop_when_stale(intermediate_result):
            if intermediate_result.fun < state["f"] - 1e-12:
                state["f"], state["stale"] = intermediate_result.fun, 0
            else:
                state["stale"] += 1
            if state["stale"] >= max(1, self.max_early_stop):
                raise StopIteration

        res = differential_evolution(cost, [(0.0, 1.0)] * n, maxiter=self.epoch, init=init, seed=self.seed,
                                     polish=False, tol=1e-7, updating="deferred", callback=stop_when_stale)
        r = self._build(res.x, layer_stats)
        if peak_memory(r, layer_stats) > max_gpu_mem_bytes:
            full = self._build(np.ones(n), layer_stats)
            if peak_memory(full, layer_stats) > max_gpu_mem_bytes:
                _budget_unreachable(type(self).__name__, max_gpu_mem_bytes, peak_memory(full, layer_stats))
            return full
        return r


class BudgetFillStrategy:
    """Greedy, then (optionally) layer-DE and tensor-DE; keeps the valid plan that offloads least."""

    def __init__(self, n_blocks: int = 0, *, threshold_mb: float = 1.0, scale: float = 1.0,
                 assignment_strategy=None, enable_layer_de: bool = True, enable_tensor_de: bool = True,
                 pop_size: int = 20, epoch: int = 60, max_early_stop: int = 20, seed: int | None = None) -> None:
        self.kw = dict(threshold_mb=threshold_mb, scale=scale, assignment_strategy=assignment_strategy)
        self.n_blocks = n_blocks
        self.enable_layer_de, self.enable_tensor_de = enable_layer_de, enable_tensor_de
        self.de_kw = dict(pop_size=pop_size, epoch=epoch, max_early_stop=max_early_stop, seed=seed)

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        solvers = [BudgetFillGreedyStrategy(self.n_blocks, **self.kw)]
        if self.enable_layer_de:
            solvers.append(BudgetFillLayerDEStrategy(self.n_blocks, **self.kw, **self.de_kw))
        if self.enable_tensor_de:
            solvers.append(BudgetFillTensorDEStrategy(self.n_blocks, **self.kw, **self.de_kw))
        interp = interpolator_for(layer_stats, memory_stats)
        best, best_key = None, None
        for s in solvers:
            with warnings.catch_warnings():
                warnings.simplefilter("ignore")
                r = s.compute(layer_stats, memory_stats, max_gpu_mem_bytes)
            sc = evaluate_strategy_result(r, layer_stats, type(s).__name__, interp, max_gpu_mem_bytes)
            key = (not sc.is_valid, _offloaded(r), sc.estimated_overhead, sc.peak_memory_bytes)
            if best_key is None or key < best_key:
                best, best_key = r, key
        if best_key[0]:
            _budget_unreachable("BudgetFillStrategy", max_gpu_mem_bytes, peak_memory(best, layer_stats))
        return best


_ = MB
