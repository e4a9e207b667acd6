"""``AdaptiveStrategy``: run several planners and keep the best-scoring plan.

Candidate set and ranking follow ``src/flextensor/strategy/adaptive.py:123-306``:
block loaders try KnapsackBlock, GlobalOffload with optimised and strict slot
assignment, BudgetFill when a memory budget exists, and (with
``extra_optimization``) DE tensor selection; the per-tensor loader tries
Knapsack. Scores order valid < invalid, then overhead, then peak bytes.
"""

from __future__ import annotations

import logging
import time
import warnings

from flextensor_b200.planner.blocks import OptimizedRoundRobinAssignment, StrictRoundRobinAssignment
from flextensor_b200.planner.common import StrategyScore, evaluate_strategy_result, interpolator_for
from flextensor_b200.planner.protocol import StrategyComputeError, StrategyResult
from flextensor_b200.planner.strategies import (
    BudgetFillStrategy,
    GlobalOffloadStrategy,
    GlobalTensorSelectionStrategy,
    KnapsackBlockStrategy,
    KnapsackStrategy,
)

logger = logging.getLogger(__name__)


class AdaptiveStrategy:
    BLOCK_LOADER_TYPES = frozenset({"allocation_block_transfer", "raw_block_transfer"})

    def __init__(self, scale: float = 1.0, loader_type: str = "allocation_block_transfer", cyclic: bool = False,
                 group_size: int = 1, threshold_mb: float = 0.1, min_blocks: int = 2, n_blocks: int = 4,
                 extra_optimization: bool = False):
        if n_blocks < 2 or min_blocks < 2 or min_blocks > n_blocks:
            raise ValueError(f"need 2 <= min_blocks ({min_blocks}) <= n_blocks ({n_blocks})")
        self.scale, self.loader_type, self.cyclic, self.group_size = scale, loader_type, cyclic, group_size
        self.threshold_mb, self.min_blocks, self.n_blocks = threshold_mb, min_blocks, n_blocks
        self.extra_optimization = extra_optimization
        self._all_scores: list[StrategyScore] = []
        self._selected_strategy_name: str | None = None

    def _candidates(self, max_gpu_mem_bytes):
        s, th, nb, mb = self.scale, self.threshold_mb, self.n_blocks, self.min_blocks
        if self.loader_type not in self.BLOCK_LOADER_TYPES:
            return [("Knapsack", KnapsackStrategy(scale=s, cyclic=self.cyclic, group_size=self.group_size,
                                                  threshold_mb=th))]
        opt = lambda: OptimizedRoundRobinAssignment(min_blocks=mb, max_blocks=nb)  # noqa: E731
        out = [
            ("KnapsackBlock", KnapsackBlockStrategy(scale=s, group_size=self.group_size, threshold_mb=th, n_blocks=nb)),
            ("GlobalOffload(Optimized)", GlobalOffloadStrategy(scale=s, threshold_mb=th, n_blocks=nb,
                                                               assignment_strategy=opt())),
            ("GlobalOffload(Strict)", GlobalOffloadStrategy(scale=s, threshold_mb=th, n_blocks=nb,
                                                            assignment_strategy=StrictRoundRobinAssignment())),
        ]
        if max_gpu_mem_bytes is not None:
            out.append(("BudgetFill", BudgetFillStrategy(n_blocks=nb, threshold_mb=th, scale=s,
                                                         assignment_strategy=opt(), enable_layer_de=True,
                                                         enable_tensor_de=False)))
        if self.extra_optimization:
            for nm, a in (("Optimized", opt()), ("Strict", StrictRoundRobinAssignment())):
                out.append((f"TensorSelection({nm})", GlobalTensorSelectionStrategy(
                    scale=s, threshold_mb=th, n_blocks=nb, pop_size=50, epoch=100, max_early_stop=50,
                    assignment_strategy=a)))
        return out

    def compute(self, layer_stats, memory_stats=None, max_gpu_mem_bytes=None) -> StrategyResult:
        interp = interpolator_for(layer_stats, memory_stats)
        best, best_score, scores = None, None, []
        for name, strat in self._candidates(max_gpu_mem_bytes):
            t0 = time.perf_counter()
            try:
                with warnings.catch_warnings():
                    warnings.simplefilter("ignore")
                    r = strat.compute(layer_stats, memory_stats, max_gpu_mem_bytes)
            except StrategyComputeError:
                logger.warning("Strategy %s failed, skipping", name, exc_info=True)
                continue
            sc = evaluate_strategy_result(r, layer_stats, name, interp, max_gpu_mem_bytes)
            scores.append(sc)
            logger.debug("candidate %-28s overhead=%.2f%% peak=%.2fGB viol=%d valid=%s (%.2fs)", name,
                         sc.estimated_overhead * 100, sc.peak_memory_bytes / 1024**3, sc.consecutive_violations,
                         sc.is_valid, time.perf_counter() - t0)
            if best_score is None or sc < best_score:
                best, best_score = r, sc
        self._all_scores = scores
        if best is None:
            raise RuntimeError("All strategy candidates failed — no result produced")
        self._selected_strategy_name = best_score.strategy_name
        if not best_score.is_valid:
            warnings.warn(f"AdaptiveStrategy: best result ({best_score.strategy_name}) is not fully valid — "
                          f"peak={best_score.peak_memory_bytes / 1024**3:.2f} GB, "
                          f"violations={best_score.consecutive_violations}", UserWarning, stacklevel=2)
        return best

    @property
    def selected_strategy_name(self) -> str:
        if self._selected_strategy_name is None:
            raise RuntimeError("selected_strategy_name is not available until compute() has been called")
        return self._selected_strategy_name

    @property
    def all_scores(self) -> list[StrategyScore]:
        return list(self._all_scores)
