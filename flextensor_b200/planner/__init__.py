"""Placement planner (pure CPU: numpy/scipy only; imports nothing from the runtime)."""

from flextensor_b200.planner.adaptive import AdaptiveStrategy
from flextensor_b200.planner.blocks import (
    AssignmentStrategy,
    MemoryBlockPlanner,
    OptimizedRoundRobinAssignment,
    StrictRoundRobinAssignment,
)
from flextensor_b200.planner.common import (
    StrategyScore,
    calculate_transfer_to_compute_map,
    evaluate_strategy_result,
    reverse_transfer_to_compute_map,
)
from flextensor_b200.planner.interpolator import MemoryTransferInterpolator
from flextensor_b200.planner.protocol import BlockStrategyData, Strategy, StrategyComputeError, StrategyResult
from flextensor_b200.planner.strategies import (
    AdaptiveKnapsackStrategy,
    BudgetFillGreedyStrategy,
    BudgetFillLayerDEStrategy,
    BudgetFillStrategy,
    BudgetFillTensorDEStrategy,
    GlobalOffloadStrategy,
    GlobalTensorSelectionStrategy,
    GreedyStrategy,
    KnapsackBlockStrategy,
    KnapsackStrategy,
    NthLayerStrategy,
)

__all__ = [
    "AdaptiveKnapsackStrategy", "AdaptiveStrategy", "AssignmentStrategy", "BlockStrategyData",
    "BudgetFillGreedyStrategy", "BudgetFillLayerDEStrategy", "BudgetFillStrategy", "BudgetFillTensorDEStrategy",
    "GlobalOffloadStrategy", "GlobalTensorSelectionStrategy", "GreedyStrategy", "KnapsackBlockStrategy",
    "KnapsackStrategy", "MemoryBlockPlanner", "MemoryTransferInterpolator", "NthLayerStrategy",
    "OptimizedRoundRobinAssignment", "Strategy", "StrategyComputeError", "StrategyResult", "StrategyScore",
    "StrictRoundRobinAssignment", "calculate_transfer_to_compute_map", "evaluate_strategy_result",
    "reverse_transfer_to_compute_map",
]
