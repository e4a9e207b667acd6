"""flextensor_b200: a Blackwell-native weight-offloading inference runtime.

Public API parity with the reference facade (``src/flextensor/__init__.py:31-141``):
``import flextensor_b200 as flextensor`` gives the same names.
"""

import os as _os

# Runtime type checks of the whole package (beartype's import hook) before any submodule loads:
# on with ENABLE_BEARTYPE=1, and never when DISABLE_BEARTYPE is set (the reference's switch). They
# are off by default here because they sit on the per-trap hot path of inference.
if _os.environ.get("ENABLE_BEARTYPE", "0") == "1" and not _os.environ.get("DISABLE_BEARTYPE"):
    try:
        from beartype import BeartypeConf as _BeartypeConf
        from beartype.claw import beartype_this_package as _beartype_this_package

        _beartype_this_package(conf=_BeartypeConf(is_pep484_tower=True))  # an int is a valid float
    except ImportError:  # beartype not installed: run unchecked
        pass

from flextensor_b200._version import __version__  # noqa: E402
from flextensor_b200.config import (
    OffloadConfig,
    PinnedMemoryMode,
    load_config,
    load_config_from_env,
    load_config_from_file,
)
from flextensor_b200.core.state import TensorManagerState
from flextensor_b200.planner import (
    AdaptiveKnapsackStrategy,
    AdaptiveStrategy,
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
    Strategy,
)
from flextensor_b200.runtime.benchmark_modes import BenchmarkReplace, PreloadToDevice, TensorBenchmarkMode
from flextensor_b200.runtime.lazy_init import load_model_from_profile
from flextensor_b200.runtime.manager import (
    DEFAULT_MANAGER_NAME,
    OffloadManager,
    OffloadModelProxy,
    OffloadPhase,
    StrategyReplanStatus,
    clear_profiling_durations,
    collect_offload_timing,
    get_gpu_memory_usage,
    get_offload_manager,
    init,
    load_profile,
    offload,
    offload_block,
    offload_from_profile,
    offload_from_state,
    offload_units,
    pause_profiling,
    release,
    request_strategy_replan,
    reset_offload_timing,
    resident_units,
    resume_profiling,
    save_profile,
    set_config,
    suspend_profiling,
    update_offload_timing,
    update_state,
)
from flextensor_b200.runtime.tensor_manager import TensorManager
from flextensor_b200.runtime.timing import OffloadTimingReport, OffloadTimingSnapshot, format_offload_timing_table
from flextensor_b200.shared_offload import SharedOffloadSession
from flextensor_b200.shm.coordinator import ShmCoordinatorError, ShmCreatorDiedError, ShmCreatorFailedError
from flextensor_b200.types import GPUMemoryUsage

__all__ = [
    "DEFAULT_MANAGER_NAME", "GPUMemoryUsage", "OffloadConfig", "OffloadManager", "PinnedMemoryMode",
    "SharedOffloadSession", "ShmCoordinatorError", "ShmCreatorDiedError", "ShmCreatorFailedError",
    "StrategyReplanStatus", "clear_profiling_durations", "collect_offload_timing", "format_offload_timing_table",
    "get_gpu_memory_usage", "get_offload_manager", "init", "load_config", "load_config_from_env",
    "load_config_from_file", "offload", "offload_block", "offload_from_profile", "offload_from_state",
    "offload_units", "request_strategy_replan", "resident_units", "reset_offload_timing", "set_config",
    "save_profile", "load_profile", "pause_profiling", "release", "resume_profiling", "suspend_profiling",
    "update_state", "update_offload_timing",
    "AdaptiveKnapsackStrategy", "AdaptiveStrategy", "BenchmarkReplace", "GlobalOffloadStrategy",
    "GlobalTensorSelectionStrategy", "BudgetFillStrategy", "BudgetFillGreedyStrategy", "BudgetFillTensorDEStrategy",
    "BudgetFillLayerDEStrategy", "GreedyStrategy", "KnapsackBlockStrategy", "KnapsackStrategy",
    "load_model_from_profile", "NthLayerStrategy", "PreloadToDevice", "Strategy", "TensorBenchmarkMode",
    "TensorManager", "OffloadTimingReport", "OffloadTimingSnapshot",
    # additions
    "OffloadModelProxy", "OffloadPhase", "TensorManagerState",
]
