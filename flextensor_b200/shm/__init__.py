"""Cross-process host weight sharing over POSIX shared memory (protocol v4)."""

from flextensor_b200.shm.coordinator import (
    CoordBlockHeader,
    CoordinatorState,
    ShmCoordinator,
    ShmCoordinatorError,
    ShmCreatorDiedError,
    ShmCreatorFailedError,
    cleanup_namespace,
    retire_abandoned,
)
from flextensor_b200.shm.namespace import (
    SHM_PROTOCOL_VERSION,
    apply_rank_suffix,
    compute_shm_namespace,
    coord_block_name,
    profile_block_name,
    weight_block_name,
)
from flextensor_b200.shm.segment import ProcessFileLock, ShmSegment
from flextensor_b200.shm.store import ShmWeightStore
from flextensor_b200.shm.sync import MultiprocessCondition, SemaphoreLock, SharedMultiString
from flextensor_b200.shm.tensor_store import SharedTensorStore

__all__ = [
    "CoordBlockHeader", "CoordinatorState", "ProcessFileLock", "SHM_PROTOCOL_VERSION", "SharedTensorStore",
    "ShmCoordinator", "ShmCoordinatorError", "ShmCreatorDiedError", "ShmCreatorFailedError", "ShmSegment",
    "ShmWeightStore", "MultiprocessCondition", "SemaphoreLock", "SharedMultiString", "apply_rank_suffix", "cleanup_namespace", "compute_shm_namespace", "coord_block_name",
    "profile_block_name", "retire_abandoned", "weight_block_name",
]
