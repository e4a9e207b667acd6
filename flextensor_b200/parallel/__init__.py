"""Multi-GPU data plane: symmetric peer heaps, striped host streaming, NCCL helpers."""

from flextensor_b200.parallel.striped import (
    StripedTransferEngine,
    disable_striped_streaming,
    enable_striped_streaming,
    striping_group,
)
from flextensor_b200.parallel.symm import SymmetricHeap

__all__ = ["StripedTransferEngine", "SymmetricHeap", "disable_striped_streaming", "enable_striped_streaming",
           "striping_group"]
