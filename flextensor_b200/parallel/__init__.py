"""Multi-GPU data plane on one node: symmetric peer heaps, striped host streaming, context /
tensor / expert parallelism with the collectives fused into the kernels, NCCL baselines, and a
bounded CPU control plane."""

from flextensor_b200.parallel.control import ControlPlane, ReplicaFatalError
from flextensor_b200.parallel.cp import ContextParallel, UlyssesAttention
from flextensor_b200.parallel.ep import ExpertParallel, NcclExpertParallel, route_topk
from flextensor_b200.parallel.striped import (
    StripedTransferEngine,
    disable_striped_streaming,
    enable_striped_streaming,
    striping_group,
)
from flextensor_b200.parallel.symm import SymmetricHeap
from flextensor_b200.parallel.tp import NcclTP, TPAllGather, TPAllReduce, TPReduceScatter, TPRMSNorm, nccl_rmsnorm

__all__ = ["ContextParallel", "ControlPlane", "ExpertParallel", "NcclExpertParallel", "NcclTP", "ReplicaFatalError",
           "StripedTransferEngine", "SymmetricHeap", "TPAllGather", "TPAllReduce", "TPRMSNorm", "TPReduceScatter", "UlyssesAttention",
           "disable_striped_streaming", "enable_striped_streaming", "nccl_rmsnorm", "route_topk", "striping_group"]
