"""Multi-GPU data plane on one node: symmetric peer heaps, striped host streaming, context /
tensor / expert parallelism with the collectives fused into the kernels, pipeline stages over NCCL
send/recv, NCCL baselines, and a bounded CPU control plane."""

from flextensor_b200.parallel.control import ControlPlane, ReplicaFatalError
from flextensor_b200.parallel.cp import ContextParallel, UlyssesAttention
from flextensor_b200.parallel.ep import ExpertParallel, NcclExpertParallel, route_topk
from flextensor_b200.parallel.striped import (
    StripedTransferEngine,
    disable_striped_streaming,
    enable_striped_streaming,
    striping_group,
)
from flextensor_b200.parallel.pp import PipelineStage, TorchP2P, pipeline_groups, split_stages
from flextensor_b200.parallel.symm import SymmetricHeap
from flextensor_b200.parallel.tp import NcclTP, TPAllGather, TPAllReduce, TPReduceScatter, TPRMSNorm, nccl_rmsnorm

__all__ = ["ContextParallel", "ControlPlane", "disable_striped_streaming", "enable_striped_streaming",
           "ExpertParallel", "nccl_rmsnorm", "NcclExpertParallel", "NcclTP", "pipeline_groups", "PipelineStage",
           "ReplicaFatalError", "route_topk", "split_stages", "StripedTransferEngine", "striping_group",
           "SymmetricHeap", "TorchP2P", "TPAllGather", "TPAllReduce", "TPReduceScatter", "TPRMSNorm",
           "UlyssesAttention"]
