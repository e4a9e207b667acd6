"""Hand-written sm_100a kernels (tcgen05 GEMM, flash attention, norms/RoPE) and their Python entry points."""

from flextensor_b200.ops.api import (
    EPI,
    attention,
    layernorm_modulate,
    linear,
    qk_rmsnorm_rope,
    rmsnorm,
)

__all__ = ["EPI", "attention", "layernorm_modulate", "linear", "qk_rmsnorm_rope", "rmsnorm"]
