"""Hand-written sm_100a kernels (tcgen05 GEMM, flash attention, norms/RoPE, fused
tensor/context-parallel collectives) and their Python entry points."""

from flextensor_b200.ops.api import (
    EPI,
    TP_EPI,
    attention,
    attention_cp,
    decode_attention,
    launch_count,
    layernorm_modulate,
    linear,
    linear_swiglu,
    qk_rmsnorm_rope,
    rmsnorm,
    rope,
    tp_ag_counter_words,
    tp_allgather_gemm,
    tp_gemm_reducescatter,
    tp_reduce,
    tp_rmsnorm,
)

__all__ = ["EPI", "TP_EPI", "attention", "attention_cp", "decode_attention", "launch_count", "layernorm_modulate", "linear",
           "linear_swiglu", "qk_rmsnorm_rope", "rmsnorm", "rope", "tp_ag_counter_words", "tp_allgather_gemm", "tp_gemm_reducescatter",
           "tp_reduce", "tp_rmsnorm"]
