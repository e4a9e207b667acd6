"""Default unit selectors for vLLM decoder models.

One offload unit per transformer layer (selected by class name, which stays stable across
vLLM releases where module paths move), plus the embedding, final norm and LM head of plain
and wrapped (``language_model.``) causal LMs. Small routing/gating tensors and sidecar modules
that vLLM drives from its own fused kernels or side streams stay resident. The same selector
set as the reference (``src/flextensor/contrib/vllm/_patterns.py:15-66``): a user switching
frameworks gets the same units.
"""

from __future__ import annotations

from typing import Any

VLLM_DEFAULT_INCLUDE_PATTERNS: list[str] = [
    "class:*DecoderLayer",
    "class:*DecoderBlock",
    "class:*TransformerBlock",
    "model.embed_tokens",
    "model.norm",
    "model.norm_f",
    "lm_head",
    "logits_processor",
    "language_model.model.embed_tokens",
    "language_model.model.norm",
    "language_model.lm_head",
    "language_model.logits_processor",
]

VLLM_DEFAULT_EXCLUDE_PATTERNS: list[str] = [
    "class:GateLinear",
    "model.layers.*.mixer.shared_experts",
    "model.layers.*.mixer.fc1_latent_proj",
    "model.layers.*.mixer.fc2_latent_proj",
    "model.layers.*.mlp.shared_expert",
    "language_model.model.layers.*.mlp.shared_expert",
    "language_model.model.layers.*.mlp.gate",
    "language_model.model.layers.*.mlp.shared_expert_gate",
    "language_model.model.layers.*.linear_attn.A_log",
    "language_model.model.layers.*.linear_attn.dt_bias",
]


def resolve_vllm_patterns(config: Any) -> tuple[list[str], list[str]]:
    """Defaults for ``include_patterns == ["*"]`` and for excludes the user never set (an
    explicitly empty exclude list stays empty)."""
    inc = list(VLLM_DEFAULT_INCLUDE_PATTERNS) if list(config.include_patterns) == ["*"] else list(
        config.include_patterns)
    exc = list(config.exclude_patterns)
    if not exc and "exclude_patterns" not in getattr(config, "model_fields_set", set()):
        exc = list(VLLM_DEFAULT_EXCLUDE_PATTERNS)
    return inc, exc
