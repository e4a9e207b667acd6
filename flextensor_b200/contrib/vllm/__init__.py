"""vLLM integration: a worker class that streams decoder-layer weights from host memory.

    vllm serve <model> --worker-cls flextensor_b200.contrib.vllm.worker.FlexTensorOffloadWorker

with ``FT_ENABLED=1`` and any other ``FT_*`` OffloadConfig fields in the environment (or a
config file named by ``FT_CONFIG_FILE``). Parity: ``src/flextensor/contrib/vllm/worker.py``
(class path), ``v2/worker.py`` (load_model takeover), ``_patterns.py`` (default selectors).
"""

from flextensor_b200.contrib.vllm.patterns import (
    VLLM_DEFAULT_EXCLUDE_PATTERNS,
    VLLM_DEFAULT_INCLUDE_PATTERNS,
    resolve_vllm_patterns,
)

__all__ = ["VLLM_DEFAULT_EXCLUDE_PATTERNS", "VLLM_DEFAULT_INCLUDE_PATTERNS", "resolve_vllm_patterns"]
