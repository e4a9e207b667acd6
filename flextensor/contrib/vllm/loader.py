"""Reference module path of the host-first model loader (registers ``load_format="flextensor"``)."""

from flextensor_b200.contrib.vllm.loader import *  # noqa: F401,F403
from flextensor_b200.contrib.vllm.loader import FlexTensorModelLoader  # noqa: F401
