"""Alias of :mod:`flextensor_b200.contrib.vllm`."""

from flextensor_b200.contrib.vllm import *  # noqa: F401,F403
