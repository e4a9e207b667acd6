"""Alias of :mod:`flextensor_b200.shared_offload`."""

from flextensor_b200.shared_offload import *  # noqa: F401,F403
from flextensor_b200.shared_offload import SharedOffloadSession  # noqa: F401
