"""Alias of :mod:`flextensor_b200.instrumentation`."""

from flextensor_b200.instrumentation import *  # noqa: F401,F403
from flextensor_b200.instrumentation import __all__  # noqa: F401
