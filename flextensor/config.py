"""Alias of :mod:`flextensor_b200.config`."""

from flextensor_b200.config import *  # noqa: F401,F403
from flextensor_b200.config import OffloadConfig, load_config, load_config_from_env, load_config_from_file  # noqa: F401
