"""``import flextensor`` compatibility facade: the public API of ai-dynamo/flextensor served by
``flextensor_b200`` (names, signatures, config schema and file formats are the same), so
existing user code and class paths such as
``flextensor.contrib.vllm.worker.FlexTensorOffloadWorker`` keep working unchanged."""

from flextensor_b200 import *  # noqa: F401,F403
from flextensor_b200 import __all__ as _all
from flextensor_b200 import __version__  # noqa: F401

__all__ = list(_all)
