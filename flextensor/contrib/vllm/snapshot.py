"""Reference class paths of the memory snapshot workers: ``--worker-cls
flextensor.contrib.vllm.snapshot.SnapshotWorker`` / ``...FlexTensorSnapshotWorker``."""

from flextensor_b200.contrib.vllm.snapshot import *  # noqa: F401,F403
from flextensor_b200.contrib.vllm.snapshot import MemorySnapshotMixin  # noqa: F401

try:
    from flextensor_b200.contrib.vllm.snapshot import FlexTensorSnapshotWorker, SnapshotWorker  # noqa: F401
except ImportError:  # vLLM not installed
    pass
