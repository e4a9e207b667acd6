"""Reference class path of the vLLM worker: ``--worker-cls
flextensor.contrib.vllm.worker.FlexTensorOffloadWorker``."""

from flextensor_b200.contrib.vllm.worker import FlexTensorOffloadWorker  # noqa: F401

__all__ = ["FlexTensorOffloadWorker"]
