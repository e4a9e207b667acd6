"""Join the offload runtime's copy stream at every eager break of a vLLM CUDA-graph capture.

vLLM's breakable CUDA-graph capture (``vllm.compilation.breakable_cudagraph``,
``BreakableCUDAGraphCapture.add_eager``) closes the current capture segment wherever an op must
run eagerly, often in the middle of a decoder layer. vLLM itself asks the offloader to join only
before the LAST segment closes. A prefetch that a layer's trap forked onto the copy stream would
then still be unjoined when the segment ends: the capture fails with an unjoined-stream error,
and the copy's readiness event belongs to a capture that no longer exists.

:func:`install_segment_join` wraps ``add_eager`` so that, while a capture is running, the
process's offloader joins its copy stream first (``join_after_forward``, which for the
FlexTensor offloader is the runtime's piecewise join). Idempotent; returns False on vLLM builds
without breakable capture. Parity: ``src/flextensor/contrib/vllm/v2/breakable_cudagraph.py:26``.
"""

from __future__ import annotations

import functools
import logging

LOGGER = logging.getLogger("vllm.flextensor_b200.graph_join")
_MARK = "__ft_joins_offloader__"


def install_segment_join() -> bool:
    try:
        from vllm.compilation.breakable_cudagraph import BreakableCUDAGraphCapture
        from vllm.model_executor.offloader.base import get_offloader
    except ImportError:
        return False
    original = BreakableCUDAGraphCapture.add_eager
    if getattr(original, _MARK, False):
        return True

    @functools.wraps(original)
    def add_eager(capture, fn):
        if getattr(capture, "_capturing", False):
            get_offloader().join_after_forward()
        return original(capture, fn)

    setattr(add_eager, _MARK, True)
    BreakableCUDAGraphCapture.add_eager = add_eager
    LOGGER.info("offload runtime joins its copy stream before every eager break of a CUDA-graph capture")
    return True
