"""vLLM offloader hook: keep decoder layers off the GPU while vLLM builds and loads them.

vLLM passes every decoder layer it constructs through the process-wide offloader's
``wrap_modules`` (``vllm/model_executor/models/utils.py``, ``make_layers``). This offloader
moves each layer's parameters to host memory as soon as the layer exists, so weight loading
fills host tensors and the whole model never has to fit on the GPU; the FlexTensor runtime
then takes the model over. Afterwards it forwards vLLM's graph-boundary calls to the runtime:
``sync_prev_onload`` (before a captured region) waits for outstanding copies, and
``join_after_forward`` (at a piecewise CUDA-graph boundary) joins the copy stream.
Parity: ``src/flextensor/contrib/vllm/v2/offloader.py:108-411`` (bootstrap staging + hooks).
"""

from __future__ import annotations

import logging

import torch
from torch import nn

LOGGER = logging.getLogger(__name__)


def _base():
    from vllm.model_executor.offloader.base import BaseOffloader

    return BaseOffloader


class FlexTensorBootstrapOffloader(_base()):  # type: ignore[misc]
    def __init__(self, stage_on_host: bool = True) -> None:
        self.stage_on_host = stage_on_host
        self.staged_modules: list[nn.Module] = []
        self.staged_bytes = 0
        self.manager = None  # set by the worker once the runtime owns the model

    def wrap_modules(self, modules_generator):
        out = []
        for m in modules_generator:
            if self.stage_on_host:
                self._stage(m)
            out.append(m)
        return out

    @torch.no_grad()
    def _stage(self, m: nn.Module) -> None:
        seen: set[int] = set()
        for p in m.parameters():
            if id(p) in seen or p.device.type != "cuda":
                continue
            seen.add(id(p))
            p.data = p.data.to("cpu")
            self.staged_bytes += p.numel() * p.element_size()
        self.staged_modules.append(m)
        if self.staged_modules and len(self.staged_modules) % 16 == 0:
            torch.cuda.empty_cache()

    def post_init(self) -> None:
        torch.cuda.empty_cache()

    def _loader(self):
        tm = self.manager.get_tensor_manager() if self.manager is not None else None
        return getattr(tm, "loader", None) if tm is not None else None

    def sync_prev_onload(self) -> None:
        ld = self._loader()
        if ld is not None:
            ld.sync_prev_onload()

    def join_after_forward(self) -> None:
        ld = self._loader()
        if ld is not None and hasattr(ld, "piece_join"):
            ld.piece_join()
