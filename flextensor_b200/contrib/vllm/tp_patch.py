"""Fused GEMM + all-reduce for vLLM's row-parallel layers (``FT_VLLM_FUSED_TP=1``).

vLLM's ``RowParallelLinear`` computes a partial product on every tensor-parallel rank and
all-reduces it (NCCL or vLLM's custom all-reduce). With this patch the partial rows leave the
tcgen05 GEMM's epilogue straight into their owner rank's staging buffer over NVLink, each owner
sums its rows in fp32 and writes them into every rank's output, and every rank waits (bounded,
on the device) for the owners' acknowledgements (:class:`~flextensor_b200.parallel.tp.TPAllReduce`).

Applied to unquantized bf16 layers without bias when vLLM runs eagerly (the epoch bookkeeping
lives on the host, so CUDA-graph replays are not supported); every other layer keeps vLLM's path.
"""

from __future__ import annotations

import logging
import types

import torch

LOGGER = logging.getLogger("vllm.flextensor_b200.tp_patch")


def _eligible(layer) -> bool:
    w = getattr(layer, "weight", None)
    return (isinstance(w, torch.Tensor) and w.dtype == torch.bfloat16 and w.dim() == 2 and w.is_cuda
            and getattr(layer, "bias", None) is None and getattr(layer, "reduce_results", False)
            and not getattr(layer, "skip_bias_add", False) and getattr(layer, "tp_size", 1) > 1
            and type(getattr(layer, "quant_method", None)).__name__ == "UnquantizedLinearMethod"
            and w.shape[1] % 8 == 0 and w.shape[0] % 32 == 0)


def patch_row_parallel(model: torch.nn.Module, max_rows: int, group) -> int:
    """Route every eligible ``RowParallelLinear`` of ``model`` through the fused all-reduce.
    Returns the number of patched layers."""
    from vllm.model_executor.layers.linear import RowParallelLinear

    from flextensor_b200.parallel.tp import TPAllReduce

    reducers: dict[int, TPAllReduce] = {}
    patched = 0
    for name, layer in model.named_modules():
        if not isinstance(layer, RowParallelLinear) or not _eligible(layer):
            continue
        n = layer.weight.shape[0]
        if n not in reducers:
            reducers[n] = TPAllReduce(max_rows, n, group=group, device=layer.weight.device.index)
        ar = reducers[n]
        orig = layer.forward

        def fused_forward(self, input_, _ar=ar, _orig=orig):
            if self.input_is_parallel:
                x = input_
            else:
                x = input_.chunk(self.tp_size, dim=-1)[self.tp_rank]
            x2 = x.reshape(-1, x.shape[-1])
            if x2.shape[0] == 0 or x2.shape[0] > _ar.max_rows or x2.dtype != torch.bfloat16:
                return _orig(input_)
            out = _ar(x2.contiguous(), self.weight).view(*x.shape[:-1], self.weight.shape[0])
            return (out, None) if self.return_bias else out

        layer.forward = types.MethodType(fused_forward, layer)
        patched += 1
    LOGGER.info("FlexTensor fused TP all-reduce on %d row-parallel layers", patched)
    return patched
