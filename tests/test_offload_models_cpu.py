"""Offload validation on decoder models (CPU device, PyTorch path): streaming the decoder
layers through the runtime must give bit-identical outputs to the resident model, for a dense
Llama-shape decoder and a sparse-MoE Mixtral-shape decoder."""

import torch

import flextensor_b200 as ft
from flextensor_b200.planner import NthLayerStrategy


def _cfg():
    return ft.OffloadConfig(pinned_memory=False, include_patterns=["layers.*"], profiling_iters=1, num_blocks=2,
                            min_blocks=2, load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))


def test_llama_layers_streamed_bitwise():
    from flextensor_b200.models.llama import LlamaModel, init_llama_params_, tiny_llama

    cfg = tiny_llama(n_layers=3)
    m = LlamaModel(cfg, impl="torch")
    init_llama_params_(m, seed=0)
    tokens = torch.randint(0, cfg.vocab, (2, 32), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        want = m(tokens)
    mm = ft.offload(m, _cfg())
    om = ft.get_offload_manager()
    with torch.no_grad():
        for _ in range(om.iters_before_inference + 2):
            assert torch.equal(mm(tokens), want)
    assert om.phase.value == "inference"
    assert om.get_tensor_manager().loader.plan.host_blocks, "layers were not streamed"


def test_mixtral_layers_streamed_bitwise():
    from flextensor_b200.models.mixtral import MixtralModel, init_mixtral_params_, tiny_mixtral

    cfg = tiny_mixtral(n_layers=2)
    m = MixtralModel(cfg, impl="torch")
    init_mixtral_params_(m, seed=0)
    tokens = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = m(tokens)
    mm = ft.offload(m, _cfg())
    om = ft.get_offload_manager()
    with torch.no_grad():
        for _ in range(om.iters_before_inference + 2):
            assert torch.equal(mm(tokens), want)
