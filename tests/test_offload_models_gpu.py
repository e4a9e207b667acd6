"""Offload validation on the GPU for the decoder models' native paths: streamed decoder layers
must give bit-identical outputs to the resident model (dense Llama-shape and sparse Mixtral-shape,
an odd number of layers so the wrapping schedule needs a third slot)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import flextensor_b200 as ft  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402
from flextensor_b200.planner import NthLayerStrategy  # noqa: E402

DEV = torch.device("cuda", 0)


def _cfg():
    return ft.OffloadConfig(include_patterns=["layers.*"], profiling_iters=1, num_blocks=2, min_blocks=2,
                            skip_discovery=True,
                            load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))


@pytest.mark.parametrize("family", ["llama", "mixtral"])
def test_streamed_decoder_bitwise(family):
    if family == "llama":
        from flextensor_b200.models.llama import LlamaModel as M, init_llama_params_ as init, tiny_llama as tiny
        cfg = tiny(n_layers=3)
    else:
        from flextensor_b200.models.mixtral import MixtralModel as M, init_mixtral_params_ as init, tiny_mixtral as tiny
        cfg = tiny(n_layers=3)
    ref = M(cfg).to(DEV)
    init(ref, seed=0)
    ref = ref.to(torch.bfloat16)
    tokens = torch.randint(0, cfg.vocab, (2, 64), device=DEV, generator=torch.Generator(device=DEV).manual_seed(0))
    with torch.no_grad():
        want = ref(tokens)
    m = M(cfg).to(DEV).to(torch.bfloat16)
    m.load_state_dict(ref.state_dict())
    mm = ft.offload(m, _cfg())
    om = ft.get_offload_manager()
    with torch.no_grad():
        for _ in range(om.iters_before_inference + 3):
            assert torch.equal(mm(tokens), want)
    assert om.phase.value == "inference"
    assert len(set(om.get_tensor_manager().loader.plan.transfer_slot.values())) == 3
    assert native.device_error(reset=True) == 0
