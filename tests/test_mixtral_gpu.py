"""Mixtral-shape MoE decoder on one GPU: native path (fused GEMMs incl. SwiGLU, attention,
RoPE) against the PyTorch path with the same weights."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.models.mixtral import MixtralModel, init_mixtral_params_, tiny_mixtral  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)


def test_mixtral_fused_matches_torch():
    cfg = tiny_mixtral()
    m = MixtralModel(cfg).to(DEV)
    init_mixtral_params_(m, seed=0)
    m = m.to(torch.bfloat16)
    tokens = torch.randint(0, cfg.vocab, (2, 128), device=DEV, generator=torch.Generator(device=DEV).manual_seed(2))
    with torch.no_grad():
        a = m(tokens).float()
        m.impl = "torch"
        b = m(tokens).float()
    assert native.device_error(reset=True) == 0
    assert float((a - b).abs().max() / b.abs().max()) < 6e-2


def test_mixtral_kv_cache_decode_matches_recompute():
    """Prefill + decode steps through the KV cache (split-KV decode kernel, GQA 2:1) against a
    full recompute of the growing sequence."""
    cfg = tiny_mixtral(dim=512, n_heads=4, n_kv_heads=2)
    m = MixtralModel(cfg).to(DEV)
    init_mixtral_params_(m, seed=3)
    m = m.to(torch.bfloat16)
    B, S, new = 2, 96, 4
    tokens = torch.randint(0, cfg.vocab, (B, S), device=DEV, generator=torch.Generator(device=DEV).manual_seed(5))
    with torch.no_grad():
        cache = m.new_cache(B, S + new)
        logits = m.prefill(tokens, cache)
        seq = tokens
        for i in range(new):
            ref = m(seq).float()
            assert float((logits.float() - ref).abs().max() / ref.abs().max()) < 3e-2, f"step {i}"
            nxt = logits.argmax(-1)
            seq = torch.cat([seq, nxt[:, None]], dim=1)
            logits = m.decode_step(nxt, cache, S + i)
    assert native.device_error(reset=True) == 0
    assert m.generate(tokens, 3).shape == (B, 3)
