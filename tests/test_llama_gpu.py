"""Llama-shape decoder on one GPU: the native path (tcgen05 GEMMs incl. the SwiGLU epilogue,
RoPE kernel, causal GQA attention) against the PyTorch path with the same weights."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.models.llama import LlamaModel, init_llama_params_, tiny_llama  # noqa: E402
from flextensor_b200.ops import api as ops  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)


def test_linear_swiglu():
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(300, 256, device=DEV, generator=g).bfloat16()
    w = (torch.randn(2 * 384, 256, device=DEV, generator=g) / 16).bfloat16()
    y = ops.linear_swiglu(x, w)
    r = x.float() @ w.float().t()
    ref = torch.nn.functional.silu(r[:, 0::2]) * r[:, 1::2]
    assert float((y.float() - ref).abs().max() / ref.abs().max()) < 2e-2


def test_rope_only_kernel():
    from flextensor_b200.models.llama import _rope_torch, rope_tables_1d

    g = torch.Generator(device=DEV).manual_seed(1)
    B, S, H, D = 2, 64, 3, 128
    x = torch.randn(B * S, H * D, device=DEV, generator=g).bfloat16()
    cos, sin = rope_tables_1d(S, D, 5e5, DEV)
    y = ops.rope(x, cos, sin, D, S)
    ref = _rope_torch(x.view(B, S, H, D).float(), cos, sin).view(B * S, H * D)
    assert float((y.float() - ref).abs().max()) < 2e-2


def test_llama_fused_matches_torch():
    cfg = tiny_llama(n_layers=2)
    m = LlamaModel(cfg, impl="fused").to(DEV)
    init_llama_params_(m, seed=0)
    m = m.to(torch.bfloat16)
    tokens = torch.randint(0, cfg.vocab, (2, 256), device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
    with torch.no_grad():
        a = m(tokens).float()
        m.impl = "torch"
        b = m(tokens).float()
    assert native.device_error(reset=True) == 0
    assert float((a - b).abs().max() / b.abs().max()) < 5e-2


def test_kv_cache_decode_matches_recompute():
    cfg = tiny_llama(n_layers=2)
    m = LlamaModel(cfg, impl="fused").to(DEV)
    init_llama_params_(m, seed=1)
    m = m.to(torch.bfloat16)
    B, S, new = 3, 100, 5
    tokens = torch.randint(0, cfg.vocab, (B, S), device=DEV, generator=torch.Generator(device=DEV).manual_seed(4))
    with torch.no_grad():
        cache = m.new_cache(B, S + new)
        logits = m.prefill(tokens, cache)
        seq = tokens
        for i in range(new):
            ref = m(seq).float()  # recompute over the whole sequence
            assert float((logits.float() - ref).abs().max() / ref.abs().max()) < 3e-2, f"step {i}"
            nxt = logits.argmax(-1)
            seq = torch.cat([seq, nxt[:, None]], dim=1)
            logits = m.decode_step(nxt, cache, S + i)
    assert native.device_error(reset=True) == 0
    out = m.generate(tokens, 4)
    assert out.shape == (B, 4)
