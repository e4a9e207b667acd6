"""Integration helpers on CPU: a two-denoiser pipeline offloaded under two named managers,
profile save + reuse; vLLM default selector resolution."""

import pytest
import torch

import flextensor_b200 as ft
from flextensor_b200.contrib.diffusers import (
    offload_pipeline,
    offload_pipeline_from_profiles,
    release_pipeline,
    save_pipeline_profiles,
)
from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
from flextensor_b200.planner import NthLayerStrategy


class Pipe:
    def __init__(self):
        cfg = tiny_config(num_layers=2)
        self.transformer = WanDiT(cfg, impl="torch")
        self.transformer_2 = WanDiT(cfg, impl="torch")
        init_wan_params_(self.transformer, seed=1)
        init_wan_params_(self.transformer_2, seed=2)
        self.vae = torch.nn.Linear(4, 4)
        self.cfg = cfg

    @property
    def components(self):
        return {"transformer": self.transformer, "transformer_2": self.transformer_2, "vae": self.vae}

    def __call__(self, lat, ctx):
        t = torch.tensor([500.0])
        x = self.transformer(lat, t, ctx)
        return self.transformer_2(x, t * 0.5, ctx)


def _inputs(cfg):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(1, cfg.in_channels, 2, 8, 8, generator=g),
            torch.randn(1, cfg.text_len, cfg.text_dim, generator=g))


def _cfg():
    return ft.OffloadConfig(pinned_memory=False, include_patterns=["blocks.*"], profiling_iters=1, num_blocks=2,
                            min_blocks=2, load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))


def test_pipeline_two_managers_and_profile_reuse(tmp_path):
    ref = Pipe()
    lat, ctx = _inputs(ref.cfg)
    with torch.no_grad():
        want = ref(lat, ctx)
    pipe = Pipe()
    offload_pipeline(pipe, _cfg(), device="cpu")
    with torch.no_grad():
        for _ in range(4):
            assert torch.equal(pipe(lat, ctx), want)
    assert ft.get_offload_manager("transformer").phase.value == "inference"
    assert ft.get_offload_manager("transformer2").phase.value == "inference"
    save_pipeline_profiles(pipe, str(tmp_path))
    release_pipeline(pipe)
    pipe2 = Pipe()
    offload_pipeline_from_profiles(pipe2, str(tmp_path), _cfg(), device="cpu")
    assert ft.get_offload_manager("transformer").phase.value == "inference"
    with torch.no_grad():
        assert torch.equal(pipe2(lat, ctx), want)
    release_pipeline(pipe2)


def test_vllm_pattern_resolution():
    from flextensor_b200.contrib.vllm.patterns import (
        VLLM_DEFAULT_EXCLUDE_PATTERNS,
        VLLM_DEFAULT_INCLUDE_PATTERNS,
        resolve_vllm_patterns,
    )

    inc, exc = resolve_vllm_patterns(ft.OffloadConfig())
    assert inc == VLLM_DEFAULT_INCLUDE_PATTERNS and exc == VLLM_DEFAULT_EXCLUDE_PATTERNS
    inc, exc = resolve_vllm_patterns(ft.OffloadConfig(include_patterns=["model.layers.*"], exclude_patterns=[]))
    assert inc == ["model.layers.*"] and exc == []  # explicit empty excludes stay empty
