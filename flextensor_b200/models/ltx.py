"""LTX-style video DiT shape for the context-parallel configuration.

48 blocks, d=4096, 32 heads (head_dim 128), FFN 16384, cross-attention to 256 text tokens of
dim 4096; 128-channel latents patchified 1x1x1 (1280x704 @ 361 frames -> 46x22x40 = 40,480
tokens). The block is the same adaLN-modulated self-attention / cross-attention / GELU-FFN
block as the Wan model (qk RMSNorm, 3-D RoPE, gated residuals), so both DiT families share
the fused kernels, the offload units (``blocks.*``) and the context-parallel path
(``WanDiT.forward(..., cp=ContextParallel(...))``).
"""

from __future__ import annotations

from flextensor_b200.models.wan import WanConfig, WanDiT, init_wan_params_

LTX_CP_CONFIG = WanConfig(dim=4096, ffn_dim=16384, num_heads=32, num_layers=48, text_dim=4096, text_len=256,
                          freq_dim=256, in_channels=128, out_channels=128, patch=(1, 1, 1))
LTX_LATENT_GRID = (46, 22, 40)   # frames, height, width after the VAE: 40,480 tokens


def LTXDiT(cfg: WanConfig = LTX_CP_CONFIG, impl: str = "fused") -> WanDiT:  # noqa: N802 - model factory
    return WanDiT(cfg, impl=impl)


__all__ = ["LTX_CP_CONFIG", "LTX_LATENT_GRID", "LTXDiT", "init_wan_params_"]
