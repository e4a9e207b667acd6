"""Llama-3-shape decoder layers, one tensor-parallel rank's shard, in plain PyTorch + NCCL: the
workload of the reference arm of ``benchmarks/e2e_llama_tp.py``.

Megatron-style TP as vLLM runs it: q/k/v heads and FFN columns split over the ranks, the
residual stream replicated, one NCCL all-reduce after the attention output projection and one
after the FFN down projection. GEMMs are ``F.linear`` (cuBLAS), attention is SDPA with GQA, the
KV cache holds this rank's KV heads. Nothing here imports ``flextensor_b200``.

Parameter names and shapes match ``flextensor_b200.models.llama.LlamaLayer`` at the same split
(``wqkv`` stacks q, k, v rows; ``w_gate_up`` interleaves gate and up rows), so both arms offload
the same bytes under the same budget.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class LlamaShape:
    dim: int = 8192
    n_layers: int = 80
    n_heads: int = 64
    n_kv_heads: int = 8
    ffn_dim: int = 28672
    rope_theta: float = 500000.0
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads


def rope_cos_sin(n: int, head_dim: int, theta: float, device):
    inv = theta ** (-torch.arange(0, head_dim, 2, dtype=torch.float64, device=device) / head_dim)
    ang = torch.arange(n, dtype=torch.float64, device=device)[:, None] * inv[None]
    return ang.cos().float(), ang.sin().float()


def _rotate(x, cos, sin):
    """x [B, S, H, D]: rotate interleaved pairs by per-position angles cos/sin [S, D/2]."""
    b, s, h, d = x.shape
    xf = x.float().view(b, s, h, d // 2, 2)
    c, sn = cos[None, :, None], sin[None, :, None]
    return torch.stack((xf[..., 0] * c - xf[..., 1] * sn, xf[..., 0] * sn + xf[..., 1] * c), -1).view(
        b, s, h, d).to(x.dtype)


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class LlamaShardLayer(nn.Module):
    def __init__(self, cfg: LlamaShape, world: int):
        super().__init__()
        self.cfg, self.world = cfg, world
        self.hq, self.hk, self.f = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.ffn_dim // world
        D = cfg.head_dim
        self.attn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.wqkv = nn.Parameter(torch.empty((self.hq + 2 * self.hk) * D, cfg.dim))
        self.wo = nn.Parameter(torch.empty(cfg.dim, self.hq * D))
        self.ffn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.w_gate_up = nn.Parameter(torch.empty(2 * self.f, cfg.dim))
        self.w_down = nn.Parameter(torch.empty(cfg.dim, self.f))

    def _all_reduce(self, y):
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(y)
        return y

    def forward(self, x, B, S, cos, sin, cache=None, pos: int = 0):
        """x [B*S, dim] (replicated) -> same. ``cache`` = (k, v) [B, L, hk, D] of this rank."""
        cfg, D = self.cfg, self.cfg.head_dim
        h = _rms(x, self.attn_norm, cfg.eps)
        q, k, v = F.linear(h, self.wqkv).split([self.hq * D, self.hk * D, self.hk * D], dim=-1)
        q = _rotate(q.reshape(B, S, self.hq, D), cos, sin)
        k = _rotate(k.reshape(B, S, self.hk, D), cos, sin)
        v = v.reshape(B, S, self.hk, D)
        if cache is not None:
            cache[0][:, pos:pos + S].copy_(k)
            cache[1][:, pos:pos + S].copy_(v)
            if S == 1:
                k, v = cache[0][:, :pos + 1], cache[1][:, :pos + 1]
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=S > 1, enable_gqa=True)
        x = x + self._all_reduce(F.linear(o.transpose(1, 2).reshape(B * S, -1), self.wo))
        h = _rms(x, self.ffn_norm, cfg.eps)
        gu = F.linear(h, self.w_gate_up)
        return x + self._all_reduce(F.linear(F.silu(gu[:, 0::2]) * gu[:, 1::2], self.w_down))


class LlamaShard(nn.Module):
    def __init__(self, cfg: LlamaShape, world: int, layers: int | None = None):
        super().__init__()
        self.cfg, self.world = cfg, world
        self.layers = nn.ModuleList([LlamaShardLayer(cfg, world) for _ in range(layers or cfg.n_layers)])

    def new_cache(self, batch: int, max_len: int, device):
        hk = self.cfg.n_kv_heads // self.world
        return [(torch.empty(batch, max_len, hk, self.cfg.head_dim, device=device, dtype=torch.bfloat16),
                 torch.empty(batch, max_len, hk, self.cfg.head_dim, device=device, dtype=torch.bfloat16))
                for _ in self.layers]

    def forward(self, x, B, S, cos, sin, cache=None, pos: int = 0):
        for i, L in enumerate(self.layers):
            x = L(x, B, S, cos, sin, None if cache is None else cache[i], pos)
        return x


def init_params_(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    g = torch.Generator(device=next(model.parameters()).device)
    g.manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm"):
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)
