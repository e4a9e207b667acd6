"""Wan2.2-14B-shape video DiT in plain PyTorch: the workload of the reference arm.

This module is what ``bench.py --impl reference`` offloads through the unmodified
reference runtime. It imports nothing from ``flextensor_b200``: every op is a stock
PyTorch call (``F.linear`` -> cuBLAS, ``F.layer_norm``, ``F.scaled_dot_product_attention``
-> cuDNN / flash SDPA), so no kernel of this repository runs on that arm.

The parameter tree (names, shapes, dtypes) matches ``flextensor_b200.models.wan.WanDiT``
so both arms offload the same bytes under the same budget:

* ``patch_embedding`` (64 -> d), ``text_embedding_{1,2}`` (4096 -> d -> d, GELU between),
  ``time_embedding_{1,2}`` (256 -> d -> d, SiLU between), ``time_projection`` (d -> 6d);
* ``blocks.{i}``: ``scale_shift_table`` [1, 6, d]; ``attn1`` (self-attention: q/k/v/out
  projections, full-width RMSNorm on q and k, 3-D RoPE on q and k); ``norm2`` (affine
  LayerNorm); ``attn2`` (cross-attention to the text tokens, RMSNorm on q and k);
  ``ffn_in`` / ``ffn_out`` (GELU-tanh FFN); adaLN shift/scale/gate on the self-attention
  and the FFN branches;
* ``head_scale_shift`` [1, 2, d] and ``proj_out`` (d -> 64).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class WanShape:
    dim: int = 5120
    ffn_dim: int = 13824
    num_heads: int = 40
    num_layers: int = 40
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    in_channels: int = 16
    out_channels: int = 16
    patch: tuple = (1, 2, 2)
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


def _timestep_features(t: torch.Tensor, dim: int) -> torch.Tensor:
    """Sinusoidal features [cos | sin] at geometric frequencies 10000^(-i/half)."""
    half = dim // 2
    i = torch.arange(half, device=t.device, dtype=torch.float64)
    ang = t.double()[:, None] * torch.pow(10000.0, -i / half)[None]
    return torch.cat([ang.cos(), ang.sin()], dim=1).float()


def _rope_angles(grid, head_dim: int, device, theta: float = 10000.0):
    """Per-token rotation angles of the 3-D RoPE: the head_dim/2 rotated pairs are split over
    the frame, height and width axes as (c - 2*(c//3), c//3, c//3)."""
    c = head_dim // 2
    parts = (c - 2 * (c // 3), c // 3, c // 3)
    out = []
    for axis, (n, pairs) in enumerate(zip(grid, parts)):
        inv = theta ** (-torch.arange(pairs, dtype=torch.float64, device=device) * 2.0 / (2 * pairs))
        a = torch.arange(n, dtype=torch.float64, device=device)[:, None] * inv[None]
        shape = [1, 1, 1, pairs]
        shape[axis] = n
        out.append(a.view(shape).expand(grid[0], grid[1], grid[2], pairs))
    ang = torch.cat(out, dim=-1).reshape(-1, c)
    return ang.cos().float().contiguous(), ang.sin().float().contiguous()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved (even, odd) pairs of x [B, S, H, Dh] by per-token angles."""
    b, s, h, d = x.shape
    xf = x.float().view(b, s, h, d // 2, 2)
    c, sn = cos[None, :, None], sin[None, :, None]
    ev, od = xf[..., 0], xf[..., 1]
    return torch.stack((ev * c - od * sn, ev * sn + od * c), dim=-1).view(b, s, h, d).to(x.dtype)


class _RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


class _Attention(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.to_q = nn.Linear(dim, dim)
        self.to_k = nn.Linear(dim, dim)
        self.to_v = nn.Linear(dim, dim)
        self.to_out = nn.Linear(dim, dim)
        self.norm_q = _RMSNorm(dim, eps)
        self.norm_k = _RMSNorm(dim, eps)


def _sdpa(q, k, v):
    """q/k/v [B, S, H, Dh] -> [B, S, H*Dh] through PyTorch's fused attention."""
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return o.transpose(1, 2).flatten(2)


class Ulysses:
    """Sequence-parallel self-attention over a process group with NCCL all-to-alls (the scheme of
    the reference's LTX example, ``examples/ltx23/outpaint/context_parallel.py:628-686``): each
    rank holds 1/P of the tokens; q/k/v go sequence -> heads, attention runs over the full
    sequence on H/P heads, and the output comes back heads -> sequence."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def _a2a(self, x, scatter_dim, gather_dim):
        import torch.distributed as dist

        send = torch.stack(x.chunk(self.world, dim=scatter_dim)).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return torch.cat(recv.unbind(0), dim=gather_dim)

    def attention(self, q, k, v):
        """q/k/v [B, S/P, H, Dh] -> [B, S/P, H*Dh]."""
        qh, kh, vh = (self._a2a(t, 2, 1) for t in (q, k, v))
        o = F.scaled_dot_product_attention(qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2))
        return self._a2a(o.transpose(1, 2), 1, 2).flatten(2)

    def gather(self, y):
        import torch.distributed as dist

        parts = [torch.empty_like(y) for _ in range(self.world)]
        dist.all_gather(parts, y.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)


class WanTorchBlock(nn.Module):
    def __init__(self, cfg: WanShape):
        super().__init__()
        d = cfg.dim
        self.cfg = cfg
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, d) / d ** 0.5)
        self.attn1 = _Attention(d, cfg.eps)
        self.norm2 = nn.LayerNorm(d, eps=cfg.eps, elementwise_affine=True)
        self.attn2 = _Attention(d, cfg.eps)
        self.ffn_in = nn.Linear(d, cfg.ffn_dim)
        self.ffn_out = nn.Linear(cfg.ffn_dim, d)

    def forward(self, x, ctx, e, cos, sin, cp=None):
        cfg = self.cfg
        B, S, D = x.shape
        H, Dh = cfg.num_heads, cfg.head_dim
        m = self.scale_shift_table.float() + e                 # [B, 6, D]
        sh1, sc1, g1, sh3, sc3, g3 = m.unsqueeze(2).unbind(1)   # each [B, 1, D]
        a = self.attn1
        h = (F.layer_norm(x.float(), (D,), eps=cfg.eps) * (1 + sc1) + sh1).to(x.dtype)
        q = _rotate(a.norm_q(a.to_q(h)).view(B, S, H, Dh), cos, sin)
        k = _rotate(a.norm_k(a.to_k(h)).view(B, S, H, Dh), cos, sin)
        v = a.to_v(h).view(B, S, H, Dh)
        o = cp.attention(q, k, v) if cp is not None else _sdpa(q, k, v)
        x = (x.float() + a.to_out(o).float() * g1).to(x.dtype)
        a = self.attn2
        h = F.layer_norm(x.float(), (D,), self.norm2.weight.float(), self.norm2.bias.float(), cfg.eps).to(x.dtype)
        L = ctx.shape[1]
        q = a.norm_q(a.to_q(h)).view(B, S, H, Dh)
        k = a.norm_k(a.to_k(ctx)).view(B, L, H, Dh)
        v = a.to_v(ctx).view(B, L, H, Dh)
        x = x + a.to_out(_sdpa(q, k, v))
        h = (F.layer_norm(x.float(), (D,), eps=cfg.eps) * (1 + sc3) + sh3).to(x.dtype)
        y = self.ffn_out(F.gelu(self.ffn_in(h), approximate="tanh"))
        return (x.float() + y.float() * g3).to(x.dtype)


class WanTorchDiT(nn.Module):
    def __init__(self, cfg: WanShape):
        super().__init__()
        self.cfg = cfg
        d = cfg.dim
        pf, ph, pw = cfg.patch
        self.patch_embedding = nn.Linear(cfg.in_channels * pf * ph * pw, d)
        self.text_embedding_1 = nn.Linear(cfg.text_dim, d)
        self.text_embedding_2 = nn.Linear(d, d)
        self.time_embedding_1 = nn.Linear(cfg.freq_dim, d)
        self.time_embedding_2 = nn.Linear(d, d)
        self.time_projection = nn.Linear(d, 6 * d)
        self.blocks = nn.ModuleList([WanTorchBlock(cfg) for _ in range(cfg.num_layers)])
        self.head_scale_shift = nn.Parameter(torch.randn(1, 2, d) / d ** 0.5)
        self.proj_out = nn.Linear(d, cfg.out_channels * pf * ph * pw)
        self._angles = {}

    def forward(self, latent, timestep, context, cp: Ulysses | None = None):
        """``cp``: sequence parallelism over a group -- this rank runs the blocks on its 1/P of
        the tokens (Ulysses self-attention) and the output is all-gathered after the head."""
        cfg = self.cfg
        dt = self.patch_embedding.weight.dtype
        B, C, Fr, Hh, Ww = latent.shape
        pf, ph, pw = cfg.patch
        grid = (Fr // pf, Hh // ph, Ww // pw)
        x = latent.to(dt).view(B, C, grid[0], pf, grid[1], ph, grid[2], pw)
        x = x.permute(0, 2, 4, 6, 1, 3, 5, 7).reshape(B, -1, C * pf * ph * pw)
        rows = None
        if cp is not None:
            shard = x.shape[1] // cp.world
            if shard * cp.world != x.shape[1]:
                raise ValueError(f"{x.shape[1]} tokens do not split over {cp.world} ranks")
            rows = slice(cp.rank * shard, (cp.rank + 1) * shard)
            x = x[:, rows].contiguous()
        x = self.patch_embedding(x)
        t = _timestep_features(timestep, cfg.freq_dim).to(dt)
        temb = self.time_embedding_2(F.silu(self.time_embedding_1(t)))
        e = self.time_projection(F.silu(temb)).float().view(-1, 6, cfg.dim)
        ctx = self.text_embedding_2(F.gelu(self.text_embedding_1(context.to(dt)), approximate="tanh"))
        key = (grid, str(x.device))
        if key not in self._angles:
            self._angles[key] = _rope_angles(grid, cfg.head_dim, x.device)
        cos, sin = self._angles[key]
        if rows is not None:
            cos, sin = cos[rows].contiguous(), sin[rows].contiguous()
        for blk in self.blocks:
            x = blk(x, ctx, e, cos, sin, cp) if cp is not None else blk(x, ctx, e, cos, sin)
        mod = self.head_scale_shift.float() + temb.float()[:, None]
        h = (F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + mod[:, 1:2]) + mod[:, 0:1]).to(dt)
        y = self.proj_out(h)
        if cp is not None:
            y = cp.gather(y)
        C = cfg.out_channels
        y = y.view(B, grid[0], grid[1], grid[2], C, pf, ph, pw).permute(0, 4, 1, 5, 2, 6, 3, 7)
        return y.reshape(B, C, grid[0] * pf, grid[1] * ph, grid[2] * pw)


def init_params_(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Seeded N(0, std) init in place on the parameters' device; norm weights set to one."""
    g = torch.Generator(device=next(model.parameters()).device)
    g.manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith(("norm_q.weight", "norm_k.weight", "norm2.weight")):
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)
