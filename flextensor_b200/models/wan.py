"""Wan2.2-14B-shape video DiT denoiser (text-to-video transformer), random-init capable.

Architecture (the shapes the benchmark config names): patch embedding
(Conv3d k=s=(1,2,2) == Linear over 64-value patches), sinusoidal timestep
embedding -> MLP -> 6-way adaLN modulation, text embedding MLP (4096 -> d),
``num_layers`` blocks of [adaLN-modulated self-attention with full-width
RMSNorm on q/k and 3-D RoPE, LayerNorm'd cross-attention to the text tokens,
adaLN-modulated GELU(tanh) FFN, gated residuals], and a modulated output head.

Two compute paths share one parameter tree (identical ``state_dict``):

* ``impl="fused"`` -- the B200 path: every projection is the tcgen05 GEMM with
  its epilogue fused (bias, GELU, ``x + gate * y`` written in place), norms are
  single-pass row kernels, q/k RMSNorm and RoPE are one kernel, attention is
  the tcgen05 flash-attention kernel.
* ``impl="torch"`` -- plain PyTorch (``F.linear``, ``F.layer_norm``, SDPA): the
  numerics oracle and the workload the reference runtime is benchmarked on.

Every ``WanBlock`` is an offload unit (``include_patterns=["blocks.*"]``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class WanConfig:
    dim: int = 5120
    ffn_dim: int = 13824
    num_heads: int = 40
    num_layers: int = 40
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    in_channels: int = 16
    out_channels: int = 16
    patch: tuple[int, int, int] = (1, 2, 2)
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


WAN_14B = WanConfig()


def tiny_config(**kw) -> WanConfig:
    base = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=128, text_len=32, freq_dim=64)
    base.update(kw)
    return WanConfig(**base)


# ----------------------------------------------------------------------------- helpers


def sinusoidal(t: torch.Tensor, dim: int) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float64) / half)
    ang = t.double()[:, None] * freqs[None]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1).float()


def rope_tables(grid: tuple[int, int, int], head_dim: int, device, theta: float = 10000.0):
    """cos/sin ``[F*H*W, head_dim/2]`` for Wan's 3-D RoPE (pairs split t/h/w = c-2(c//3), c//3, c//3)."""
    c = head_dim // 2
    splits = [c - 2 * (c // 3), c // 3, c // 3]
    f, h, w = grid
    axes = []
    for n, pairs in zip((f, h, w), splits):
        d = 2 * pairs
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=device) / d))
        axes.append(torch.outer(torch.arange(n, dtype=torch.float64, device=device), inv))
    ang = torch.cat([
        axes[0][:, None, None, :].expand(f, h, w, splits[0]),
        axes[1][None, :, None, :].expand(f, h, w, splits[1]),
        axes[2][None, None, :, :].expand(f, h, w, splits[2]),
    ], dim=-1).reshape(f * h * w, c)
    return torch.cos(ang).float().contiguous(), torch.sin(ang).float().contiguous()


def apply_rope_torch(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x ``[B, S, H, Dh]`` (fp32), interleaved pairs rotated by per-position angles."""
    b, s, h, d = x.shape
    xr = x.view(b, s, h, d // 2, 2)
    re, im = xr[..., 0], xr[..., 1]
    c, sn = cos[None, :, None, :], sin[None, :, None, :]
    return torch.stack([re * c - im * sn, re * sn + im * c], dim=-1).view(b, s, h, d)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):  # torch path
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


class Attention(nn.Module):
    def __init__(self, dim: int, heads: int, eps: float, kv_dim: int | None = None):
        super().__init__()
        kv_dim = kv_dim or dim
        self.heads = heads
        self.to_q = nn.Linear(dim, dim)
        self.to_k = nn.Linear(kv_dim, dim)
        self.to_v = nn.Linear(kv_dim, dim)
        self.to_out = nn.Linear(dim, dim)
        self.norm_q = RMSNorm(dim, eps)
        self.norm_k = RMSNorm(dim, eps)


class WanBlock(nn.Module):
    def __init__(self, cfg: WanConfig, impl: str = "fused"):
        super().__init__()
        self.cfg = cfg
        self.impl = impl
        d = cfg.dim
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, d) / d ** 0.5)
        self.attn1 = Attention(d, cfg.num_heads, cfg.eps)
        self.norm2 = nn.LayerNorm(d, eps=cfg.eps, elementwise_affine=True)
        self.attn2 = Attention(d, cfg.num_heads, cfg.eps)
        self.ffn_in = nn.Linear(d, cfg.ffn_dim)
        self.ffn_out = nn.Linear(cfg.ffn_dim, d)

    # ------------------------------------------------------------------ fused B200 path
    def _forward_fused(self, x, ctx, e, rope, seq_len, cp=None):
        from flextensor_b200 import ops

        cfg = self.cfg
        B = x.shape[0]
        H, Dh = cfg.num_heads, cfg.head_dim
        x2 = x.view(-1, cfg.dim)
        mods = (self.scale_shift_table.float() + e).contiguous()        # [B, 6, D] fp32
        shift1, scale1, gate1 = mods[:, 0], mods[:, 1], mods[:, 2]
        shift3, scale3, gate3 = mods[:, 3], mods[:, 4], mods[:, 5]
        cos, sin = rope
        a1 = self.attn1
        h = ops.layernorm_modulate(x2, scale1, shift1, mod_rows=seq_len, eps=cfg.eps)
        q = ops.linear(h, a1.to_q.weight, a1.to_q.bias)
        ops.qk_rmsnorm_rope(q, a1.norm_q.weight, cos, sin, Dh, seq_len, eps=cfg.eps, out=q)
        if cp is not None:
            # context parallel: K/V rows go straight into this rank's rows of the shared
            # full-sequence buffer; the attention kernel gathers the other ranks' rows itself
            k, v = cp.begin()
            ops.linear(h, a1.to_k.weight, a1.to_k.bias, out=k)
            ops.linear(h, a1.to_v.weight, a1.to_v.bias, out=v)
            ops.qk_rmsnorm_rope(k, a1.norm_k.weight, cos, sin, Dh, seq_len, eps=cfg.eps, out=k)
            cp.publish()
            o = cp.attention(q.view(B, seq_len, H, Dh))
        else:
            k = ops.linear(h, a1.to_k.weight, a1.to_k.bias)
            v = ops.linear(h, a1.to_v.weight, a1.to_v.bias)
            ops.qk_rmsnorm_rope(k, a1.norm_k.weight, cos, sin, Dh, seq_len, eps=cfg.eps, out=k)
            o = ops.attention(q.view(B, seq_len, H, Dh), k.view(B, seq_len, H, Dh), v.view(B, seq_len, H, Dh))
        ops.linear(o.view(-1, cfg.dim), a1.to_out.weight, a1.to_out.bias, epi="gate_res", residual=x2,
                   gate=gate1, gate_rows=seq_len, out=x2)
        # cross attention (LayerNorm with affine, no modulation)
        a2 = self.attn2
        ops.layernorm_modulate(x2, weight=self.norm2.weight, bias=self.norm2.bias, eps=cfg.eps, out=h)
        q = ops.linear(h, a2.to_q.weight, a2.to_q.bias, out=q)
        ops.rmsnorm(q, a2.norm_q.weight, eps=cfg.eps, out=q)
        c2 = ctx.reshape(-1, cfg.dim)
        kc = ops.linear(c2, a2.to_k.weight, a2.to_k.bias)
        ops.rmsnorm(kc, a2.norm_k.weight, eps=cfg.eps, out=kc)
        vc = ops.linear(c2, a2.to_v.weight, a2.to_v.bias)
        L = ctx.shape[1]
        o = ops.attention(q.view(B, seq_len, H, Dh), kc.view(B, L, H, Dh), vc.view(B, L, H, Dh), out=o)
        ops.linear(o.view(-1, cfg.dim), a2.to_out.weight, a2.to_out.bias, epi="res", residual=x2, out=x2)
        # FFN
        ops.layernorm_modulate(x2, scale3, shift3, mod_rows=seq_len, eps=cfg.eps, out=h)
        f = ops.linear(h, self.ffn_in.weight, self.ffn_in.bias, epi="gelu")
        ops.linear(f, self.ffn_out.weight, self.ffn_out.bias, epi="gate_res", residual=x2, gate=gate3,
                   gate_rows=seq_len, out=x2)
        return x

    # ------------------------------------------------------------------ plain torch path
    def _forward_torch(self, x, ctx, e, rope, seq_len, cp=None):
        cfg = self.cfg
        B = x.shape[0]
        H, Dh = cfg.num_heads, cfg.head_dim
        mods = (self.scale_shift_table.float() + e)
        shift1, scale1, gate1, shift3, scale3, gate3 = (mods[:, i:i + 1] for i in range(6))
        cos, sin = rope
        a1 = self.attn1
        h = (F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + scale1) + shift1).to(x.dtype)
        q = a1.norm_q(F.linear(h, a1.to_q.weight, a1.to_q.bias))
        k = a1.norm_k(F.linear(h, a1.to_k.weight, a1.to_k.bias))
        v = F.linear(h, a1.to_v.weight, a1.to_v.bias)
        q = apply_rope_torch(q.view(B, seq_len, H, Dh).float(), cos, sin).to(x.dtype)
        k = apply_rope_torch(k.view(B, seq_len, H, Dh).float(), cos, sin).to(x.dtype)
        sdpa = lambda qq, kk, vv: F.scaled_dot_product_attention(  # noqa: E731
            qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2)).transpose(1, 2)
        if cp is not None:  # Ulysses all-to-all (NCCL baseline)
            o = cp(q, k, v.view(B, seq_len, H, Dh), sdpa)
        else:
            o = sdpa(q, k, v.view(B, seq_len, H, Dh))
        y = F.linear(o.reshape(B, seq_len, cfg.dim), a1.to_out.weight, a1.to_out.bias)
        x = (x.float() + y.float() * gate1).to(x.dtype)
        a2 = self.attn2
        h = F.layer_norm(x.float(), (cfg.dim,), self.norm2.weight.float(), self.norm2.bias.float(),
                         eps=cfg.eps).to(x.dtype)
        q = a2.norm_q(F.linear(h, a2.to_q.weight, a2.to_q.bias)).view(B, seq_len, H, Dh)
        L = ctx.shape[1]
        k = a2.norm_k(F.linear(ctx, a2.to_k.weight, a2.to_k.bias)).view(B, L, H, Dh)
        v = F.linear(ctx, a2.to_v.weight, a2.to_v.bias).view(B, L, H, Dh)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
        x = x + F.linear(o.reshape(B, seq_len, cfg.dim), a2.to_out.weight, a2.to_out.bias)
        h = (F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + scale3) + shift3).to(x.dtype)
        f = F.gelu(F.linear(h, self.ffn_in.weight, self.ffn_in.bias), approximate="tanh")
        y = F.linear(f, self.ffn_out.weight, self.ffn_out.bias)
        return (x.float() + y.float() * gate3).to(x.dtype)

    def forward(self, x, ctx, e, rope_cos, rope_sin, cp=None):
        seq_len = x.shape[1]
        if self.impl == "fused":
            return self._forward_fused(x, ctx, e, (rope_cos, rope_sin), seq_len, cp)
        return self._forward_torch(x, ctx, e, (rope_cos, rope_sin), seq_len, cp)


class WanDiT(nn.Module):
    def __init__(self, cfg: WanConfig = WAN_14B, impl: str = "fused"):
        super().__init__()
        self.cfg = cfg
        self.impl = impl
        d = cfg.dim
        pf, ph, pw = cfg.patch
        self.patch_embedding = nn.Linear(cfg.in_channels * pf * ph * pw, d)
        self.text_embedding_1 = nn.Linear(cfg.text_dim, d)
        self.text_embedding_2 = nn.Linear(d, d)
        self.time_embedding_1 = nn.Linear(cfg.freq_dim, d)
        self.time_embedding_2 = nn.Linear(d, d)
        self.time_projection = nn.Linear(d, 6 * d)
        self.blocks = nn.ModuleList([WanBlock(cfg, impl) for _ in range(cfg.num_layers)])
        self.head_scale_shift = nn.Parameter(torch.randn(1, 2, d) / d ** 0.5)
        self.proj_out = nn.Linear(d, cfg.out_channels * pf * ph * pw)
        self._rope_cache: dict = {}

    def set_impl(self, impl: str) -> None:
        self.impl = impl
        for b in self.blocks:
            b.impl = impl

    def _lin(self, x, layer: nn.Linear, epi: str = "bias"):
        if self.impl == "fused" and x.is_cuda:
            from flextensor_b200 import ops

            return ops.linear(x.contiguous(), layer.weight, layer.bias, epi=epi)
        y = F.linear(x, layer.weight, layer.bias)
        return F.gelu(y, approximate="tanh") if epi == "gelu" else y

    def patchify(self, latent: torch.Tensor):
        B, C, Fr, Hh, Ww = latent.shape
        pf, ph, pw = self.cfg.patch
        f, h, w = Fr // pf, Hh // ph, Ww // pw
        x = latent.view(B, C, f, pf, h, ph, w, pw).permute(0, 2, 4, 6, 1, 3, 5, 7)
        return x.reshape(B, f * h * w, C * pf * ph * pw), (f, h, w)

    def unpatchify(self, x: torch.Tensor, grid):
        B = x.shape[0]
        f, h, w = grid
        pf, ph, pw = self.cfg.patch
        C = self.cfg.out_channels
        x = x.view(B, f, h, w, C, pf, ph, pw).permute(0, 4, 1, 5, 2, 6, 3, 7)
        return x.reshape(B, C, f * pf, h * ph, w * pw)

    def rope(self, grid, device):
        key = (grid, str(device))
        t = self._rope_cache.get(key)
        if t is None:
            t = rope_tables(grid, self.cfg.head_dim, device)
            self._rope_cache[key] = t
        return t

    def condition(self, timestep: torch.Tensor, context: torch.Tensor):
        """Time embedding ``temb`` [B, dim], the six adaLN vectors ``e`` [B, 6, dim] (fp32) and
        the projected text context ``ctx`` [B, L, dim]."""
        cfg = self.cfg
        dt = self.patch_embedding.weight.dtype
        t = sinusoidal(timestep, cfg.freq_dim).to(dt)
        temb = self._lin(F.silu(self._lin(t, self.time_embedding_1).float()).to(dt), self.time_embedding_2)
        e = self._lin(F.silu(temb.float()).to(dt), self.time_projection).float().view(-1, 6, cfg.dim)
        ctx = self._lin(context.to(dt), self.text_embedding_1, "gelu")
        ctx = self._lin(ctx, self.text_embedding_2).contiguous()
        return temb, e, ctx

    def head(self, x: torch.Tensor, temb: torch.Tensor) -> torch.Tensor:
        """Modulated final LayerNorm and the output projection (patch tokens, not yet unpatchified)."""
        cfg = self.cfg
        mod = self.head_scale_shift.float() + temb.float()[:, None]
        shift, scale = mod[:, 0:1], mod[:, 1:2]
        h = (F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + scale) + shift).to(self.patch_embedding.weight.dtype)
        return self._lin(h, self.proj_out)

    def forward(self, latent: torch.Tensor, timestep: torch.Tensor, context: torch.Tensor, cp=None) -> torch.Tensor:
        """``cp``: a :class:`~flextensor_b200.parallel.cp.ContextParallel` (fused path) or
        :class:`~flextensor_b200.parallel.cp.UlyssesAttention` (torch path); each rank then runs
        the blocks on its 1/N of the tokens and the output is gathered after the head."""
        cfg = self.cfg
        dt = self.patch_embedding.weight.dtype
        x, grid = self.patchify(latent.to(dt))
        rank_rows = None
        if cp is not None:
            import torch.distributed as dist

            world = dist.get_world_size(cp.group)
            shard = x.shape[1] // world
            if shard * world != x.shape[1]:
                raise ValueError(f"{x.shape[1]} tokens do not split evenly over {world} ranks")
            rank_rows = slice(dist.get_rank(cp.group) * shard, (dist.get_rank(cp.group) + 1) * shard)
            x = x[:, rank_rows].contiguous()
        x = self._lin(x, self.patch_embedding, "bias").contiguous()
        temb, e, ctx = self.condition(timestep, context)
        cos, sin = self.rope(grid, x.device)
        if rank_rows is not None:
            cos, sin = cos[rank_rows].contiguous(), sin[rank_rows].contiguous()
        for blk in self.blocks:
            x = blk(x, ctx, e, cos, sin, cp=cp) if cp is not None else blk(x, ctx, e, cos, sin)
        y = self.head(x, temb)
        if cp is not None:
            y = _gather_seq(y, cp.group)
        return self.unpatchify(y, grid)


def _gather_seq(y: torch.Tensor, group) -> torch.Tensor:
    import torch.distributed as dist

    parts = [torch.empty_like(y) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, y.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def init_wan_params_(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Deterministic random init in place on whatever device the parameters live on."""
    g = torch.Generator(device=next(model.parameters()).device)
    g.manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm_q.weight") or name.endswith("norm_k.weight") or name.endswith("norm2.weight"):
                p.fill_(1.0)
            elif p.dim() == 1:
                p.normal_(0.0, std, generator=g)
            else:
                p.normal_(0.0, std, generator=g)
