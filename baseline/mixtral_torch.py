"""Mixtral-8x22B-shape MoE decoder layers, one expert-parallel rank, in plain PyTorch + NCCL: the
workload of the reference arm of ``benchmarks/e2e_mixtral_ep.py``.

Each rank runs attention for its own sequences (data parallel) and owns ``E / world`` experts of
every layer. MoE: top-2 of the router logits, softmax over the two, rows sorted by expert, NCCL
``all_to_all_single`` to the experts' owners, SwiGLU expert FFNs with ``F.linear`` (cuBLAS), and
a second all-to-all back, then the router-weighted sum. Attention: RMSNorm, GQA with SDPA, RoPE,
KV cache for decode. Nothing here imports ``flextensor_b200``.

Parameter names and shapes match ``flextensor_b200.models.mixtral.MixtralModel``'s layers at the
same rank (``attn`` = the Llama attention block with a 1-wide unused FFN, ``router``,
``experts.{j}.w_gate_up`` with interleaved gate/up rows, ``experts.{j}.w_down``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from llama_torch import _rms, _rotate


@dataclass
class MixtralShape:
    dim: int = 6144
    n_layers: int = 56
    n_heads: int = 48
    n_kv_heads: int = 8
    ffn_dim: int = 16384
    rope_theta: float = 1000000.0
    eps: float = 1e-5
    n_experts: int = 8
    topk: int = 2

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads


class _Attn(nn.Module):
    def __init__(self, cfg: MixtralShape):
        super().__init__()
        D = cfg.head_dim
        self.attn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.wqkv = nn.Parameter(torch.empty((cfg.n_heads + 2 * cfg.n_kv_heads) * D, cfg.dim))
        self.wo = nn.Parameter(torch.empty(cfg.dim, cfg.n_heads * D))
        self.ffn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.w_gate_up = nn.Parameter(torch.empty(2, cfg.dim))   # unused (shape parity)
        self.w_down = nn.Parameter(torch.empty(cfg.dim, 1))      # unused (shape parity)


class _Expert(nn.Module):
    def __init__(self, d: int, f: int):
        super().__init__()
        self.w_gate_up = nn.Parameter(torch.empty(2 * f, d))
        self.w_down = nn.Parameter(torch.empty(d, f))


class MixtralEPLayer(nn.Module):
    def __init__(self, cfg: MixtralShape, rank: int, world: int):
        super().__init__()
        self.cfg, self.rank, self.world = cfg, rank, world
        self.el = cfg.n_experts // world
        self.attn = _Attn(cfg)
        self.ffn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.router = nn.Parameter(torch.empty(cfg.n_experts, cfg.dim))
        self.experts = nn.ModuleList([_Expert(cfg.dim, cfg.ffn_dim) for _ in range(self.el)])

    def _attention(self, x, B, S, cos, sin, cache, pos):
        cfg, a, D = self.cfg, self.attn, self.cfg.head_dim
        h = _rms(x, a.attn_norm, cfg.eps)
        q, k, v = F.linear(h, a.wqkv).split([cfg.n_heads * D, cfg.n_kv_heads * D, cfg.n_kv_heads * D], dim=-1)
        q = _rotate(q.reshape(B, S, cfg.n_heads, D), cos, sin)
        k = _rotate(k.reshape(B, S, cfg.n_kv_heads, D), cos, sin)
        v = v.reshape(B, S, cfg.n_kv_heads, D)
        if cache is not None:
            cache[0][:, pos:pos + S].copy_(k)
            cache[1][:, pos:pos + S].copy_(v)
            if S == 1:
                k, v = cache[0][:, :pos + 1], cache[1][:, :pos + 1]
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=S > 1, enable_gqa=True)
        return x + F.linear(o.transpose(1, 2).reshape(B * S, -1), a.wo)

    def _moe(self, h, x):
        import torch.distributed as dist

        cfg, W = self.cfg, self.world
        logits = F.linear(h.float(), self.router.float())
        val, idx = torch.topk(logits, cfg.topk, dim=-1)
        wts = torch.softmax(val, dim=-1)
        T, k = idx.shape
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        send = h.index_select(0, order // k)
        counts = torch.bincount(flat, minlength=cfg.n_experts)
        if W > 1:
            per_rank = counts.view(W, self.el).sum(1)
            recv_counts = torch.empty_like(per_rank)
            dist.all_to_all_single(recv_counts, per_rank)
            sc, rc = per_rank.tolist(), recv_counts.tolist()
            recv = torch.empty(sum(rc), h.shape[1], dtype=h.dtype, device=h.device)
            dist.all_to_all_single(recv, send, rc, sc)
            parts = [torch.empty_like(counts) for _ in range(W)]
            dist.all_gather(parts, counts)
            cnt_all = torch.stack(parts)
            mine = cnt_all[:, self.rank * self.el:(self.rank + 1) * self.el]
        else:
            recv, mine = send, counts.view(1, -1)
        out = torch.empty_like(recv)
        start = 0
        for src in range(mine.shape[0]):
            for j in range(self.el):
                n = int(mine[src, j])
                if n:
                    ex = self.experts[j]
                    gu = F.linear(recv[start:start + n], ex.w_gate_up)
                    out[start:start + n] = F.linear(F.silu(gu[:, 0::2]) * gu[:, 1::2], ex.w_down)
                start += n
        if W > 1:
            back = torch.empty_like(send)
            dist.all_to_all_single(back, out, sc, rc)
        else:
            back = out
        pos = torch.empty_like(order)
        pos[order] = torch.arange(order.numel(), device=order.device)
        y = back.index_select(0, pos).view(T, k, -1)
        return (x.float() + (y.float() * wts.unsqueeze(-1)).sum(1)).to(x.dtype)

    def forward(self, x, B, S, cos, sin, cache=None, pos: int = 0):
        x = self._attention(x, B, S, cos, sin, cache, pos)
        return self._moe(_rms(x, self.ffn_norm, self.cfg.eps), x)


class MixtralEP(nn.Module):
    def __init__(self, cfg: MixtralShape, rank: int, world: int, layers: int | None = None):
        super().__init__()
        self.cfg = cfg
        self.layers = nn.ModuleList([MixtralEPLayer(cfg, rank, world) for _ in range(layers or cfg.n_layers)])

    def new_cache(self, batch: int, max_len: int, device):
        c = self.cfg
        return [(torch.empty(batch, max_len, c.n_kv_heads, c.head_dim, device=device, dtype=torch.bfloat16),
                 torch.empty(batch, max_len, c.n_kv_heads, c.head_dim, device=device, dtype=torch.bfloat16))
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
