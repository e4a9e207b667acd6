"""Mixtral-8x22B-shape sparse-MoE decoder (GQA attention + top-2 of 8 SwiGLU experts).

Attention is the Llama block (``models/llama.py``, native kernels). The MoE feed-forward:
router logits -> top-2 -> softmax over the two; each expert is a SwiGLU FFN whose gate/up
rows are interleaved (one GEMM with the SwiGLU epilogue) followed by the down GEMM.

Three MoE paths share one parameter tree:

* single GPU (``ep=None``): per-expert gather -> fused GEMMs -> weighted scatter-add;
* expert parallel, fused (``ep=ExpertParallel``): each rank keeps its own tokens and owns
  ``E/world`` experts; dispatch / combine run inside the expert GEMM kernels over NVLink
  (``parallel/ep.py``, ``ops/csrc/moe_sm100.cu``);
* expert parallel, NCCL (``ep=NcclExpertParallel``): all-to-all around the same GEMMs.

``layers.*`` are the offload units: with expert parallelism a rank's unit holds only its own
experts' weights, which is what the runtime streams from host memory.
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from flextensor_b200.models.llama import LlamaConfig, LlamaLayer, _rms_torch, rope_tables_1d


@dataclass
class MixtralConfig(LlamaConfig):
    dim: int = 6144
    n_layers: int = 56
    n_heads: int = 48
    n_kv_heads: int = 8
    ffn_dim: int = 16384
    vocab: int = 32768
    rope_theta: float = 1000000.0
    n_experts: int = 8
    topk: int = 2


MIXTRAL_8X22B = MixtralConfig()


def tiny_mixtral(**kw) -> MixtralConfig:
    base = dict(dim=256, n_layers=2, n_heads=2, n_kv_heads=2, ffn_dim=256, vocab=512, n_experts=4, topk=2)
    base.update(kw)
    return MixtralConfig(**base)


class Expert(nn.Module):
    def __init__(self, d: int, f: int):
        super().__init__()
        self.w_gate_up = nn.Parameter(torch.empty(2 * f, d))
        self.w_down = nn.Parameter(torch.empty(d, f))


class MixtralLayer(nn.Module):
    def __init__(self, cfg: MixtralConfig, expert_ids: list[int] | None = None):
        super().__init__()
        self.cfg = cfg
        self.attn = LlamaLayer(cfg, ffn=1)   # attention weights (its 1-wide dense FFN is unused)
        self.ffn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.router = nn.Parameter(torch.empty(cfg.n_experts, cfg.dim))
        self.expert_ids = list(range(cfg.n_experts)) if expert_ids is None else list(expert_ids)
        self.experts = nn.ModuleList([Expert(cfg.dim, cfg.ffn_dim) for _ in self.expert_ids])

    def moe_single(self, h: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, out: torch.Tensor, impl: str):
        from flextensor_b200 import ops

        acc = out.float()
        for j, e in enumerate(self.expert_ids):
            hit = (ids == e)
            rows = hit.any(-1).nonzero().squeeze(-1)
            if rows.numel() == 0:
                continue
            w = (wts * hit).sum(-1)[rows]
            xe = h.index_select(0, rows)
            ex = self.experts[j]
            if impl == "fused":
                y = ops.linear(ops.linear_swiglu(xe, ex.w_gate_up), ex.w_down, None, epi="none")
            else:
                gu = F.linear(xe, ex.w_gate_up)
                y = F.linear(F.silu(gu[:, 0::2]) * gu[:, 1::2], ex.w_down)
            acc.index_add_(0, rows, y.float() * w[:, None])
        out.copy_(acc.to(out.dtype))
        return out

    def forward(self, x, B, S, rope, impl: str = "fused", ep=None, cache=None, pos: int = 0):
        """``cache`` = (k_cache, v_cache) of this layer: prefill (``pos == 0``) fills positions
        [0, S); a decode step (S == 1) appends position ``pos`` and attends over [0, pos] with the
        split-KV decode kernel (native path only)."""
        from flextensor_b200 import ops
        from flextensor_b200.parallel.ep import NcclExpertParallel, route_topk

        cfg = self.cfg
        if impl == "fused":
            x = self.attn.attention_fused(x, B, S, rope, cache, pos)
        else:
            x = self.attn.attention_torch(x, B, S, rope)
        h = ops.rmsnorm(x, self.ffn_norm, eps=cfg.eps) if impl == "fused" else _rms_torch(x, self.ffn_norm, cfg.eps)
        ids, wts = route_topk(h, self.router, cfg.topk)
        if ep is None:
            return self.moe_single(h, ids, wts, x, impl)
        if isinstance(ep, NcclExpertParallel):
            return ep(h, ids, wts, [e.w_gate_up for e in self.experts], [e.w_down for e in self.experts], x)
        slots = ep.dispatch(h, ids)
        ep.experts([e.w_gate_up for e in self.experts], [e.w_down for e in self.experts])
        return ep.combine(slots, wts, residual=x, out=x)


class MixtralModel(nn.Module):
    def __init__(self, cfg: MixtralConfig = MIXTRAL_8X22B, impl: str = "fused", rank: int = 0, world: int = 1,
                 layers: int | None = None):
        super().__init__()
        self.cfg, self.impl = cfg, impl
        el = cfg.n_experts // world
        mine = list(range(rank * el, (rank + 1) * el))
        self.embed = nn.Embedding(cfg.vocab, cfg.dim)
        self.layers = nn.ModuleList([MixtralLayer(cfg, mine) for _ in range(layers or cfg.n_layers)])
        self.norm = nn.Parameter(torch.ones(cfg.dim))
        self.lm_head = nn.Parameter(torch.empty(cfg.vocab, cfg.dim))
        self._rope = {}

    def rope(self, S, device):
        key = (S, str(device))
        if key not in self._rope:
            self._rope[key] = rope_tables_1d(S, self.cfg.head_dim, self.cfg.rope_theta, device)
        return self._rope[key]

    def hidden(self, tokens: torch.Tensor, ep=None) -> torch.Tensor:
        B, S = tokens.shape
        x = self.embed(tokens).reshape(B * S, -1).contiguous()
        rope = self.rope(S, x.device)
        for layer in self.layers:
            x = layer(x, B, S, rope, self.impl, ep=ep)
        return x

    def forward(self, tokens: torch.Tensor, ep=None) -> torch.Tensor:
        B, S = tokens.shape
        x = self.hidden(tokens, ep)
        h = _rms_torch(x.view(B, S, -1)[:, -1], self.norm, self.cfg.eps)
        return F.linear(h, self.lm_head)

    # ---------------------------------------------------------------- KV-cache generation
    def new_cache(self, batch: int, max_len: int, device=None, dtype=torch.bfloat16):
        cfg = self.cfg
        dev = device or self.lm_head.device
        return [(torch.empty(batch, max_len, cfg.n_kv_heads, cfg.head_dim, device=dev, dtype=dtype),
                 torch.empty(batch, max_len, cfg.n_kv_heads, cfg.head_dim, device=dev, dtype=dtype))
                for _ in self.layers]

    def _logits(self, h_last):
        return F.linear(_rms_torch(h_last, self.norm, self.cfg.eps), self.lm_head)

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, cache, ep=None) -> torch.Tensor:
        """Run the prompts (native path), fill the cache, return last-position logits."""
        B, S = tokens.shape
        x = self.embed(tokens).reshape(B * S, -1).contiguous()
        cos, sin = self.rope(cache[0][0].shape[1], x.device)
        rope_s = (cos[:S], sin[:S])
        for layer, c in zip(self.layers, cache):
            x = layer(x, B, S, rope_s, self.impl, ep=ep, cache=c, pos=0)
        return self._logits(x.view(B, S, -1)[:, -1])

    @torch.no_grad()
    def decode_step(self, token: torch.Tensor, cache, pos: int, ep=None) -> torch.Tensor:
        """One new token per sequence at position ``pos``; returns its logits ``[B, vocab]``."""
        B = token.shape[0]
        x = self.embed(token.view(B)).contiguous()
        cos, sin = self.rope(cache[0][0].shape[1], x.device)
        rope_p = (cos[pos:pos + 1].contiguous(), sin[pos:pos + 1].contiguous())
        for layer, c in zip(self.layers, cache):
            x = layer(x, B, 1, rope_p, self.impl, ep=ep, cache=c, pos=pos)
        return self._logits(x)

    @torch.no_grad()
    def generate(self, tokens: torch.Tensor, max_new: int, ep=None) -> torch.Tensor:
        """Greedy continuation ``[B, max_new]`` with a KV cache."""
        B, S = tokens.shape
        cache = self.new_cache(B, S + max_new, tokens.device)
        logits = self.prefill(tokens, cache, ep)
        out = []
        for i in range(max_new):
            nxt = logits.argmax(-1)
            out.append(nxt)
            if i + 1 < max_new:
                logits = self.decode_step(nxt, cache, S + i, ep)
        return torch.stack(out, dim=1)


class MixtralStack(nn.Module):
    """The decoder layers alone (no embedding / head): the offloadable body for end-to-end runs.
    ``ep``: an :class:`~flextensor_b200.parallel.ep.ExpertParallel` per token-row count (e.g. the
    prefill's and the decode step's), chosen by the rows of ``x``."""

    def __init__(self, cfg: MixtralConfig = MIXTRAL_8X22B, rank: int = 0, world: int = 1, layers: int | None = None):
        super().__init__()
        self.cfg = cfg
        el = cfg.n_experts // world
        mine = list(range(rank * el, (rank + 1) * el))
        self.layers = nn.ModuleList([MixtralLayer(cfg, mine) for _ in range(layers or cfg.n_layers)])

    def new_cache(self, batch: int, max_len: int, device=None, dtype=torch.bfloat16):
        c = self.cfg
        dev = device or torch.device("cuda", torch.cuda.current_device())
        return [(torch.empty(batch, max_len, c.n_kv_heads, c.head_dim, device=dev, dtype=dtype),
                 torch.empty(batch, max_len, c.n_kv_heads, c.head_dim, device=dev, dtype=dtype))
                for _ in self.layers]

    def forward(self, x, B, S, rope, ep: dict | None = None, cache=None, pos: int = 0):
        e = None if not ep else ep.get(x.shape[0])
        for i, L in enumerate(self.layers):
            x = L(x, B, S, rope, "fused", ep=e, cache=None if cache is None else cache[i], pos=pos)
        return x


@torch.no_grad()
def init_mixtral_params_(model: nn.Module, seed: int = 0, std: float = 0.02, full_experts: int | None = None) -> None:
    """Deterministic init; an expert's weights depend only on (seed, layer, global expert id),
    so expert-parallel shards match the single-GPU model."""
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev)
    for name, p in model.named_parameters():
        if ".experts." in name:
            continue
        g.manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
        if name.endswith("norm") or name.endswith("attn_norm") or name.endswith("ffn_norm"):
            p.fill_(1.0)
        else:
            p.normal_(0.0, std, generator=g)
    for li, layer in enumerate(model.layers):
        for j, e in enumerate(layer.expert_ids):
            ex = layer.experts[j]
            g.manual_seed(seed * 7919 + li * 131 + e)
            ex.w_gate_up.normal_(0.0, std, generator=g)
            ex.w_down.normal_(0.0, std, generator=g)
