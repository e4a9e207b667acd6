"""Llama-3-shape decoder (GQA, RoPE, SwiGLU), random-init, with single-GPU and tensor-parallel
paths built on the native kernels.

Weight layout is chosen for the kernels (``state_dict`` differs from HF checkpoints, which are
not used here): ``wqkv`` stacks q, k, v rows; ``w_gate_up`` interleaves gate and up rows
(row 2j = gate_j, row 2j+1 = up_j) so one GEMM with the SwiGLU epilogue produces
``silu(gate) * up``; RoPE rotates interleaved pairs.

Tensor parallelism (``LlamaTP``): heads, FFN columns and their weight rows/columns are split
over the ranks, and the residual stream is sequence-parallel (each rank holds 1/N of the token
rows between layers). Per layer: RMSNorm of the own rows straight into the all-gather buffer ->
all-gather+QKV GEMM -> RoPE -> causal GQA attention on the local heads -> o_proj
GEMM+reduce-scatter -> owner reduce with the residual -> RMSNorm -> all-gather+gate/up GEMM
(SwiGLU) -> down GEMM+reduce-scatter -> reduce. ``collective="nccl"`` runs the same GEMMs around
NCCL all-gather / reduce-scatter (the baseline).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class LlamaConfig:
    dim: int = 8192
    n_layers: int = 80
    n_heads: int = 64
    n_kv_heads: int = 8
    ffn_dim: int = 28672
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads


LLAMA3_70B = LlamaConfig()


def tiny_llama(**kw) -> LlamaConfig:
    base = dict(dim=512, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=1024, vocab=1024)
    base.update(kw)
    return LlamaConfig(**base)


def rope_tables_1d(seq_len: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device=device) / head_dim))
    ang = torch.outer(torch.arange(seq_len, dtype=torch.float64, device=device), inv)
    return torch.cos(ang).float().contiguous(), torch.sin(ang).float().contiguous()


def _rope_torch(x, cos, sin):  # x [B, S, H, D] fp32, interleaved pairs
    b, s, h, d = x.shape
    xr = x.view(b, s, h, d // 2, 2)
    re, im = xr[..., 0], xr[..., 1]
    c, sn = cos[None, :s, None, :], sin[None, :s, None, :]
    return torch.stack([re * c - im * sn, re * sn + im * c], dim=-1).view(b, s, h, d)


def _rms_torch(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class LlamaLayer(nn.Module):
    def __init__(self, cfg: LlamaConfig, n_heads: int | None = None, n_kv: int | None = None,
                 ffn: int | None = None):
        super().__init__()
        self.cfg = cfg
        hq, hk, f = n_heads or cfg.n_heads, n_kv or cfg.n_kv_heads, ffn or cfg.ffn_dim
        self.hq, self.hk, self.f = hq, hk, f
        D = cfg.head_dim
        self.attn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.wqkv = nn.Parameter(torch.empty((hq + 2 * hk) * D, cfg.dim))
        self.wo = nn.Parameter(torch.empty(cfg.dim, hq * D))
        self.ffn_norm = nn.Parameter(torch.ones(cfg.dim))
        self.w_gate_up = nn.Parameter(torch.empty(2 * f, cfg.dim))
        self.w_down = nn.Parameter(torch.empty(cfg.dim, f))

    # ---------------------------------------------------------------- single GPU
    def forward_torch(self, x, B, S, rope):
        cfg = self.cfg
        x = self.attention_torch(x, B, S, rope)
        h = _rms_torch(x, self.ffn_norm, cfg.eps)
        gu = F.linear(h, self.w_gate_up)
        return x + F.linear(F.silu(gu[:, 0::2]) * gu[:, 1::2], self.w_down)

    def attention_fused(self, x, B, S, rope, cache=None, pos: int = 0):
        """x += o_proj(causal GQA attention(RMSNorm(x))), native kernels, in place.

        ``cache`` = (k_cache, v_cache) ``[B, L_max, Hk, 128]``: prefill (``pos == 0``, S tokens)
        stores the rotated keys and the values of positions [0, S); a decode step (S == 1,
        ``rope`` holding position ``pos``) appends position ``pos`` and attends over [0, pos]."""
        from flextensor_b200 import ops

        cfg, D = self.cfg, self.cfg.head_dim
        h = ops.rmsnorm(x, self.attn_norm, eps=cfg.eps)
        qkv = ops.linear(h, self.wqkv, None, epi="none")
        qn, kn = self.hq * D, self.hk * D
        q, k, v = qkv[:, :qn], qkv[:, qn:qn + kn], qkv[:, qn + kn:]
        ops.rope(q, *rope, D, S, out=q)
        ops.rope(k, *rope, D, S, out=k)
        qv, kv_, vv = q.view(B, S, self.hq, D), k.view(B, S, self.hk, D), v.view(B, S, self.hk, D)
        if cache is None:
            o = ops.attention(qv, kv_, vv, causal=True)
        else:
            kc, vc = cache
            kc[:, pos:pos + S].copy_(kv_)
            vc[:, pos:pos + S].copy_(vv)
            if S == 1:  # decode: one query per sequence over the cached keys [0, pos]
                o = ops.decode_attention(qv, kc, vc, pos + 1)
            else:
                o = ops.attention(qv, kv_, vv, causal=True)
        ops.linear(o.reshape(B * S, -1), self.wo, None, epi="res", residual=x, out=x)
        return x

    def attention_torch(self, x, B, S, rope):
        cfg, D = self.cfg, self.cfg.head_dim
        h = _rms_torch(x, self.attn_norm, cfg.eps)
        qkv = F.linear(h, self.wqkv)
        q, k, v = qkv.split([self.hq * D, self.hk * D, self.hk * D], dim=-1)
        q = _rope_torch(q.reshape(B, S, self.hq, D).float(), *rope).to(x.dtype)
        k = _rope_torch(k.reshape(B, S, self.hk, D).float(), *rope).to(x.dtype)
        v = v.reshape(B, S, self.hk, D)
        rep = self.hq // self.hk
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.repeat_interleave(rep, 2).transpose(1, 2),
                                           v.repeat_interleave(rep, 2).transpose(1, 2), is_causal=True)
        return x + F.linear(o.transpose(1, 2).reshape(B * S, -1), self.wo)

    def forward_fused(self, x, B, S, rope, cache=None, pos: int = 0):
        from flextensor_b200 import ops

        cfg = self.cfg
        x = self.attention_fused(x, B, S, rope, cache, pos)
        h = ops.rmsnorm(x, self.ffn_norm, eps=cfg.eps)
        f = ops.linear_swiglu(h, self.w_gate_up)
        ops.linear(f, self.w_down, None, epi="res", residual=x, out=x)
        return x

    # ---------------------------------------------------------------- tensor parallel (one rank's shard)
    def forward_tp(self, x_local, B, S, rope, tp, cache=None, pos: int = 0):
        """One rank's shard. ``cache`` = this rank's (k_cache, v_cache) ``[B, L_max, hk, 128]``:
        prefill (``pos == 0``) stores positions [0, S); a decode step (S == 1) appends position
        ``pos`` and attends over [0, pos] with the split-KV decode kernel."""
        from flextensor_b200 import ops

        cfg, D = self.cfg, self.cfg.head_dim
        qn, kn = self.hq * D, self.hk * D
        ag_fused = tp.collective in ("fused", "fused_ag")
        rs_fused = tp.collective in ("fused", "fused_rs")
        _ag, _rs = tp.tp_buffers(B * S)

        def gathered_gemm(norm_w, w, epi):
            if ag_fused:  # RMSNorm of the own rows straight into the all-gather buffer
                ops.rmsnorm(x_local, norm_w, eps=cfg.eps, out=_ag.begin())
                _ag.publish()
                return _ag.gemm(w, epi=epi)
            h = tp._nccl.all_gather(ops.rmsnorm(x_local, norm_w, eps=cfg.eps))
            return ops.linear_swiglu(h, w) if epi == "swiglu" else ops.linear(h, w, None, epi="none")

        def scattered_gemm(a, w):
            nonlocal x_local
            if rs_fused:
                _rs.gemm(a, w)
                _rs.reduce(x_local, residual=x_local)
            else:
                x_local += tp._nccl.reduce_scatter(ops.linear(a, w, None, epi="none"))

        qkv = gathered_gemm(self.attn_norm, self.wqkv, "none")
        q, k, v = qkv[:, :qn], qkv[:, qn:qn + kn], qkv[:, qn + kn:]
        ops.rope(q, *rope, D, S, out=q)
        ops.rope(k, *rope, D, S, out=k)
        qv, kv_, vv = q.view(B, S, self.hq, D), k.view(B, S, self.hk, D), v.view(B, S, self.hk, D)
        if cache is not None:
            kc, vc = cache
            kc[:, pos:pos + S].copy_(kv_)
            vc[:, pos:pos + S].copy_(vv)
        if cache is not None and S == 1:
            o = ops.decode_attention(qv, cache[0], cache[1], pos + 1)
        else:
            o = ops.attention(qv, kv_, vv, causal=True)
        scattered_gemm(o.view(B * S, -1), self.wo)
        f = gathered_gemm(self.ffn_norm, self.w_gate_up, "swiglu")
        scattered_gemm(f, self.w_down)
        return x_local

    def forward(self, x, B, S, rope, impl="fused", tp=None, cache=None, pos: int = 0):
        if tp is not None:
            return self.forward_tp(x, B, S, rope, tp, cache, pos)
        if cache is not None:
            return self.forward_fused(x, B, S, rope, cache, pos)
        return self.forward_fused(x, B, S, rope) if impl == "fused" else self.forward_torch(x, B, S, rope)


class LlamaModel(nn.Module):
    def __init__(self, cfg: LlamaConfig = LLAMA3_70B, impl: str = "fused"):
        super().__init__()
        self.cfg = cfg
        self.impl = impl
        self.embed = nn.Embedding(cfg.vocab, cfg.dim)
        self.layers = nn.ModuleList([LlamaLayer(cfg) for _ in range(cfg.n_layers)])
        self.norm = nn.Parameter(torch.ones(cfg.dim))
        self.lm_head = nn.Parameter(torch.empty(cfg.vocab, cfg.dim))
        self._rope = {}

    def rope(self, S, device):
        key = (S, str(device))
        if key not in self._rope:
            self._rope[key] = rope_tables_1d(S, self.cfg.head_dim, self.cfg.rope_theta, device)
        return self._rope[key]

    def forward(self, tokens: torch.Tensor, last_only: bool = True) -> torch.Tensor:
        """tokens ``[B, S]`` (equal-length prompts) -> logits ``[B, vocab]`` of the last position
        (or ``[B, S, vocab]``)."""
        B, S = tokens.shape
        x = self.embed(tokens).reshape(B * S, -1).contiguous()
        rope = self.rope(S, x.device)
        for layer in self.layers:
            x = layer(x, B, S, rope, self.impl)
        h = x.view(B, S, -1)[:, -1] if last_only else x.view(B, S, -1)
        h = _rms_torch(h, self.norm, self.cfg.eps)
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
    def prefill(self, tokens: torch.Tensor, cache) -> torch.Tensor:
        """Native path: run the prompts, fill the cache, return last-position logits."""
        B, S = tokens.shape
        x = self.embed(tokens).reshape(B * S, -1).contiguous()
        rope = self.rope(cache[0][0].shape[1], x.device)
        rope_s = (rope[0][:S], rope[1][:S])
        for layer, c in zip(self.layers, cache):
            x = layer(x, B, S, rope_s, self.impl, cache=c, pos=0)
        return self._logits(x.view(B, S, -1)[:, -1])

    @torch.no_grad()
    def decode_step(self, token: torch.Tensor, cache, pos: int) -> torch.Tensor:
        """One new token per sequence at position ``pos``; returns its logits ``[B, vocab]``."""
        B = token.shape[0]
        x = self.embed(token.view(B)).contiguous()
        cos, sin = self.rope(cache[0][0].shape[1], x.device)
        rope_p = (cos[pos:pos + 1].contiguous(), sin[pos:pos + 1].contiguous())
        for layer, c in zip(self.layers, cache):
            x = layer(x, B, 1, rope_p, self.impl, cache=c, pos=pos)
        return self._logits(x)

    @torch.no_grad()
    def generate(self, tokens: torch.Tensor, max_new: int) -> torch.Tensor:
        """Greedy continuation ``[B, max_new]`` with a KV cache."""
        B, S = tokens.shape
        cache = self.new_cache(B, S + max_new, tokens.device)
        logits = self.prefill(tokens, cache)
        out = []
        for i in range(max_new):
            nxt = logits.argmax(-1)
            out.append(nxt)
            if i + 1 < max_new:
                logits = self.decode_step(nxt, cache, S + i)
        return torch.stack(out, dim=1)


def init_llama_params_(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    g = torch.Generator(device=next(model.parameters()).device)
    g.manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm") or name == "norm":
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)


# ----------------------------------------------------------------------------- tensor parallel
class LlamaTP(nn.Module):
    """One rank's shard of the decoder layers (heads / FFN split over ``world`` ranks)."""

    def __init__(self, cfg: LlamaConfig, rank: int, world: int, layers: int | None = None):
        super().__init__()
        if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.ffn_dim % world:
            raise ValueError("heads, kv heads and FFN width must split evenly over the ranks")
        self.cfg, self.rank, self.world = cfg, rank, world
        n = layers if layers is not None else cfg.n_layers
        self.layers = nn.ModuleList([LlamaLayer(cfg, cfg.n_heads // world, cfg.n_kv_heads // world,
                                                cfg.ffn_dim // world) for _ in range(n)])
        self._ag = self._rs = self._nccl = None

    @torch.no_grad()
    def load_from_full(self, full: LlamaModel) -> "LlamaTP":
        cfg, r, W, D = self.cfg, self.rank, self.world, self.cfg.head_dim
        hq, hk, f = cfg.n_heads // W, cfg.n_kv_heads // W, cfg.ffn_dim // W
        for mine, src in zip(self.layers, full.layers):
            qn, kn = cfg.n_heads * D, cfg.n_kv_heads * D
            q = src.wqkv[:qn].view(cfg.n_heads, D, -1)[r * hq:(r + 1) * hq].reshape(hq * D, -1)
            k = src.wqkv[qn:qn + kn].view(cfg.n_kv_heads, D, -1)[r * hk:(r + 1) * hk].reshape(hk * D, -1)
            v = src.wqkv[qn + kn:].view(cfg.n_kv_heads, D, -1)[r * hk:(r + 1) * hk].reshape(hk * D, -1)
            mine.wqkv.copy_(torch.cat([q, k, v]))
            mine.wo.copy_(src.wo.view(cfg.dim, cfg.n_heads, D)[:, r * hq:(r + 1) * hq].reshape(cfg.dim, -1))
            mine.w_gate_up.copy_(src.w_gate_up.view(cfg.ffn_dim, 2, -1)[r * f:(r + 1) * f].reshape(2 * f, -1))
            mine.w_down.copy_(src.w_down[:, r * f:(r + 1) * f])
            mine.attn_norm.copy_(src.attn_norm)
            mine.ffn_norm.copy_(src.ffn_norm)
        return self

    def setup(self, tokens_total: int, group=None, collective: str = "fused", pair: bool = False) -> None:
        """``collective``: ``fused`` (all-gather inside the column-parallel GEMMs, reduce-scatter
        from the row-parallel GEMM epilogues), ``nccl`` (NCCL around plain GEMMs), or one fused
        side only: ``fused_ag`` / ``fused_rs``. ``pair``: the experimental CTA-pair (cta_group::2)
        kernels for the fused sides."""
        from flextensor_b200.parallel.tp import NcclTP, TPAllGather, TPReduceScatter

        if collective not in ("fused", "nccl", "fused_ag", "fused_rs"):
            raise ValueError(f"unknown collective {collective!r}")
        self.collective = collective
        self._group, self._pair = group, pair
        self._nccl = NcclTP(group)
        self._by_rows: dict[int, tuple] = {}
        self._ag, self._rs = self._make(tokens_total)
        self._by_rows[tokens_total] = (self._ag, self._rs)

    def _make(self, rows: int):
        from flextensor_b200.parallel.tp import TPAllGather, TPReduceScatter

        ag = rs = None
        if self.collective in ("fused", "fused_ag"):
            ag = TPAllGather(rows, self.cfg.dim, self._group, pair=self._pair)
        if self.collective in ("fused", "fused_rs"):
            rs = TPReduceScatter(rows, self.cfg.dim, self._group, pair=self._pair)
        return ag, rs

    def add_rows(self, tokens_total: int) -> None:
        """Fused-collective buffers for another row count (e.g. the decode step's B rows next to
        the prefill's B*S); every rank must call it, in the same order."""
        if tokens_total not in self._by_rows:
            self._by_rows[tokens_total] = self._make(tokens_total)

    def tp_buffers(self, rows: int):
        """(all-gather, reduce-scatter) objects sized for ``rows`` token rows."""
        if rows not in self._by_rows:
            raise ValueError(f"no fused TP buffers for {rows} rows: call setup()/add_rows() on every rank first")
        return self._by_rows[rows]

    def close(self) -> None:
        for ag, rs in getattr(self, "_by_rows", {}).values():
            for o in (ag, rs):
                if o is not None:
                    o.close()
        self._by_rows = {}
        self._ag = self._rs = None

    def new_cache(self, batch: int, max_len: int, device=None, dtype=torch.bfloat16):
        """This rank's KV cache: its ``n_kv_heads / world`` heads of every layer."""
        D = self.cfg.head_dim
        hk = self.cfg.n_kv_heads // self.world
        dev = device or torch.device("cuda", torch.cuda.current_device())
        return [(torch.empty(batch, max_len, hk, D, device=dev, dtype=dtype),
                 torch.empty(batch, max_len, hk, D, device=dev, dtype=dtype)) for _ in self.layers]

    def forward(self, x_local: torch.Tensor, B: int, S: int, rope, cache=None, pos: int = 0) -> torch.Tensor:
        """x_local ``[B*S/world, dim]`` (this rank's token rows) -> same rows after all layers.
        Each layer is called as a module (``layers.*`` are offload units). ``cache``: from
        :meth:`new_cache` (prefill at ``pos == 0``, then one decode step per call with S == 1)."""
        single = self.world == 1  # one rank: plain native layers, no collectives
        for i, L in enumerate(self.layers):
            x_local = L(x_local, B, S, rope, tp=None if single else self, cache=None if cache is None else cache[i],
                        pos=pos)
        return x_local
