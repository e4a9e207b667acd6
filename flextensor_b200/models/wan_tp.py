"""Tensor parallelism for the Wan DiT blocks: attention heads and FFN columns split across the
ranks of one node.

Mirrors the TP layout of the reference's LTX benchmark driver
(``examples/ltx23/outpaint/benchmarks/integrated_e2e.py:159-220``: ``col_shard`` for Q/K/V and
the FFN input, ``row_shard`` with an ``all_reduce`` forward hook for the output projections,
``DistRMSNorm`` all-reducing the Q/K sums of squares) in two implementations:

``impl="fused"`` (the B200 data plane). The residual stream stays sequence-parallel: each rank
holds 1/N of the token rows between projections and runs the adaLN/LayerNorm on those rows only.

* A column-parallel projection gathers every rank's rows inside the GEMM:
  :class:`~flextensor_b200.parallel.tp.TPAllGather`, the tcgen05 kernel pulling peer rows over
  NVLink while it multiplies. K and V reuse the gathered buffer.
* The Q/K RMSNorm over the full hidden size sends per-row partial sums of squares over peer
  stores and applies RoPE on the way out (:class:`~flextensor_b200.parallel.tp.TPRMSNorm`).
* A row-parallel projection stores its partial rows straight into the owners' staging from the
  GEMM epilogue. The owner sums them and applies bias, adaLN gate and residual in one pass
  (:class:`~flextensor_b200.parallel.tp.TPReduceScatter`).

``impl="nccl"`` is the reference's layout on the same kernels. The residual stream is
replicated, the row-parallel outputs and the sums of squares go through NCCL ``all_reduce``, and
the gated residual is applied in PyTorch. It is the baseline that ``benchmarks/tp_wan.py`` times
against the fused path.

Batch size 1 (the serving shape); the sequence length must split evenly over the ranks.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from flextensor_b200.models.wan import WanDiT, _gather_seq, sinusoidal


def _shard_rows(lin: nn.Linear, rank: int, world: int) -> None:
    n = lin.weight.shape[0] // world
    sl = slice(rank * n, (rank + 1) * n)
    lin.weight = nn.Parameter(lin.weight.data[sl].contiguous(), requires_grad=False)
    if lin.bias is not None:
        lin.bias = nn.Parameter(lin.bias.data[sl].contiguous(), requires_grad=False)


def _shard_cols(lin: nn.Linear, rank: int, world: int) -> None:
    k = lin.weight.shape[1] // world
    lin.weight = nn.Parameter(lin.weight.data[:, rank * k:(rank + 1) * k].contiguous(), requires_grad=False)


def _shard_vec(p: nn.Parameter, rank: int, world: int) -> nn.Parameter:
    n = p.shape[0] // world
    return nn.Parameter(p.data[rank * n:(rank + 1) * n].contiguous(), requires_grad=False)


class WanTensorParallel:
    """Shards ``model``'s blocks in place for this rank and runs its forward tensor-parallel."""

    def __init__(self, model: WanDiT, group=None, impl: str = "fused", max_tokens: int | None = None,
                 text_len: int | None = None):
        import torch.distributed as dist

        if impl not in ("fused", "nccl"):
            raise ValueError(f"impl must be 'fused' or 'nccl', got {impl!r}")
        self.model, self.group, self.impl = model, group, impl
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        cfg = model.cfg
        W = self.world
        if cfg.num_heads % W or cfg.ffn_dim % W:
            raise ValueError(f"{cfg.num_heads} heads / FFN {cfg.ffn_dim} do not split over {W} ranks")
        for blk in model.blocks:
            for a in (blk.attn1, blk.attn2):
                for lin in (a.to_q, a.to_k, a.to_v):
                    _shard_rows(lin, self.rank, W)
                _shard_cols(a.to_out, self.rank, W)
                a.norm_q.weight = _shard_vec(a.norm_q.weight, self.rank, W)
                a.norm_k.weight = _shard_vec(a.norm_k.weight, self.rank, W)
            _shard_rows(blk.ffn_in, self.rank, W)
            _shard_cols(blk.ffn_out, self.rank, W)
        self.d_local = cfg.dim // W
        self.h_local = cfg.num_heads // W
        self.ag = self.rs = self.rms = None
        if impl == "fused":
            if max_tokens is None:
                raise ValueError("the fused path needs max_tokens (the sequence length it is sized for)")
            from flextensor_b200.parallel.tp import TPAllGather, TPReduceScatter, TPRMSNorm

            self.ag = TPAllGather(max_tokens, cfg.dim, group)
            self.rs = TPReduceScatter(max_tokens, cfg.dim, group)
            self.rms = TPRMSNorm(max(max_tokens, text_len or cfg.text_len), group)
        self.S = max_tokens

    # ------------------------------------------------------------------ blocks
    def _block_fused(self, blk, x2, ctx2, mods, cos, sin, S):
        from flextensor_b200 import ops

        cfg = self.model.cfg
        D, Dh, Hl = cfg.dim, cfg.head_dim, self.h_local
        shift1, scale1, gate1 = mods[:, 0], mods[:, 1], mods[:, 2]
        shift3, scale3, gate3 = mods[:, 3], mods[:, 4], mods[:, 5]
        a1, a2 = blk.attn1, blk.attn2
        # self-attention: LN on our rows -> gathered inside the Q GEMM; K, V on the gathered rows
        h = self.ag.begin()
        ops.layernorm_modulate(x2, scale1, shift1, eps=cfg.eps, out=h)
        self.ag.publish()
        q = self.ag.gemm(a1.to_q.weight, a1.to_q.bias, epi="bias")
        full = self.ag.full()
        k = ops.linear(full, a1.to_k.weight, a1.to_k.bias)
        v = ops.linear(full, a1.to_v.weight, a1.to_v.bias)
        self.rms(q, a1.norm_q.weight, D, cfg.eps, cos, sin, Dh, S, out=q)
        self.rms(k, a1.norm_k.weight, D, cfg.eps, cos, sin, Dh, S, out=k)
        o = ops.attention(q.view(1, S, Hl, Dh), k.view(1, S, Hl, Dh), v.view(1, S, Hl, Dh))
        self.rs.gemm(o.view(S, self.d_local), a1.to_out.weight)
        self.rs.reduce(x2, residual=x2, bias=a1.to_out.bias, gate=gate1)
        # cross-attention over the (replicated) text context
        h = self.ag.begin()
        ops.layernorm_modulate(x2, weight=blk.norm2.weight, bias=blk.norm2.bias, eps=cfg.eps, out=h)
        self.ag.publish()
        q = self.ag.gemm(a2.to_q.weight, a2.to_q.bias, epi="bias")
        self.rms(q, a2.norm_q.weight, D, cfg.eps, out=q)
        kc = ops.linear(ctx2, a2.to_k.weight, a2.to_k.bias)
        self.rms(kc, a2.norm_k.weight, D, cfg.eps, out=kc)
        vc = ops.linear(ctx2, a2.to_v.weight, a2.to_v.bias)
        L = ctx2.shape[0]
        o = ops.attention(q.view(1, S, Hl, Dh), kc.view(1, L, Hl, Dh), vc.view(1, L, Hl, Dh), out=o)
        self.rs.gemm(o.view(S, self.d_local), a2.to_out.weight)
        self.rs.reduce(x2, residual=x2, bias=a2.to_out.bias)
        # FFN
        h = self.ag.begin()
        ops.layernorm_modulate(x2, scale3, shift3, eps=cfg.eps, out=h)
        self.ag.publish()
        f = self.ag.gemm(blk.ffn_in.weight, blk.ffn_in.bias, epi="gelu")
        self.rs.gemm(f, blk.ffn_out.weight)
        self.rs.reduce(x2, residual=x2, bias=blk.ffn_out.bias, gate=gate3)
        return x2

    def _block_nccl(self, blk, x2, ctx2, mods, cos, sin, S):
        import torch.distributed as dist

        from flextensor_b200 import ops
        from flextensor_b200.parallel.tp import nccl_rmsnorm

        cfg = self.model.cfg
        D, Dh, Hl, g = cfg.dim, cfg.head_dim, self.h_local, self.group
        shift1, scale1, gate1 = mods[:, 0], mods[:, 1], mods[:, 2]
        shift3, scale3, gate3 = mods[:, 3], mods[:, 4], mods[:, 5]
        a1, a2 = blk.attn1, blk.attn2

        def row_parallel(inp, lin, gate):
            y = ops.linear(inp, lin.weight, None, epi="none")
            dist.all_reduce(y, group=g)
            y = y.float() + lin.bias.float()
            if gate is not None:
                y = y * gate
            x2.copy_((x2.float() + y).to(x2.dtype))

        h = ops.layernorm_modulate(x2, scale1, shift1, eps=cfg.eps)
        q = ops.linear(h, a1.to_q.weight, a1.to_q.bias)
        k = ops.linear(h, a1.to_k.weight, a1.to_k.bias)
        v = ops.linear(h, a1.to_v.weight, a1.to_v.bias)
        q = ops.rope(nccl_rmsnorm(q, a1.norm_q.weight, D, cfg.eps, g), cos, sin, Dh, S)
        k = ops.rope(nccl_rmsnorm(k, a1.norm_k.weight, D, cfg.eps, g), cos, sin, Dh, S)
        o = ops.attention(q.view(1, S, Hl, Dh), k.view(1, S, Hl, Dh), v.view(1, S, Hl, Dh))
        row_parallel(o.view(S, self.d_local), a1.to_out, gate1)
        h = ops.layernorm_modulate(x2, weight=blk.norm2.weight, bias=blk.norm2.bias, eps=cfg.eps, out=h)
        q = nccl_rmsnorm(ops.linear(h, a2.to_q.weight, a2.to_q.bias), a2.norm_q.weight, D, cfg.eps, g)
        kc = nccl_rmsnorm(ops.linear(ctx2, a2.to_k.weight, a2.to_k.bias), a2.norm_k.weight, D, cfg.eps, g)
        vc = ops.linear(ctx2, a2.to_v.weight, a2.to_v.bias)
        L = ctx2.shape[0]
        o = ops.attention(q.view(1, S, Hl, Dh), kc.view(1, L, Hl, Dh), vc.view(1, L, Hl, Dh), out=o)
        row_parallel(o.view(S, self.d_local), a2.to_out, None)
        h = ops.layernorm_modulate(x2, scale3, shift3, eps=cfg.eps, out=h)
        f = ops.linear(h, blk.ffn_in.weight, blk.ffn_in.bias, epi="gelu")
        row_parallel(f, blk.ffn_out, gate3)
        return x2

    # ------------------------------------------------------------------ model
    def forward(self, latent: torch.Tensor, timestep: torch.Tensor, context: torch.Tensor) -> torch.Tensor:
        m, cfg = self.model, self.model.cfg
        if latent.shape[0] != 1:
            raise ValueError("tensor-parallel Wan runs batch size 1")
        dt = m.patch_embedding.weight.dtype
        x, grid = m.patchify(latent.to(dt))
        S = x.shape[1]
        if self.impl == "fused":
            if S != self.S:
                raise ValueError(f"sized for {self.S} tokens, got {S}")
            R = S // self.world
            x = x[:, self.rank * R:(self.rank + 1) * R]
        x2 = m._lin(x.contiguous(), m.patch_embedding, "bias").reshape(-1, cfg.dim).contiguous()
        t = sinusoidal(timestep, cfg.freq_dim).to(dt)
        temb = m._lin(F.silu(m._lin(t, m.time_embedding_1).float()).to(dt), m.time_embedding_2)
        e = m._lin(F.silu(temb.float()).to(dt), m.time_projection).float().view(-1, 6, cfg.dim)
        ctx = m._lin(context.to(dt), m.text_embedding_1, "gelu")
        ctx2 = m._lin(ctx, m.text_embedding_2).reshape(-1, cfg.dim).contiguous()
        cos, sin = m.rope(grid, x2.device)
        block = self._block_fused if self.impl == "fused" else self._block_nccl
        for blk in m.blocks:
            mods = (blk.scale_shift_table.float() + e).contiguous()
            x2 = block(blk, x2, ctx2, mods, cos, sin, S)
        mod = m.head_scale_shift.float() + temb.float()[:, None]
        shift, scale = mod[:, 0:1], mod[:, 1:2]
        h = (F.layer_norm(x2.float()[None], (cfg.dim,), eps=cfg.eps) * (1 + scale) + shift).to(dt)
        y = m._lin(h, m.proj_out)
        if self.impl == "fused":
            y = _gather_seq(y, self.group)
        return m.unpatchify(y, grid)

    __call__ = forward

    def close(self) -> None:
        for obj in (self.ag, self.rs, self.rms):
            if obj is not None:
                obj.close()
        self.ag = self.rs = self.rms = None
