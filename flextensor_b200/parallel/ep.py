"""Expert parallelism for MoE layers with dispatch and combine fused into the expert GEMMs.

Every rank is a token source (its own batch rows) and owns ``E / world`` experts. Per MoE
layer:

1. route (source side): top-k router, rows packed by expert into the source's send buffer in
   the symmetric heap, ``{cnt[E], off[E]}`` table written next to it, epoch flag published;
2. ``moe_dispatch_gemm`` (expert side): gate/up GEMM of the routed rows with SwiGLU in the
   epilogue; the kernel pulls each source's rows over NVLink itself (``ops/csrc/moe_sm100.cu``)
   and acknowledges the sources;
3. ``moe_combine_gemm`` (expert side): down GEMM whose epilogue stores each output row into the
   combine buffer of the source that sent it, then flags every source;
4. ``moe_reduce`` (source side): residual + router-weighted sum of the top-k expert rows.

No NCCL all-to-all on the data path; :class:`NcclExpertParallel` is that baseline
(``all_to_all_single`` dispatch and combine around per-expert GEMMs).
"""

from __future__ import annotations

import torch

from flextensor_b200.ops import native
from flextensor_b200.parallel.symm import SymmetricHeap


def route_topk(x: torch.Tensor, router_w: torch.Tensor, topk: int):
    """Mixtral routing: top-k of the router logits, softmax over the selected logits.
    Returns (expert ids [T, k] int64, weights [T, k] fp32)."""
    logits = torch.nn.functional.linear(x.float(), router_w.float())
    val, idx = torch.topk(logits, topk, dim=-1)
    return idx, torch.softmax(val, dim=-1)


class ExpertParallel:
    def __init__(self, tokens_per_rank: int, d: int, f: int, n_experts: int, topk: int = 2, group=None,
                 device: int | None = None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.T, self.d, self.f, self.E, self.topk = tokens_per_rank, d, f, n_experts, topk
        self.el = n_experts // self.world
        self.rows = tokens_per_rank * topk                      # rows one source sends per layer
        dev = torch.cuda.current_device() if device is None else device
        self.device = torch.device("cuda", dev)
        # worst case: every source routes every row to this rank's experts, plus group padding
        self.max_rows = ((self.world * self.rows + self.el * 128) + 127) // 128 * 128
        W = self.world
        # heap layout: page 0 flags (send flags | send acks | comb flags, W u64 each, from byte
        # 256), page 1 the {cnt[E], off[E]} table, then the send and combine buffers
        if 3 * W * 8 + 256 > 4096 or 2 * n_experts * 4 > 4096:
            raise ValueError("too many ranks / experts for the header pages")
        self.flag_off, self.tbl_off, self.send_off = 256, 4096, 8192
        send_bytes = (self.rows * d * 2 + 4095) // 4096 * 4096
        self.comb_off = self.send_off + send_bytes
        total = self.comb_off + send_bytes
        self.heap = SymmetricHeap(total, group, dev)
        P = self.heap.ptrs
        self.send_flags = [p + self.flag_off for p in P]
        self.send_acks = [p + self.flag_off + W * 8 for p in P]
        self.comb_flags = [p + self.flag_off + 2 * W * 8 for p in P]
        self.a_local = torch.empty(self.max_rows, d, dtype=torch.bfloat16, device=self.device)
        self.h_local = torch.empty(self.max_rows, f, dtype=torch.bfloat16, device=self.device)
        self.counters = torch.zeros(2 * W + 1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        dist.barrier(group=group)

    # ------------------------------------------------------------------ views of the local heap
    def _send(self) -> torch.Tensor:
        return self.heap.view(self.send_off, self.rows * self.d * 2).view(torch.bfloat16).view(self.rows, self.d)

    def _comb(self) -> torch.Tensor:
        return self.heap.view(self.comb_off, self.rows * self.d * 2).view(torch.bfloat16).view(self.rows, self.d)

    def _table(self) -> torch.Tensor:
        return self.heap.view(self.tbl_off, 2 * self.E * 4).view(torch.int32)

    # ------------------------------------------------------------------ one MoE layer
    def dispatch(self, x: torch.Tensor, expert_ids: torch.Tensor) -> torch.Tensor:
        """Source side: pack ``x`` rows by expert, publish. Returns ``pos [T, k]`` (int32)."""
        T, k = expert_ids.shape
        if T != self.T or k != self.topk:
            raise ValueError(f"expected {self.T} tokens x top-{self.topk}, got {tuple(expert_ids.shape)}")
        self.epoch += 1
        if self.epoch > 1:  # experts finished pulling our previous rows
            native.lib().p2p_wait_acks_raw(self.send_flags, self.send_acks, self.rank, 1, 0, self.epoch - 1)
        flat = expert_ids.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=self.E).to(torch.int32)
        offs = torch.cumsum(counts, 0, dtype=torch.int32) - counts
        tbl = self._table()
        tbl[:self.E].copy_(counts)
        tbl[self.E:].copy_(offs)
        torch.index_select(x, 0, order // k, out=self._send())
        pos = torch.empty_like(order)
        pos[order] = torch.arange(order.numel(), device=order.device)
        native.lib().p2p_publish_raw(self.send_flags, self.send_acks, self.rank, 1, 0, self.epoch)
        return pos.view(T, k).to(torch.int32)

    def experts(self, w_gate_up: list[torch.Tensor], w_down: list[torch.Tensor]) -> None:
        """Expert side: the two fused GEMMs for this rank's ``E/world`` experts."""
        from flextensor_b200.ops.api import _count

        W, P = self.world, self.heap.ptrs
        lib = native.lib()
        tables = [p + self.tbl_off for p in P]
        lib.moe_gemm(True, self.rank, self.el, self.d, self.f, self.max_rows, [p + self.send_off for p in P], tables,
                     self.send_flags[self.rank], 1, [a + 8 * self.rank for a in self.send_acks], self.a_local,
                     self.h_local, list(w_gate_up), [], [], self.epoch, self.counters)
        lib.moe_gemm(False, self.rank, self.el, self.d, self.f, self.max_rows, [], tables,
                     self.send_flags[self.rank], 1, [], self.a_local, self.h_local, list(w_down),
                     [p + self.comb_off for p in P], [c + 8 * self.rank for c in self.comb_flags], self.epoch,
                     self.counters)
        _count(2)

    def combine(self, pos: torch.Tensor, weights: torch.Tensor, residual: torch.Tensor | None,
                out: torch.Tensor) -> torch.Tensor:
        from flextensor_b200.ops.api import _count

        native.lib().moe_reduce(self._comb(), pos, weights.float().contiguous(), residual, out,
                                self.comb_flags[self.rank], 1, self.world, self.rank, self.epoch)
        _count()
        return out

    def close(self) -> None:
        import torch.distributed as dist

        if self.heap is None:
            return
        torch.cuda.synchronize(self.device)
        if self.epoch:
            native.lib().p2p_wait_acks_raw(self.send_flags, self.send_acks, self.rank, 1, 0, self.epoch)
        torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        self.heap.close()
        self.heap = None


class NcclExpertParallel:
    """Baseline: NCCL all-to-all dispatch / combine around per-expert GEMMs."""

    def __init__(self, n_experts: int, group=None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.E = n_experts
        self.el = n_experts // self.world

    def __call__(self, x, expert_ids, weights, w_gate_up, w_down, residual):
        import torch.distributed as dist

        from flextensor_b200 import ops

        T, k = expert_ids.shape
        flat = expert_ids.reshape(-1)
        order = torch.argsort(flat, stable=True)
        send = x.index_select(0, order // k)
        counts = torch.bincount(flat, minlength=self.E)
        per_rank = counts.view(self.world, self.el).sum(1)
        recv_counts = torch.empty_like(per_rank)
        dist.all_to_all_single(recv_counts, per_rank, group=self.group)
        sc, rc = per_rank.tolist(), recv_counts.tolist()
        recv = torch.empty(sum(rc), x.shape[1], dtype=x.dtype, device=x.device)
        dist.all_to_all_single(recv, send, rc, sc, group=self.group)
        # expert ids of the received rows: exchange the per-expert counts too
        cnt_all = torch.empty(self.world, self.E, dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(cnt_all, counts, group=self.group)
        mine = cnt_all[:, self.rank * self.el:(self.rank + 1) * self.el]   # [src, local expert]
        out = torch.empty_like(recv)
        start = 0
        for src in range(self.world):
            for j in range(self.el):
                n = int(mine[src, j])
                if n:
                    seg = recv[start:start + n]
                    h = ops.linear_swiglu(seg, w_gate_up[j])
                    out[start:start + n] = ops.linear(h, w_down[j], None, epi="none")
                start += n
        back = torch.empty_like(send)
        dist.all_to_all_single(back, out, sc, rc, group=self.group)
        pos = torch.empty_like(order)
        pos[order] = torch.arange(order.numel(), device=order.device)
        y = back.index_select(0, pos).view(T, k, -1)
        return (residual.float() + (y.float() * weights.unsqueeze(-1)).sum(1)).to(x.dtype)
