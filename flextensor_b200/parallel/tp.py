"""Tensor parallelism inside one node with the collectives fused into the GEMMs.

Sequence-parallel layout (Megatron style): between layers every rank holds 1/N of the token
rows of the residual stream. A column-parallel projection needs all rows
(:class:`TPAllGather` -> ``tp_allgather_gemm``: the kernel pulls peers' rows over NVLink
while multiplying); a row-parallel projection produces partial sums of all rows that must be
reduced onto the rows' owners (:class:`TPReduceScatter` -> ``tp_gemm_reducescatter`` stores
each partial row straight into its owner's staging slot; the owner's ``tp_reduce`` adds the N
partials and the residual).

Both objects double-buffer their symmetric-heap slots and gate reuse with epoch flags and
acknowledgements (bounded device-side waits), so consecutive layers never wait on the host.
:class:`TPAllReduce` is the GEMM + all-reduce form for layers whose output stays replicated,
and :class:`TPRMSNorm` the RMSNorm over a head-sharded hidden dimension (partial sums of squares
over peer stores). :class:`NcclTP` and :func:`nccl_rmsnorm` are the unfused baselines
(``all_gather_into_tensor`` + GEMM, GEMM + ``reduce_scatter_tensor``, ``all_reduce`` of the sums).
"""

from __future__ import annotations

import torch

from flextensor_b200.ops import native
from flextensor_b200.parallel.symm import SymmetricHeap

N_SLOTS = 2


class _Flags:
    def __init__(self, heap: SymmetricHeap, world: int, offset: int = 0):
        self.bytes = world * N_SLOTS * 8
        self.flags = [p + offset for p in heap.ptrs]
        self.acks = [p + offset + self.bytes for p in heap.ptrs]


class TPAllGather:
    """Full ``[M, K]`` activation buffers; this rank writes rows ``[rank*R, (rank+1)*R)``."""

    def __init__(self, rows_total: int, k: int, group=None, device: int | None = None, pair: bool = False):
        import torch.distributed as dist

        self.group = group
        self.pair = pair  # experimental CTA-pair (cta_group::2) kernel
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if rows_total % self.world:
            raise ValueError(f"{rows_total} rows do not split over {self.world} ranks")
        self.M, self.K, self.R = rows_total, k, rows_total // self.world
        dev = torch.cuda.current_device() if device is None else device
        hdr = 4096
        self.slot_bytes = (rows_total * k * 2 + 4095) // 4096 * 4096
        self.heap = SymmetricHeap(hdr + N_SLOTS * self.slot_bytes, group, dev)
        self.f = _Flags(self.heap, self.world)
        self.off = [hdr + s * self.slot_bytes for s in range(N_SLOTS)]
        from flextensor_b200.ops.api import tp_ag_counter_words

        self.counters = torch.zeros(tp_ag_counter_words(rows_total, self.world), dtype=torch.int32,
                                    device=f"cuda:{dev}")
        self.epochs = [0] * N_SLOTS
        self.calls = 0
        self._cur = None
        dist.barrier(group=group)

    def _buf(self, slot: int) -> torch.Tensor:
        return self.heap.view(self.off[slot], self.M * self.K * 2).view(torch.bfloat16).view(self.M, self.K)

    def begin(self) -> torch.Tensor:
        """Claim the next slot; returns this rank's rows ``[R, K]`` to write into."""
        slot = self.calls % N_SLOTS
        self.calls += 1
        self.epochs[slot] += 1
        e = self.epochs[slot]
        if e > 1:  # peers finished pulling our rows of this slot's previous use
            native.lib().p2p_wait_acks_raw(self.f.flags, self.f.acks, self.rank, N_SLOTS, slot, e - 1)
        self._cur = (slot, e)
        return self._buf(slot)[self.rank * self.R:(self.rank + 1) * self.R]

    def publish(self) -> None:
        slot, e = self._cur
        native.lib().p2p_publish_raw(self.f.flags, self.f.acks, self.rank, N_SLOTS, slot, e)

    def full(self) -> torch.Tensor:
        """The current slot's ``[M, K]`` buffer: after :meth:`gemm` it holds every rank's rows,
        so further GEMMs on the same activations (K and V after Q) need no second gather."""
        return self._buf(self._cur[0])

    def gemm(self, weight: torch.Tensor, bias: torch.Tensor | None = None, epi: str = "none",
             out: torch.Tensor | None = None) -> torch.Tensor:
        from flextensor_b200.ops.api import tp_allgather_gemm

        slot, e = self._cur
        return tp_allgather_gemm(
            self._buf(slot), weight, peer_a=[p + self.off[slot] for p in self.heap.ptrs],
            flags_ptr=self.f.flags[self.rank] + slot * 8, flag_stride=N_SLOTS,
            peer_acks=[self.f.acks[p] + (self.rank * N_SLOTS + slot) * 8 for p in range(self.world)],
            rank=self.rank, epoch=e, counters=self.counters, bias=bias, epi=epi, out=out,
            _pair=getattr(self, "pair", False))

    def close(self) -> None:
        _close(self)


class TPReduceScatter:
    """Staging ``[world, R, N]`` per slot on every rank; rank r owns output rows ``[r*R, (r+1)*R)``."""

    def __init__(self, rows_total: int, n: int, group=None, device: int | None = None, pair: bool = False):
        import torch.distributed as dist

        self.group = group
        self.pair = pair  # experimental CTA-pair (cta_group::2) kernel
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if rows_total % self.world:
            raise ValueError(f"{rows_total} rows do not split over {self.world} ranks")
        self.M, self.N, self.R = rows_total, n, rows_total // self.world
        dev = torch.cuda.current_device() if device is None else device
        hdr = 4096
        self.slot_bytes = (self.world * self.R * n * 2 + 4095) // 4096 * 4096
        self.heap = SymmetricHeap(hdr + N_SLOTS * self.slot_bytes, group, dev)
        self.f = _Flags(self.heap, self.world)
        self.off = [hdr + s * self.slot_bytes for s in range(N_SLOTS)]
        self.counters = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
        self.epochs = [0] * N_SLOTS
        self.calls = 0
        self._cur = None
        dist.barrier(group=group)

    def _stage(self, slot: int) -> torch.Tensor:
        n = self.world * self.R * self.N
        return self.heap.view(self.off[slot], n * 2).view(torch.bfloat16).view(self.world, self.R, self.N)

    def gemm(self, a: torch.Tensor, weight: torch.Tensor) -> None:
        """Partial ``a [M, K] @ weight[N, K].T`` -> owners' staging slots (sender side)."""
        from flextensor_b200.ops.api import tp_gemm_reducescatter

        slot = self.calls % N_SLOTS
        self.calls += 1
        self.epochs[slot] += 1
        e = self.epochs[slot]
        if e > 1:  # every owner reduced (and acknowledged) this slot's previous use
            native.lib().p2p_wait_acks_raw(self.f.flags, self.f.acks, self.rank, N_SLOTS, slot, e - 1)
        self._cur = (slot, e)
        tp_gemm_reducescatter(a, weight, stage=[p + self.off[slot] for p in self.heap.ptrs],
                              peer_flags=[self.f.flags[p] + (self.rank * N_SLOTS + slot) * 8 for p in range(self.world)],
                              rank=self.rank, epoch=e, counters=self.counters, _pair=getattr(self, "pair", False))

    def reduce(self, out: torch.Tensor, residual: torch.Tensor | None = None, bias: torch.Tensor | None = None,
               gate: torch.Tensor | None = None, gate_rows: int = 0) -> torch.Tensor:
        """Owner side: ``out [R, N] = residual + gate * (sum of all ranks' partial rows + bias)``
        (``gate``: fp32 ``[groups, N]``, one row per ``gate_rows`` rows of the full sequence)."""
        from flextensor_b200.ops.api import tp_reduce

        slot, e = self._cur
        return tp_reduce(self._stage(slot), self.world, self.R, out, flags_ptr=self.f.flags[self.rank] + slot * 8,
                         flag_stride=N_SLOTS, epoch=e,
                         peer_acks=[self.f.acks[q] + (self.rank * N_SLOTS + slot) * 8 for q in range(self.world)],
                         rank=self.rank, residual=residual, bias=bias, gate=gate,
                         gate_rows=gate_rows or self.M, grow0=self.rank * self.R)

    def close(self) -> None:
        _close(self)


class TPAllReduce:
    """GEMM + all-reduce for row-parallel layers whose output is replicated (no sequence
    parallelism, e.g. vLLM's ``RowParallelLinear``): the partial rows go to their owners from the
    GEMM epilogue (reduce-scatter), each owner sums its rows and writes them into every rank's
    output buffer, and each rank waits for every owner's acknowledgement. Row counts may vary
    per call up to ``max_rows``; outputs are views of a double-buffered heap slot that stays
    valid until two calls later."""

    def __init__(self, max_rows: int, n: int, group=None, device: int | None = None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.max_rows, self.N = max_rows, n
        self.R_max = (max_rows + self.world - 1) // self.world
        dev = torch.cuda.current_device() if device is None else device
        hdr = 4096
        self.stage_bytes = (self.world * self.R_max * n * 2 + 4095) // 4096 * 4096
        self.out_bytes = (max_rows * n * 2 + 4095) // 4096 * 4096
        slot = self.stage_bytes + self.out_bytes
        self.heap = SymmetricHeap(hdr + N_SLOTS * slot, group, dev)
        self.f = _Flags(self.heap, self.world)
        self.stage_off = [hdr + s * slot for s in range(N_SLOTS)]
        self.out_off = [hdr + s * slot + self.stage_bytes for s in range(N_SLOTS)]
        self.counters = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
        self.epochs = [0] * N_SLOTS
        self.calls = 0
        dist.barrier(group=group)

    def __call__(self, a: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        from flextensor_b200.ops.api import tp_gemm_reducescatter, tp_reduce

        M = a.shape[0]
        if M > self.max_rows or weight.shape[0] != self.N:
            raise ValueError(f"TPAllReduce sized for {self.max_rows} x {self.N}, got {M} x {weight.shape[0]}")
        W, lib = self.world, native.lib()
        R = (M + W - 1) // W
        slot = self.calls % N_SLOTS
        self.calls += 1
        self.epochs[slot] += 1
        e = self.epochs[slot]
        if e > 1:
            lib.p2p_wait_acks_raw(self.f.flags, self.f.acks, self.rank, N_SLOTS, slot, e - 1)
        P = self.heap.ptrs
        tp_gemm_reducescatter(a, weight, stage=[p + self.stage_off[slot] for p in P],
                              peer_flags=[self.f.flags[p] + (self.rank * N_SLOTS + slot) * 8 for p in range(W)],
                              rank=self.rank, epoch=e, counters=self.counters)
        stage = self.heap.view(self.stage_off[slot], W * R * self.N * 2).view(torch.bfloat16).view(W, R, self.N)
        out = self.heap.view(self.out_off[slot], M * self.N * 2).view(torch.bfloat16).view(M, self.N)
        rows = max(0, min(R, M - self.rank * R))
        tp_reduce(stage, W, rows, out, flags_ptr=self.f.flags[self.rank] + slot * 8, flag_stride=N_SLOTS, epoch=e,
                  peer_acks=[self.f.acks[q] + (self.rank * N_SLOTS + slot) * 8 for q in range(W)], rank=self.rank,
                  out_peers=[p + self.out_off[slot] for p in P], row_base=self.rank * R, stage_rows=R)
        lib.p2p_wait_acks_raw(self.f.flags, self.f.acks, self.rank, N_SLOTS, slot, e)  # every owner's rows are in
        return out

    def close(self) -> None:
        _close(self)


class TPRMSNorm:
    """RMSNorm whose hidden dimension is split across the ranks (head-sharded Q/K norms of a
    tensor-parallel attention): each call sends the per-row partial sums of squares of this
    rank's columns to every rank over peer stores and scales the local columns once all ranks'
    partials are in; optional RoPE on the way out. Up to ``max_rows`` rows per call;
    double-buffered partial slots, reuse gated by acknowledgements (no host synchronisation)."""

    def __init__(self, max_rows: int, group=None, device: int | None = None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.stage_rows = max(32, (max_rows + 31) // 32 * 32)
        dev = torch.cuda.current_device() if device is None else device
        hdr = 4096
        self.slot_bytes = (self.world * self.stage_rows * 4 + 4095) // 4096 * 4096
        self.heap = SymmetricHeap(hdr + N_SLOTS * self.slot_bytes, group, dev)
        self.f = _Flags(self.heap, self.world)
        self.off = [hdr + s * self.slot_bytes for s in range(N_SLOTS)]
        self.counter = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
        self.epochs = [0] * N_SLOTS
        self.calls = 0
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor, weight: torch.Tensor | None, d_full: int, eps: float = 1e-6,
                 cos: torch.Tensor | None = None, sin: torch.Tensor | None = None, head_dim: int = 0,
                 seq_len: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        from flextensor_b200.ops.api import tp_rmsnorm

        rows = x.numel() // x.shape[-1]
        if rows > self.stage_rows:
            raise ValueError(f"TPRMSNorm sized for {self.stage_rows} rows, got {rows}")
        slot = self.calls % N_SLOTS
        self.calls += 1
        self.epochs[slot] += 1
        e = self.epochs[slot]
        if e > 1:  # every rank finished reading our partials of this slot's previous use
            native.lib().p2p_wait_acks_raw(self.f.flags, self.f.acks, self.rank, N_SLOTS, slot, e - 1)
        W = self.world
        return tp_rmsnorm(x, weight, d_full=d_full, part_peers=[p + self.off[slot] for p in self.heap.ptrs],
                          stage_rows=self.stage_rows,
                          peer_flags=[self.f.flags[q] + (self.rank * N_SLOTS + slot) * 8 for q in range(W)],
                          flags_ptr=self.f.flags[self.rank] + slot * 8, flag_stride=N_SLOTS,
                          peer_acks=[self.f.acks[q] + (self.rank * N_SLOTS + slot) * 8 for q in range(W)],
                          rank=self.rank, epoch=e, counter=self.counter, eps=eps, cos=cos, sin=sin,
                          head_dim=head_dim, seq_len=seq_len, out=out)

    def close(self) -> None:
        _close(self)


def nccl_rmsnorm(x: torch.Tensor, weight: torch.Tensor | None, d_full: int, eps: float = 1e-6, group=None):
    """Unfused baseline of :class:`TPRMSNorm`: partial sum of squares, NCCL all-reduce, scale."""
    import torch.distributed as dist

    ss = x.float().pow(2).sum(-1, keepdim=True)
    dist.all_reduce(ss, group=group)
    y = x.float() * torch.rsqrt(ss / d_full + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(x.dtype)


def _close(obj) -> None:
    import torch.distributed as dist

    if obj.heap is None:
        return
    torch.cuda.synchronize()
    for slot in range(N_SLOTS):
        if obj.epochs[slot]:
            native.lib().p2p_wait_acks_raw(obj.f.flags, obj.f.acks, obj.rank, N_SLOTS, slot, obj.epochs[slot])
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier(group=obj.group)
    obj.heap.close()
    obj.heap = None


class NcclTP:
    """Unfused baseline: NCCL all-gather / reduce-scatter around the same GEMM kernels."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)

    def all_gather(self, x_local: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        out = torch.empty(self.world * x_local.shape[0], *x_local.shape[1:], dtype=x_local.dtype,
                          device=x_local.device)
        dist.all_gather_into_tensor(out, x_local.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, partial: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        out = torch.empty(partial.shape[0] // self.world, *partial.shape[1:], dtype=partial.dtype,
                          device=partial.device)
        dist.reduce_scatter_tensor(out, partial.contiguous(), group=self.group)
        return out
