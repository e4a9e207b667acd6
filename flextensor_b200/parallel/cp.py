"""Context parallelism for video DiTs: the sequence is split across the GPUs of one node and
self-attention runs on the local queries over the keys of every rank.

Data plane (no NCCL in the attention path): every rank holds, in a symmetric heap, two
full-sequence K/V buffers ``[2, S, H*128]`` (a K block, then a V block) (one per parity of the attention call, so a
call's rows stay readable while the next call is being projected). For each attention call:

1. ``begin()`` -- before the projections overwrite this rank's rows of the slot, wait (on the
   device, bounded) until every peer acknowledged the previous use of the slot;
2. the K and V projections write this rank's rows straight into the slot (GEMM output with a
   row stride), q/k RMSNorm + RoPE run in place;
3. ``publish()`` -- one thread stores the call's epoch into every peer's flag array;
4. ``attention()`` -- the fused kernel (``attention_sm100.cu``, CP variant) gathers the peers'
   rows into the local slot over NVLink while computing, and acknowledges each peer once its
   rows are local.

Replaces the reference's Ulysses all-to-all attention (``examples/ltx23/outpaint/
context_parallel.py:628-686``) and its gather-KV cross-attention (``:689-727``); the
all-to-all version is kept in :class:`UlyssesAttention` as the NCCL baseline.
"""

from __future__ import annotations

import torch

from flextensor_b200.ops import native
from flextensor_b200.parallel.symm import SymmetricHeap

N_SLOTS = 2


class ContextParallel:
    def __init__(self, seq_len: int, kv_heads: int, group=None, device: int | None = None, batch: int = 1):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if seq_len % self.world:
            raise ValueError(f"sequence length {seq_len} must be divisible by the CP size {self.world}")
        if batch != 1:
            raise ValueError("context-parallel buffers are laid out for batch 1 (run CFG halves as two calls)")
        self.seq_len = seq_len
        self.shard = seq_len // self.world
        self.kv_heads = kv_heads
        self.kv_dim = kv_heads * 128
        self.device = torch.cuda.current_device() if device is None else device
        slot_bytes = seq_len * 2 * self.kv_dim * 2
        self.flag_bytes = self.world * N_SLOTS * 8
        hdr = 4096 * ((2 * self.flag_bytes + 8 * self.world + 4095) // 4096)
        self.slot_off = [hdr + s * slot_bytes for s in range(N_SLOTS)]
        self.heap = SymmetricHeap(hdr + N_SLOTS * slot_bytes, group, self.device)
        self.flags = [p for p in self.heap.ptrs]                       # [world][N_SLOTS] u64 per rank
        self.acks = [p + self.flag_bytes for p in self.heap.ptrs]
        self.counters = torch.zeros(2 * self.world, dtype=torch.int32, device=f"cuda:{self.device}")
        self.epochs = [0] * N_SLOTS
        self.calls = 0
        self._cur: tuple[int, int] | None = None
        dist.barrier(group=group)

    # ------------------------------------------------------------------ buffers
    def slot_kv(self, slot: int) -> torch.Tensor:
        """The local full-sequence K/V buffer of ``slot`` as ``[2, S, kv_dim]`` bf16."""
        n = self.seq_len * 2 * self.kv_dim
        return self.heap.view(self.slot_off[slot], n * 2).view(torch.bfloat16).view(2, self.seq_len, self.kv_dim)

    def shard_rows(self, t: torch.Tensor, dim: int = 1) -> torch.Tensor:
        return t.narrow(dim, self.rank * self.shard, self.shard)

    # ------------------------------------------------------------------ protocol
    def begin(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Claim the next slot; returns this rank's (K rows, V rows) views ``[shard, kv_dim]``."""
        slot = self.calls % N_SLOTS
        self.calls += 1
        self.epochs[slot] += 1
        epoch = self.epochs[slot]
        if epoch > 1:
            native.lib().p2p_wait_acks_raw(self.flags, self.acks, self.rank, N_SLOTS, slot, epoch - 1)
        self._cur = (slot, epoch)
        kv = self.slot_kv(slot)
        rows = slice(self.rank * self.shard, (self.rank + 1) * self.shard)
        return kv[0, rows], kv[1, rows]

    def publish(self) -> None:
        slot, epoch = self._cur
        native.lib().p2p_publish_raw(self.flags, self.acks, self.rank, N_SLOTS, slot, epoch)

    def attention(self, q: torch.Tensor, scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """q ``[1, shard, Hq, 128]`` -> attention over all ranks' keys of the current slot."""
        from flextensor_b200.ops.api import attention_cp

        slot, epoch = self._cur
        kv = self.slot_kv(slot).view(1, 2, self.seq_len, self.kv_heads, 128)
        flags_local = self.flags[self.rank] + slot * 8           # entry of rank q at [q * N_SLOTS + slot]
        acks = [self.acks[p] + (self.rank * N_SLOTS + slot) * 8 for p in range(self.world)]
        return attention_cp(q, kv, peer_kv=[p + self.slot_off[slot] for p in self.heap.ptrs], flags_ptr=flags_local,
                            flag_stride=N_SLOTS, peer_acks=acks, rank=self.rank, shard_rows=self.shard,
                            epoch=epoch, counters=self.counters, scale=scale, out=out)

    def gather_kv_attention(self, q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                            scale: float | None = None) -> torch.Tensor:
        """Cross-attention of any queries ``q [1, Sq, Hq, 128]`` (e.g. replicated audio tokens)
        over keys/values that are sharded by sequence across the ranks (e.g. the video tokens):
        each rank contributes ``k_local / v_local [shard, kv_dim]`` and the fused kernel gathers
        the rest (the reference's gather-KV cross-attention, without an NCCL all-gather)."""
        kr, vr = self.begin()
        kr.copy_(k_local.reshape(self.shard, self.kv_dim))
        vr.copy_(v_local.reshape(self.shard, self.kv_dim))
        self.publish()
        return self.attention(q, scale=scale)

    def gather_sequence(self, x_local: torch.Tensor) -> torch.Tensor:
        """All-gather ``[B, shard, C]`` -> ``[B, S, C]`` (small tensors after the output head)."""
        import torch.distributed as dist

        parts = [torch.empty_like(x_local) for _ in range(self.world)]
        dist.all_gather(parts, x_local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def close(self) -> None:
        import torch.distributed as dist

        if self.heap is None:
            return
        torch.cuda.synchronize(self.device)
        for slot in range(N_SLOTS):  # peers must be done reading our rows before the heap goes
            if self.epochs[slot]:
                native.lib().p2p_wait_acks_raw(self.flags, self.acks, self.rank, N_SLOTS, slot, self.epochs[slot])
        torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        self.heap.close()
        self.heap = None


class UlyssesAttention:
    """NCCL baseline: all-to-all sequence<->heads, local attention over the full sequence on
    H/P heads, all-to-all back (the reference's Ulysses scheme). q/k/v ``[1, shard, H, 128]``."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)

    def _a2a(self, x: torch.Tensor, scatter_dim: int, gather_dim: int) -> torch.Tensor:
        import torch.distributed as dist

        send = torch.stack(x.chunk(self.world, dim=scatter_dim)).contiguous()  # [P, ...] chunk p -> rank p
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return torch.cat(recv.unbind(0), dim=gather_dim)

    def __call__(self, q, k, v, attn_fn):
        if q.shape[2] % self.world or k.shape[2] % self.world:
            raise ValueError("Ulysses needs heads divisible by the CP size")
        qh, kh, vh = (self._a2a(t, 2, 1) for t in (q, k, v))   # [1, S, H/P, 128]
        o = attn_fn(qh, kh, vh)
        return self._a2a(o, 1, 2)                               # back to [1, shard, H, 128]
