"""Address wiring of the tensor-parallel signalling (8 emulated ranks, CPU only): for every
sender / owner pair and both double-buffer slots, the flag word a sender writes is the one the
owner polls, and the acknowledgement an owner writes is the one the sender waits on
(``p2p_wait_acks`` reads ``acks[own][peer * N_SLOTS + slot]``, ``p2p_publish`` writes
``flags[peer][own * N_SLOTS + slot]``). The kernels are replaced by recorders."""

import pytest
import torch

from flextensor_b200.parallel import tp as T
from flextensor_b200.parallel.symm import SymmetricHeap

W = 8
HEAP = [0x10_0000_0000 * (r + 1) for r in range(W)]  # fake heap bases, one per rank


_T = torch.zeros(4, 8)  # stands in for every tensor argument: only the wiring is checked


class _Heap(SymmetricHeap):
    """Peer pointers only (no device memory): ``SymmetricHeap.__init__`` is not run."""

    def __init__(self):
        self.ptrs = HEAP


def _obj(cls, rank, **extra):
    o = cls.__new__(cls)
    o.rank, o.world, o.heap = rank, W, _Heap()
    o.f = T._Flags(o.heap, W)
    o.epochs, o.calls = [0] * T.N_SLOTS, 0
    o.__dict__.update(extra)
    return o


def _flag_written_by_publisher(publisher, reader, slot):  # p2p_publish / kernel flag stores
    return T._Flags(_Heap(), W).flags[reader] + (publisher * T.N_SLOTS + slot) * 8


def _ack_waited_by(owner_of_ack_array, peer, slot):  # p2p_wait_acks
    return T._Flags(_Heap(), W).acks[owner_of_ack_array] + (peer * T.N_SLOTS + slot) * 8


@pytest.mark.parametrize("slot", [0, 1])
def test_reduce_scatter_flags_and_acks_meet(monkeypatch, slot):
    sent, polled = {}, {}
    import flextensor_b200.ops.api as api

    monkeypatch.setattr(api, "tp_gemm_reducescatter",
                        lambda a, w, *, stage, peer_flags, rank, epoch, counters, **kw: (sent.setdefault(rank, peer_flags), _T)[1])
    monkeypatch.setattr(api, "tp_reduce", lambda stage, world, rows, out, *, flags_ptr, flag_stride, peer_acks, rank,
                        **kw: (polled.setdefault(rank, (flags_ptr, flag_stride, peer_acks)), _T)[1])
    for r in range(W):
        o = _obj(T.TPReduceScatter, r, M=W * 4, N=8, R=4, counters=None, off=[4096, 8192], slot_bytes=4096,
                 _cur=None)
        o._stage = lambda s: None
        o.calls = slot
        o.gemm(_T, _T)
        o.reduce(_T)
    for owner in range(W):
        flags_ptr, stride, acks = polled[owner]
        for sender in range(W):
            assert sent[sender][owner] == flags_ptr + sender * stride * 8  # what the owner polls
            assert sent[sender][owner] == _flag_written_by_publisher(sender, owner, slot)
            assert acks[sender] == _ack_waited_by(sender, owner, slot)


@pytest.mark.parametrize("slot", [0, 1])
def test_all_gather_flags_and_acks_meet(monkeypatch, slot):
    seen = {}
    import flextensor_b200.ops.api as api

    monkeypatch.setattr(api, "tp_allgather_gemm", lambda a, w, *, peer_a, flags_ptr, flag_stride, peer_acks, rank,
                        epoch, counters, **kw: (seen.setdefault(rank, (flags_ptr, flag_stride, peer_acks)), _T)[1])
    for r in range(W):
        o = _obj(T.TPAllGather, r, M=W * 4, K=8, R=4, counters=None, off=[4096, 8192], slot_bytes=4096)
        o._cur = (slot, 1)
        o._buf = lambda s: None
        o.gemm(_T)
    for reader in range(W):
        flags_ptr, stride, acks = seen[reader]
        for pub in range(W):
            # the reader polls the word the publisher's p2p_publish writes into the reader's flags
            assert flags_ptr + pub * stride * 8 == _flag_written_by_publisher(pub, reader, slot)
            # the reader's ack lands where the publisher's p2p_wait_acks looks for this reader
            assert acks[pub] == _ack_waited_by(pub, reader, slot)


@pytest.mark.parametrize("slot", [0, 1])
def test_distributed_rmsnorm_flags_and_acks_meet(monkeypatch, slot):
    seen = {}
    import flextensor_b200.ops.api as api

    monkeypatch.setattr(api, "tp_rmsnorm", lambda x, w, **kw: (seen.setdefault(kw["rank"], kw), _T)[1])
    monkeypatch.setattr(T.native, "lib", lambda: type("L", (), {"p2p_wait_acks_raw": staticmethod(lambda *a: None)}))
    for r in range(W):
        o = _obj(T.TPRMSNorm, r, stage_rows=64, off=[4096, 8192], counter=None)
        o.calls = slot
        o(torch.zeros(4, 8), None, 64)
    for owner in range(W):
        kw = seen[owner]
        for sender in range(W):
            assert seen[sender]["peer_flags"][owner] == kw["flags_ptr"] + sender * kw["flag_stride"] * 8
            assert kw["peer_acks"][sender] == _ack_waited_by(sender, owner, slot)
            assert seen[sender]["part_peers"][owner] == HEAP[owner] + [4096, 8192][slot]
