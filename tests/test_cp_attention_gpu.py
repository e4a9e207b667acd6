"""Context-parallel attention with the fused K/V all-gather, emulated on one GPU.

Each emulated rank owns a separate full-sequence K|V buffer holding only its own rows; every
peer's epoch flag is set before the single launch (so the kernel never waits on another
launch). The kernel must (1) compute softmax attention of the local queries over all ranks'
keys (fp32 reference), (2) leave the peers' rows gathered in the local buffer and (3) write the
epoch into every peer's ack word."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.ops import api as ops  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)


def _ref(q, k, v):
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    rep = qf.shape[1] // kf.shape[1]
    kf, vf = kf.repeat_interleave(rep, 1), vf.repeat_interleave(rep, 1)
    return torch.nn.functional.scaled_dot_product_attention(qf, kf, vf).transpose(1, 2)


def _setup(B, W, S_loc, Hq, Hk, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    Sk = W * S_loc
    k = torch.randn(B, Sk, Hk, 128, device=DEV, generator=g).bfloat16()
    v = torch.randn(B, Sk, Hk, 128, device=DEV, generator=g).bfloat16()
    q = torch.randn(B, S_loc, Hq, 128, device=DEV, generator=g).bfloat16()
    bufs = []
    for p in range(W):
        kv = torch.zeros(B, 2, Sk, Hk, 128, device=DEV, dtype=torch.bfloat16)
        rows = slice(p * S_loc, (p + 1) * S_loc)
        kv[:, 0, rows] = k[:, rows]
        kv[:, 1, rows] = v[:, rows]
        bufs.append(kv)
    return q, k, v, bufs


@pytest.mark.parametrize("B,W,S_loc,Hq,Hk,rank", [(1, 4, 300, 4, 4, 1), (2, 2, 256, 2, 2, 0), (1, 8, 130, 8, 2, 7),
                                                 (1, 3, 1000, 2, 2, 2)])
def test_cp_attention_matches_full_attention(B, W, S_loc, Hq, Hk, rank):
    q, k, v, bufs = _setup(B, W, S_loc, Hq, Hk, seed=W * 100 + rank)
    flags = torch.zeros(W, dtype=torch.int64, device=DEV)
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]  # acks[p][rank]
    counters = torch.zeros(2 * W, dtype=torch.int32, device=DEV)
    for epoch in (3, 4):  # twice in a row: scratch counters must be re-zeroed by the launcher
        if epoch == 4:  # fresh peer rows in the local buffer and new data
            q, k, v, bufs2 = _setup(B, W, S_loc, Hq, Hk, seed=epoch)
            for p in range(W):
                bufs[p].copy_(bufs2[p])
        flags.fill_(epoch)
        out = ops.attention_cp(q, bufs[rank], peer_kv=[b.data_ptr() for b in bufs], flags_ptr=flags.data_ptr(),
                               flag_stride=1, peer_acks=[a.data_ptr() + 8 * rank for a in acks], rank=rank,
                               shard_rows=S_loc, epoch=epoch, counters=counters)
        torch.cuda.synchronize()
        assert native.device_error(reset=True) == 0
        err = (out.float() - _ref(q, k, v)).abs().max().item()
        assert err < 2e-2, f"max abs err {err}"
        assert torch.equal(bufs[rank][:, 0], k) and torch.equal(bufs[rank][:, 1], v), "K/V not gathered"
        for p in range(W):
            if p != rank:
                assert int(acks[p][rank]) == epoch, f"peer {p} not acked"
