"""Host-side logic of striped streaming (no GPU): stripe layout, stripe-only packing and
process-group selection on a 2-rank gloo group."""

import os
import socket

import pytest
import torch

from flextensor_b200.core.host_store import pack_tensors, pack_tensors_stripe, stripe_len, stripe_range


def _items(seed=0):
    g = torch.Generator().manual_seed(seed)
    shapes = [(33, 17), (5,), (128, 64), (1,), (7, 3, 11)]
    return [(i, f"t{i}", torch.randn(*s, generator=g).to(torch.bfloat16)) for i, s in enumerate(shapes)]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_stripes_cover_the_packed_block(world):
    items = _items()
    full = pack_tensors("L", items, pinned=False)
    total = full.nbytes
    got = torch.zeros(total, dtype=torch.uint8)
    covered = 0
    for r in range(world):
        blk = pack_tensors_stripe("L", items, r, world, pinned=False)
        assert blk.nbytes == total and blk.stripe_only
        b0, b1 = blk.stripe
        assert (b0, b1) == stripe_range(total, r, world)
        assert b0 % 256 == 0
        got[b0:b1] = blk.data[: b1 - b0]
        covered += b1 - b0
        assert [(e.offset, e.nbytes) for e in blk.entries] == [(e.offset, e.nbytes) for e in full.entries]
    assert covered == total
    for e in full.entries:  # padding bytes between tensors are don't-care
        assert torch.equal(got[e.offset:e.offset + e.nbytes], full.data[e.offset:e.offset + e.nbytes])


def test_stripe_len_rule():
    assert stripe_len(1000, 4) == 256
    assert stripe_len(4096, 4) == 1024
    assert stripe_len(4097, 4) == 1280
    assert stripe_range(300, 3, 4) == (300, 300)  # ranks past the end hold nothing


def test_stripe_only_block_refuses_host_views():
    blk = pack_tensors_stripe("L", _items(), 0, 2, pinned=False)
    with pytest.raises(RuntimeError, match="one stripe"):
        blk.view(blk.entries[0])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _group_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from flextensor_b200.parallel import striped

    before = striped.striping_group()
    striped.enable_striped_streaming()
    g = striped.striping_group()
    striped.disable_striped_streaming()
    q.put((rank, before is None, g is not None and dist.get_world_size(g) == world))
    dist.destroy_process_group()


def test_striping_group_uses_default_group():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_group_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
    assert res == [(0, True, True), (1, True, True)]


def _wan_tp_shard_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
    from flextensor_b200.models.wan_tp import WanTensorParallel

    cfg = tiny_config(dim=512, ffn_dim=1024, num_heads=4, num_layers=1)
    m = WanDiT(cfg, impl="torch")
    init_wan_params_(m, seed=0)
    full = {n: p.detach().numpy().copy() for n, p in m.named_parameters()}  # numpy: pickled by value
    WanTensorParallel(m, impl="nccl")
    shards = {n: p.detach().numpy().copy() for n, p in m.named_parameters()}
    q.put((rank, full, shards))
    dist.destroy_process_group()


def test_wan_tensor_parallel_shards_cover_the_model():
    """Head/FFN sharding of the Wan blocks (the reference driver's col_shard / row_shard /
    DistRMSNorm layout): concatenating the 2 ranks' shards gives back every full tensor; row-
    parallel biases stay whole (added once after the reduction)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_wan_tp_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=120) for _ in ps), key=lambda t: t[0])
    for p in ps:
        p.join(30)
    full = {n: torch.from_numpy(a) for n, a in res[0][1].items()}
    s0 = {n: torch.from_numpy(a) for n, a in res[0][2].items()}
    s1 = {n: torch.from_numpy(a) for n, a in res[1][2].items()}
    for n, t in full.items():
        if ".blocks." not in f".{n}":
            assert torch.equal(s0[n], t) and torch.equal(s1[n], t), n
            continue
        leaf = n.split(".", 2)[2]
        if leaf.endswith("to_out.weight") or leaf == "ffn_out.weight":
            assert torch.equal(torch.cat([s0[n], s1[n]], 1), t), n
        elif leaf.endswith("to_out.bias") or leaf == "ffn_out.bias" or leaf.startswith("norm2") \
                or leaf == "scale_shift_table":
            assert torch.equal(s0[n], t) and torch.equal(s1[n], t), n
        else:
            assert torch.equal(torch.cat([s0[n], s1[n]], 0), t), n
