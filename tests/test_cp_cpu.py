"""Ulysses (all-to-all) context parallelism of the DiT on CPU with 2 gloo ranks: the sharded
model must reproduce the single-process output."""

import os
import socket

import torch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
    from flextensor_b200.parallel.cp import UlyssesAttention

    cfg = tiny_config(num_layers=2, num_heads=2, dim=256)
    m = WanDiT(cfg, impl="torch")
    init_wan_params_(m, seed=0)
    g = torch.Generator().manual_seed(1)
    lat = torch.randn(1, cfg.in_channels, 2, 8, 8, generator=g)
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g)
    t = torch.tensor([300.0])
    with torch.no_grad():
        want = m(lat, t, ctx)
        got = m(lat, t, ctx, cp=UlyssesAttention())
    q.put((rank, float((got - want).abs().max())))
    dist.destroy_process_group()


def test_ulysses_cp_matches_single_process():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(30)
    for rank, err in res:
        assert err < 1e-4, f"rank {rank}: max abs err {err}"
