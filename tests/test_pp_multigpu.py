"""Pipeline-parallel Wan DiT on 2 GPUs: the blocks split into two stages on the fused sm_100a
kernels, activations over NCCL send/recv. Both ends must reproduce the unsplit model for every
micro-batch (same kernels on the same rows, so only non-deterministic reductions could differ)."""

import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 CUDA devices", allow_module_level=True)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker_body(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
    from flextensor_b200.models.wan_pp import WanPipelineParallel

    dev = torch.device("cuda", rank)
    cfg = tiny_config(dim=512, ffn_dim=1024, num_heads=4, num_layers=4)
    model = WanDiT(cfg).to(dev)
    init_wan_params_(model, seed=0)
    model = model.to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    lat = [torch.randn(1, cfg.in_channels, 2, 16, 16, device=dev, generator=g).bfloat16() for _ in range(3)]
    ctx = [torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16() for _ in range(3)]
    ts = [torch.tensor([300.0 * (i + 1)], device=dev) for i in range(3)]
    with torch.no_grad():
        ref = [model(lat[i], ts[i], ctx[i]).float() for i in range(3)]
    pp = WanPipelineParallel(model, depth=2)
    errs = []
    for _ in range(2):
        outs = pp(lat, ts, ctx)
        torch.cuda.synchronize()
        if outs is not None:
            errs.append(max(float((o.float() - r).abs().max() / r.abs().max()) for o, r in zip(outs, ref)))
    dist.barrier()
    for grp in (pp.groups.links[0], pp.groups.links[1], pp.groups.back):
        dist.destroy_process_group(grp)
    dist.destroy_process_group()
    q.put((rank, errs, len(model.blocks)))


def _worker(rank, world, port, q):
    try:
        _worker_body(rank, world, port, q)
    except BaseException:  # report instead of leaving the parent waiting on the queue
        import traceback

        q.put((rank, "error", traceback.format_exc()))
        raise


def test_pp_wan_two_stages():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=300) for _ in ps), key=lambda t: t[0])
    for p in ps:
        p.join(60)
    for r in res:
        assert r[1] != "error", f"rank {r[0]} failed:\n{r[2]}"
    assert [r[2] for r in res] == [2, 2]
    for rank, errs, _ in res:
        assert len(errs) == 2, rank
        assert max(errs) < 1e-2, f"rank {rank}: pipelined output differs from the unsplit model ({errs})"
