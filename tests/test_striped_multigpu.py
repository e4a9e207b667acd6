"""Striped host streaming on 2+ GPUs: each rank copies 1/N of every block over PCIe and pulls the
rest from its peers over NVLink; outputs must equal the all-resident model bitwise."""

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


def _worker(rank, world, port, q, on_device, gather="ce"):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", FT_STRIPED_GATHER=gather)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import flextensor_b200 as ft
    from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
    from flextensor_b200.ops import native
    from flextensor_b200.parallel import enable_striped_streaming
    from flextensor_b200.planner import NthLayerStrategy

    dev = torch.device("cuda", rank)
    cfg = tiny_config(num_layers=4)
    torch.manual_seed(0)
    m = WanDiT(cfg, impl="fused").to(torch.bfloat16)
    init_wan_params_(m, seed=0)
    ref = WanDiT(cfg, impl="fused").to(torch.bfloat16)
    ref.load_state_dict(m.state_dict())
    ref = ref.to(dev)
    lat = torch.randn(1, cfg.in_channels, 2, 16, 16, device=dev, dtype=torch.bfloat16)
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, dtype=torch.bfloat16)
    ts = torch.tensor([77.0], device=dev)
    with torch.no_grad():
        want = ref(lat, ts, ctx)
    if on_device:
        m = m.to(dev)  # device-resident source: packed stripe by stripe straight from the GPU
    enable_striped_streaming()
    om = ft.get_offload_manager()
    mm = om.offload(m, ft.OffloadConfig(gpu_device=rank, include_patterns=["blocks.*"], skip_discovery=True,
                                        profiling_iters=1, num_blocks=2, min_blocks=2,
                                        load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True)))
    ok = True
    with torch.no_grad():
        for _ in range(5):
            ok &= bool(torch.equal(mm(lat, ts, ctx), want))
    torch.cuda.synchronize()
    loader = om.get_tensor_manager().loader
    engine = f"{type(loader.engine).__name__}/{loader.engine.gather}"
    stripe_only = all(b.stripe_only for b in loader.plan.host_blocks.values()) and bool(loader.plan.host_blocks)
    err = native.device_error(reset=True)
    dist.barrier()
    om.release()  # preserve_model: every parameter comes back to the host, whole
    want_sd = {k: v.cpu() for k, v in ref.state_dict().items()}
    restored = all(torch.equal(v.cpu(), want_sd[k]) for k, v in m.state_dict().items())
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, ok, engine, err, stripe_only, restored))


@pytest.mark.parametrize("gather", ["sm", "ce"])
@pytest.mark.parametrize("on_device", [False, True], ids=["host_source", "device_source_stripe_only"])
def test_striped_streaming_two_ranks(on_device, gather):
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, on_device, gather)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(60)
    for rank, ok, engine, err, stripe_mode_ok, restored in res:
        assert engine == f"StripedTransferEngine/{gather}"
        assert err == 0
        assert ok, f"rank {rank} output differs from the resident model"
        assert stripe_mode_ok, f"rank {rank}: host blocks are not stripe-only"
        assert restored, f"rank {rank}: release() did not give back the original weights"
