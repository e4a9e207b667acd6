"""Tensor-parallel Wan DiT on 2 GPUs (heads and FFN columns split): the fused path
(sequence-parallel residual, all-gather inside the column-parallel GEMMs, reduce-scatter from the
row-parallel GEMM epilogues, distributed Q/K RMSNorm over peer stores) and the NCCL baseline
(the reference driver's all_reduce layout) must both reproduce the unsharded model."""

import copy
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
    from flextensor_b200.models.wan_tp import WanTensorParallel
    from flextensor_b200.ops import native

    dev = torch.device("cuda", rank)
    cfg = tiny_config(dim=512, ffn_dim=1024, num_heads=4, num_layers=2)
    full = WanDiT(cfg).to(dev)
    init_wan_params_(full, seed=0)
    with torch.no_grad():  # non-trivial Q/K norm weights, so the weight shards are exercised
        for n, p in full.named_parameters():
            if "norm_q" in n or "norm_k" in n:
                p.uniform_(0.5, 1.5)
    full = full.to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    lat = torch.randn(1, cfg.in_channels, 2, 16, 16, device=dev, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16()
    t = torch.tensor([700.0], device=dev)
    S = 2 * 8 * 8
    errs = {}
    with torch.no_grad():
        ref = full(lat, t, ctx).float()
        for impl in ("fused", "nccl"):
            tp = WanTensorParallel(copy.deepcopy(full), impl=impl, max_tokens=S)
            for _ in range(2):  # twice: slots alternate and acknowledgements gate their reuse
                out = tp(lat, t, ctx).float()
            errs[impl] = float((out - ref).abs().max() / ref.abs().max())
            torch.cuda.synchronize()
            tp.close()
    word = native.device_error(reset=True)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, errs, word))


def _worker(rank, world, port, q):
    try:
        _worker_body(rank, world, port, q)
    except BaseException:  # report instead of leaving the parent waiting on the queue
        import traceback

        q.put((rank, "error", traceback.format_exc()))
        raise


def test_tp_wan_two_ranks():
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
    for rank, errs, word in res:
        assert word == 0, f"rank {rank}: device error {word}"
        assert errs["fused"] < 3e-2, f"rank {rank}: fused TP rel err {errs['fused']}"
        assert errs["nccl"] < 3e-2, f"rank {rank}: NCCL TP rel err {errs['nccl']}"
