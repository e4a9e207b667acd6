"""Expert-parallel Mixtral layers on 2 GPUs (each rank its own tokens, half of the experts):
the fused dispatch/combine path and the NCCL all-to-all path must reproduce the single-GPU
model that holds every expert."""

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
    from flextensor_b200.models.mixtral import MixtralModel, init_mixtral_params_, tiny_mixtral
    from flextensor_b200.ops import native
    from flextensor_b200.parallel.ep import ExpertParallel, NcclExpertParallel

    dev = torch.device("cuda", rank)
    cfg = tiny_mixtral(n_layers=2)
    full = MixtralModel(cfg).to(dev)
    init_mixtral_params_(full, seed=0)
    full = full.to(torch.bfloat16)
    part = MixtralModel(cfg, rank=rank, world=world).to(dev)
    init_mixtral_params_(part, seed=0)
    part = part.to(torch.bfloat16)
    B, S = 2, 128
    tokens = torch.randint(0, cfg.vocab, (B, S), device=dev, generator=torch.Generator(device=dev).manual_seed(11 + rank))
    errs = {}
    with torch.no_grad():
        ref = full.hidden(tokens).float()
        ep = ExpertParallel(B * S, cfg.dim, cfg.ffn_dim, cfg.n_experts, cfg.topk)
        for _ in range(2):
            got = part.hidden(tokens, ep=ep).float()
        errs["fused"] = float((got - ref).abs().max() / ref.abs().max())
        torch.cuda.synchronize()
        ep.close()
        got = part.hidden(tokens, ep=NcclExpertParallel(cfg.n_experts)).float()
        errs["nccl"] = float((got - ref).abs().max() / ref.abs().max())
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


def test_ep_mixtral_two_ranks():
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
        assert errs["fused"] < 5e-2, f"rank {rank}: fused EP rel err {errs['fused']}"
        assert errs["nccl"] < 5e-2, f"rank {rank}: NCCL EP rel err {errs['nccl']}"
