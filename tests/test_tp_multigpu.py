"""Tensor-parallel Llama layers on 2 GPUs: the fused all-gather->GEMM / GEMM->reduce-scatter
path and the NCCL baseline must both reproduce the single-GPU layers."""

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
    from flextensor_b200.models.llama import LlamaModel, LlamaTP, init_llama_params_, tiny_llama
    from flextensor_b200.ops import native

    dev = torch.device("cuda", rank)
    cfg = tiny_llama(n_layers=3)
    full = LlamaModel(cfg).to(dev)
    init_llama_params_(full, seed=0)
    full = full.to(torch.bfloat16)
    B, S = 2, 256
    M, R = B * S, B * S // world
    tokens = torch.randint(0, cfg.vocab, (B, S), device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    rope = full.rope(S, dev)
    errs = {}
    with torch.no_grad():
        x = full.embed(tokens).reshape(M, -1).contiguous()
        ref = x.clone()
        for L in full.layers:
            ref = L(ref, B, S, rope)
        for coll in ("fused", "nccl"):
            tp = LlamaTP(cfg, rank, world).to(dev).to(torch.bfloat16).load_from_full(full)
            tp.setup(M, collective=coll)
            for _ in range(2):  # twice: slots alternate and acks gate reuse
                xl = x[rank * R:(rank + 1) * R].clone()
                out = tp(xl, B, S, rope)
            errs[coll] = float((out.float() - ref[rank * R:(rank + 1) * R].float()).abs().max()
                               / ref.float().abs().max())
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


def test_tp_llama_two_ranks():
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
