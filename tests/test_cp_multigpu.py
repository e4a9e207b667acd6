"""Context-parallel DiT forward on 2 GPUs: the fused path (K/V all-gather inside the attention
kernel over NVLink) and the Ulysses NCCL path must reproduce the single-GPU output."""

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
    from flextensor_b200.ops import native
    from flextensor_b200.parallel.cp import ContextParallel, UlyssesAttention

    dev = torch.device("cuda", rank)
    cfg = tiny_config(num_layers=3, num_heads=2, dim=256)
    m = WanDiT(cfg, impl="fused").to(dev).to(torch.bfloat16)
    init_wan_params_(m, seed=0)
    g = torch.Generator(device=dev).manual_seed(1)
    lat = torch.randn(1, cfg.in_channels, 4, 16, 16, device=dev, generator=g).bfloat16()   # 256 tokens
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16()
    t = torch.tensor([300.0], device=dev)
    tokens = 4 * 8 * 8
    cp = ContextParallel(tokens, kv_heads=cfg.num_heads)
    with torch.no_grad():
        want = m(lat, t, ctx).float()
        errs = []
        for _ in range(3):  # several calls: slots alternate, epochs advance, acks gate reuse
            got = m(lat, t, ctx, cp=cp).float()
            errs.append(float((got - want).abs().max()))
        m.set_impl("torch")
        want_t = m(lat, t, ctx).float()
        got_u = m(lat, t, ctx, cp=UlyssesAttention()).float()
        err_u = float((got_u - want_t).abs().max())
        # gather-KV cross-attention: 200 replicated "audio" queries over the sequence-sharded
        # keys / values (each rank contributes its shard; the kernel gathers the rest)
        gk = torch.Generator(device=dev).manual_seed(9)
        Hk = cfg.num_heads
        k_full = torch.randn(1, tokens, Hk, 128, device=dev, generator=gk).bfloat16()
        v_full = torch.randn(1, tokens, Hk, 128, device=dev, generator=gk).bfloat16()
        qa = torch.randn(1, 200, Hk, 128, device=dev, generator=gk).bfloat16()
        sh = tokens // world
        rows = slice(rank * sh, (rank + 1) * sh)
        errs_g = []
        for _ in range(2):
            og = cp.gather_kv_attention(qa, k_full[0, rows], v_full[0, rows]).float()
            ref = torch.nn.functional.scaled_dot_product_attention(
                qa.float().transpose(1, 2), k_full.float().transpose(1, 2), v_full.float().transpose(1, 2)
            ).transpose(1, 2)
            errs_g.append(float((og - ref).abs().max()))
    torch.cuda.synchronize()
    err_word = native.device_error(reset=True)
    cp.close()
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, max(errs), err_u, err_word, float(want.abs().max()), max(errs_g)))


def _worker(rank, world, port, q):
    try:
        _worker_body(rank, world, port, q)
    except BaseException:  # report instead of leaving the parent waiting on the queue
        import traceback

        q.put((rank, "error", traceback.format_exc()))
        raise


def test_cp_dit_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=300) for _ in ps), key=lambda t: t[0])
    for r in res:
        assert r[1] != "error", f"rank {r[0]} failed:\n{r[2]}"
    for p in ps:
        p.join(60)
    for rank, err, err_u, word, scale, err_g in res:
        assert word == 0, f"rank {rank}: device error word {word}"
        assert err_g < 2e-2, f"rank {rank}: gather-KV cross-attention max abs err {err_g}"
        assert err < 0.03 * max(1.0, scale), f"rank {rank}: fused CP max abs err {err} (output scale {scale})"
        assert err_u < 0.03 * max(1.0, scale), f"rank {rank}: Ulysses max abs err {err_u}"
