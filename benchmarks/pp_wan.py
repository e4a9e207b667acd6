"""Pipeline-parallel Wan2.2-14B-shape DiT: ``--layers`` blocks split into N stages, ``--micro``
micro-batches per denoising step (2 = the classifier-free-guidance halves).

    torchrun --nproc-per-node N benchmarks/pp_wan.py [--layers 40] [--micro 2] [--iters 3]

Each rank holds only its stage's blocks, balanced by parameter bytes. One step runs every
micro-batch over the 32,760-token latent (81 frames at 480x832) through the pipeline; the
activations between stages go over NCCL send/recv while the next micro-batch computes.

Reports device ms per step (max over ranks, CUDA events). Rank 0 then runs the same
micro-batches through the whole model alone for comparison. The GPipe bound on the speed-up is
M*N / (M + N - 1) for M micro-batches on N stages, plus the activation bytes crossing each
stage boundary per step (a bf16 ``[tokens, dim]`` tensor per micro-batch).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _timed(fn, iters):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--micro", type=int, default=2)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--depth", type=int, default=2)
    ap.add_argument("--frames", type=int, default=21, help="latent frames (21 = 81 video frames)")
    a = ap.parse_args()
    import torch.distributed as dist

    from flextensor_b200.models.wan import WAN_14B, WanConfig, WanDiT, init_wan_params_
    from flextensor_b200.models.wan_pp import WanPipelineParallel

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = WanConfig(**{**WAN_14B.__dict__, "num_layers": a.layers})
    grid = (a.frames, 60, 104)
    S = grid[0] * (grid[1] // 2) * (grid[2] // 2)
    g = torch.Generator(device=dev).manual_seed(0)
    lat = [torch.randn(1, cfg.in_channels, *grid, device=dev, generator=g).bfloat16() for _ in range(a.micro)]
    ctx = [torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16() for _ in range(a.micro)]
    ts = [torch.tensor([500.0], device=dev) for _ in range(a.micro)]

    def build():
        with torch.device("meta"):
            m = WanDiT(cfg)
        return m

    m = build()
    pp = WanPipelineParallel(m, depth=a.depth)  # drops the other stages' blocks while still on meta
    m = m.to(torch.bfloat16).to_empty(device=dev)
    init_wan_params_(m, seed=0)
    m.eval().requires_grad_(False)
    res = {"n_gpus": W, "tokens": S, "layers": a.layers, "micro_batches": a.micro, "stages": pp.bounds}
    with torch.no_grad():
        for _ in range(2):
            pp(lat, ts, ctx)
        torch.cuda.synchronize()
        dist.barrier()
        ms = torch.tensor([_timed(lambda: pp(lat, ts, ctx), a.iters)], device=dev, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    res["pp_ms_per_step"] = round(float(ms.item()), 3)
    del pp, m
    torch.cuda.empty_cache()
    dist.barrier()
    if rank == 0:
        full = build().to_empty(device=dev).to(torch.bfloat16)
        init_wan_params_(full, seed=0)
        full.eval().requires_grad_(False)

        def step():
            for i in range(a.micro):
                full(lat[i], ts[i], ctx[i])

        with torch.no_grad():
            for _ in range(2):
                step()
            torch.cuda.synchronize()
            one = _timed(step, a.iters)
        res["single_gpu_ms_per_step"] = round(one, 3)
        res["speedup_vs_single_gpu"] = round(one / res["pp_ms_per_step"], 3)
        res["gpipe_bound"] = round(a.micro * W / (a.micro + W - 1), 3)
        res["boundary_bytes_per_step"] = a.micro * S * cfg.dim * 2
        print(json.dumps(res))
        del full
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
