"""End to end: LTX-shape video DiT with context parallelism, weights offloaded.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        benchmarks/e2e_ltx_cp.py [--impl ours|reference] [--steps K] [--warmup W]

Model: 48 blocks, d=4096, 32 heads, FFN 16384, cross-attention to 256 text tokens of dim 4096;
128-channel latent 46x22x40 = 40,480 tokens, sequence-sharded over the N ranks; random-init
bf16 weights, synthetic N(0,1) inputs. 50 % of the weight bytes may stay on each GPU; the
rest is streamed from host memory every denoise step.

* ``ours``: ``flextensor_b200`` -- fused tcgen05 kernels, the K/V all-gather fused into the
  attention kernel over NVLink (``ContextParallel``), and striped host streaming (every rank
  holds the same weights, so each copies 1/N of every block over its own host link and the
  rest comes from its peers).
* ``reference``: the unmodified reference runtime (``baseline/_ref``) offloading the same
  architecture in plain PyTorch (``baseline/wan_torch.py``: cuBLAS, SDPA) with Ulysses
  all-to-all sequence parallelism over NCCL -- the reference's own LTX scheme.

One JSON line (rank 0): seconds per denoise step (CUDA events, max over ranks), peak GPU GB,
% of transfer time hidden, clocks.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402  (shared harness: clocks, process group, arm import, offload config)

GRID = (46, 22, 40)
TOKENS = GRID[0] * GRID[1] * GRID[2]
RESIDENT = 0.5


def build(impl: str, layers: int, device, world: int, host_fits=None):
    import torch

    if impl == "ours":
        from flextensor_b200.models.ltx import LTX_CP_CONFIG
        from flextensor_b200.models.wan import WanConfig, WanDiT, init_wan_params_

        cfg = WanConfig(**{**LTX_CP_CONFIG.__dict__, "num_layers": layers})
        with torch.device("meta"):
            model = WanDiT(cfg, impl="fused")
        init = init_wan_params_
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        from wan_torch import WanShape, WanTorchDiT, init_params_

        cfg = WanShape(dim=4096, ffn_dim=16384, num_heads=32, num_layers=layers, text_dim=4096, text_len=256,
                       freq_dim=256, in_channels=128, out_channels=128, patch=(1, 1, 1))
        with torch.device("meta"):
            model = WanTorchDiT(cfg)
        init = init_params_
    if host_fits is not None and not host_fits(model):
        return None, cfg
    model = model.to(torch.bfloat16).to_empty(device=device)  # bf16 before any bytes exist
    init(model, seed=0)
    if impl == "reference":
        bench.to_pageable(model)
    model.eval()
    model.requires_grad_(False)
    return model, cfg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--profiling-iters", type=int, default=3)
    a = ap.parse_args()
    import torch

    rss0 = bench._rss_bytes()
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank, world, local, pg = bench.dist_setup(world)
    device = torch.device("cuda", local)
    ft, why = bench.import_arm(a.impl)
    if ft is None:
        if rank == 0:
            print(json.dumps({"impl": a.impl, "unavailable": why}))
        return
    if world > 1 and a.impl == "ours":
        from flextensor_b200.parallel import enable_striped_streaming

        enable_striped_streaming()
    def host_fits(meta_model) -> bool:
        ok, why = bench.host_gate(pg, bench.host_need_bytes(meta_model, a.impl, 1 - RESIDENT, "blocks."), world,
                                  bench.host_start_bytes(meta_model, a.impl))
        if not ok and rank == 0:
            print(json.dumps({"impl": a.impl, "n_gpus": world, "unavailable": why}))
        return ok

    model, cfg = build(a.impl, a.layers, device, world, host_fits)
    if model is None:
        return bench.close_dist(pg)
    total = sum(p.numel() * p.element_size() for p in model.parameters())
    frac = RESIDENT * total / torch.cuda.get_device_properties(device).total_memory
    om = ft.get_offload_manager()
    rss_built = bench._rss_bytes()
    model = om.offload(model, bench.make_config(ft, local, frac, a.profiling_iters))
    rss_offloaded = bench._rss_bytes()
    cp = None
    if world > 1:
        if a.impl == "ours":
            from flextensor_b200.parallel.cp import ContextParallel

            cp = ContextParallel(TOKENS, kv_heads=cfg.num_heads)
        else:
            from wan_torch import Ulysses

            cp = Ulysses()
    g = torch.Generator(device=device).manual_seed(7)
    lat = torch.randn(1, cfg.in_channels, *GRID, device=device, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=device, generator=g).bfloat16()
    ts = torch.tensor([500.0], device=device)

    def step():
        return model(lat, ts, ctx, cp=cp) if cp is not None else model(lat, ts, ctx)

    t0 = time.perf_counter()
    with torch.no_grad():
        for _ in range(om.iters_before_inference):
            step()
        for _ in range(a.warmup):
            step()
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t0
    rss_setup = bench._rss_bytes()
    torch.cuda.reset_peak_memory_stats(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    clocks = bench.ClockSampler(local)
    clocks.start()
    bench.barrier(pg)
    ev = []
    with torch.no_grad():
        for _ in range(a.steps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            step()
            e.record()
            ev.append((s, e))
    torch.cuda.synchronize()
    bench.barrier(pg)
    ck = clocks.stop()
    host_peak = round(bench.allreduce_max((bench._peak_rss_bytes() - rss0) / 1e9, pg), 1)
    rss_stages = {k: round((v - rss0) / 1e9, 1) for k, v in (
        ("built", rss_built), ("offloaded", rss_offloaded), ("setup", rss_setup), ("end", bench._rss_bytes()))}
    ms = sum(s.elapsed_time(e) for s, e in ev) / len(ev)
    eng = bench._engine(om) if a.impl == "ours" else None
    heap = getattr(eng, "device_bytes", 0) if eng is not None else 0
    cp_heap = cp.heap.nbytes if (cp is not None and getattr(cp, "heap", None) is not None) else 0
    peak = (torch.cuda.max_memory_allocated(device) + heap + cp_heap) / 1e9
    hidden = None
    try:
        rep = om.collect_offload_timing()
        if rep is not None and getattr(rep, "total_transfer_sum", 0) > 0:
            hidden = round(100.0 * max(0.0, 1.0 - rep.total_wait_sum / rep.total_transfer_sum), 2)
    except Exception:  # noqa: BLE001
        pass
    ms_max = bench.allreduce_max(ms, pg)
    peak_max = bench.allreduce_max(peak, pg)
    if rank == 0:
        print(json.dumps({
            "metric": "s/step (one denoise step), LTX-shape DiT, context parallel, 50% weights offloaded",
            "value": round(ms_max / 1000, 4), "unit": "s/step", "impl": a.impl, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "peak_gpu_gb": round(peak_max, 2), "transfer_hidden_pct": hidden,
            "weights_gb": round(total / 1e9, 2), "setup_s": round(setup_s, 1), "host_peak_gb_per_rank": host_peak, "host_rss_gb_rank0": rss_stages, "clocks": ck,
            "config": {"model": f"LTX-shape DiT ({a.layers} blocks, d=4096, 32 heads, FFN 16384, 40480 tokens, "
                                "text 256x4096)" + ("" if a.layers == 48 else " [NOT the full config]"),
                       "parallelism": (f"cp{world} " + ("fused K/V all-gather in attention + striped streaming"
                                                        if a.impl == "ours" else "Ulysses all-to-all (NCCL)"))
                       if world > 1 else "single GPU",
                       "l2": "flushed (256 MB write) before every timed step"},
            "data": "synthetic (random-init weights, N(0,1) inputs)"}))
    if cp is not None and hasattr(cp, "close"):
        cp.close()
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
