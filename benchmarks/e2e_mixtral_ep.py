"""End to end: Mixtral-8x22B-shape MoE decoder layers with expert parallelism, part of every
rank's weights streamed from host memory (64 x (1024 prompt + 128 decode)).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        benchmarks/e2e_mixtral_ep.py [--impl ours|reference] [--decode-steps D] [--layers L]

Model: 56 layers, d=6144, 48 q / 8 KV heads, 8 experts top-2, expert FFN 16384 (SwiGLU), bf16
random-init weights. Each rank runs attention for its own 64/N sequences and owns 8/N experts
of every layer; the layers are the offload units. With N = 8 a rank holds ~44 GB of weights;
``--resident`` of them (default 0.75) may stay on the GPU and the rest streams from host memory
every forward (the N ranks' streamed experts are all different, so together they need N times
that in host RAM: 25 % streamed keeps 8 ranks at ~90 GB of the GPU boxes' 196 GB). Embedding and
LM head are not part of the timed work (both arms).

* ``ours``: ``flextensor_b200.models.mixtral.MixtralStack`` -- dispatch fused into the gate/up
  GEMM and combine into the down GEMM's epilogue over NVLink (``ExpertParallel``), native
  attention, split-KV decode attention.
* ``reference``: the unmodified reference runtime (``baseline/_ref``) offloading
  ``baseline/mixtral_torch.py`` (NCCL all-to-all dispatch / combine, cuBLAS expert GEMMs, SDPA).

Timed (CUDA events, max over ranks): one prefill of 64 x 1024 tokens filling the KV cache, then
``--decode-steps`` decode steps. One JSON line from rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

BATCH, PROMPT, NEW = 64, 1024, 128


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=56)
    ap.add_argument("--decode-steps", type=int, default=8)
    ap.add_argument("--resident", type=float, default=0.75)
    ap.add_argument("--profiling-iters", type=int, default=3)
    a = ap.parse_args()
    import torch

    rss0 = bench._rss_bytes()
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank, world, local, pg = bench.dist_setup(world)
    dev = torch.device("cuda", local)
    ft, why = bench.import_arm(a.impl)
    if ft is None:
        if rank == 0:
            print(json.dumps({"impl": a.impl, "unavailable": why}))
        return
    if BATCH % world:
        raise SystemExit(f"{BATCH} sequences do not split over {world} ranks")
    B = BATCH // world

    def host_fits(meta_model) -> bool:
        ok, why = bench.host_gate(pg, bench.host_need_bytes(meta_model, a.impl, 1 - a.resident, "layers."), world,
                                  bench.host_start_bytes(meta_model, a.impl))
        if not ok and rank == 0:
            print(json.dumps({"impl": a.impl, "n_gpus": world, "unavailable": why}))
        return ok

    if a.impl == "ours":
        from flextensor_b200.models.llama import rope_tables_1d
        from flextensor_b200.models.mixtral import MIXTRAL_8X22B, MixtralStack, init_mixtral_params_

        cfg = MIXTRAL_8X22B
        with torch.device("meta"):
            model = MixtralStack(cfg, rank, world, layers=a.layers)
        if not host_fits(model):
            return bench.close_dist(pg)
        model = model.to(torch.bfloat16).to_empty(device=dev)  # bf16 before any bytes exist
        init_mixtral_params_(model, seed=0)
        ep = {}
        if world > 1:
            from flextensor_b200.parallel.ep import ExpertParallel

            for rows in (B * PROMPT, B):
                ep[rows] = ExpertParallel(rows, cfg.dim, cfg.ffn_dim, cfg.n_experts, cfg.topk)
        cos, sin = rope_tables_1d(PROMPT + NEW, cfg.head_dim, cfg.rope_theta, dev)

        def fwd(x, S, cache, pos, c, s):
            return model(x, B, S, (c, s), ep=ep, cache=cache, pos=pos)
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        from llama_torch import rope_cos_sin
        from mixtral_torch import MixtralEP, MixtralShape, init_params_

        cfg = MixtralShape()
        with torch.device("meta"):
            model = MixtralEP(cfg, rank, world, layers=a.layers)
        if not host_fits(model):
            return bench.close_dist(pg)
        model = model.to(torch.bfloat16).to_empty(device=dev)  # bf16 before any bytes exist
        init_params_(model, seed=rank)
        bench.to_pageable(model)
        cos, sin = rope_cos_sin(PROMPT + NEW, cfg.head_dim, cfg.rope_theta, dev)
        ep = {}

        def fwd(x, S, cache, pos, c, s):
            return model(x, B, S, c, s, cache=cache, pos=pos)
    model.eval()
    model.requires_grad_(False)
    total = sum(p.numel() * p.element_size() for p in model.parameters())
    frac = a.resident * total / torch.cuda.get_device_properties(dev).total_memory
    om = ft.get_offload_manager()
    config = bench.make_config(ft, local, frac, a.profiling_iters).model_copy(update={"include_patterns": ["layers.*"]})
    rss_built = bench._rss_bytes()
    model = om.offload(model, config)
    rss_offloaded = bench._rss_bytes()
    cache = model.new_cache(B, PROMPT + NEW, dev)
    g = torch.Generator(device=dev).manual_seed(21 + rank)
    x_pre = torch.randn(B * PROMPT, cfg.dim, device=dev, generator=g).bfloat16()
    x_dec = torch.randn(B, cfg.dim, device=dev, generator=g).bfloat16()
    c_pre, s_pre = cos[:PROMPT].contiguous(), sin[:PROMPT].contiguous()
    t0 = time.perf_counter()
    with torch.no_grad():
        for _ in range(om.iters_before_inference + 1):
            fwd(x_pre.clone(), PROMPT, cache, 0, c_pre, s_pre)
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t0
    rss_setup = bench._rss_bytes()
    torch.cuda.reset_peak_memory_stats(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    clocks = bench.ClockSampler(local)
    clocks.start()
    bench.barrier(pg)
    with torch.no_grad():
        flush.fill_(1)
        ps, pe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ps.record()
        fwd(x_pre.clone(), PROMPT, cache, 0, c_pre, s_pre)
        pe.record()
        dec = []
        for i in range(a.decode_steps):
            pos = PROMPT + i
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fwd(x_dec.clone(), 1, cache, pos, cos[pos:pos + 1].contiguous(), sin[pos:pos + 1].contiguous())
            e.record()
            dec.append((s, e))
    torch.cuda.synchronize()
    bench.barrier(pg)
    ck = clocks.stop()
    host_peak = round(bench.allreduce_max((bench._peak_rss_bytes() - rss0) / 1e9, pg), 1)
    rss_stages = {k: round((v - rss0) / 1e9, 1) for k, v in (
        ("built", rss_built), ("offloaded", rss_offloaded), ("setup", rss_setup), ("end", bench._rss_bytes()))}
    pre_ms = bench.allreduce_max(ps.elapsed_time(pe), pg)
    dec_ms = bench.allreduce_max(sum(s.elapsed_time(e) for s, e in dec) / max(1, len(dec)), pg)
    peak = bench.allreduce_max(torch.cuda.max_memory_allocated(dev) / 1e9, pg)
    hidden = None
    try:
        rep = om.collect_offload_timing()
        if rep is not None and getattr(rep, "total_transfer_sum", 0) > 0:
            hidden = round(100.0 * max(0.0, 1.0 - rep.total_wait_sum / rep.total_transfer_sum), 2)
    except Exception:  # noqa: BLE001
        pass
    if rank == 0:
        print(json.dumps({
            "metric": "s/step (prefill, decode) & peak GPU GB, Mixtral-8x22B-shape layers at EP, experts streamed",
            "value": round((pre_ms + NEW * dec_ms) / 1000.0, 3),
            "unit": "s per request batch (prefill + 128 decode steps, from measured steps)",
            "impl": a.impl, "n_gpus": world, "prefill_s": round(pre_ms / 1000, 4),
            "decode_ms_per_step": round(dec_ms, 3), "decode_steps_timed": a.decode_steps,
            "peak_gpu_gb": round(peak, 2), "transfer_hidden_pct": hidden,
            "weights_gb_per_rank": round(total / 1e9, 2), "resident_fraction": a.resident,
            "setup_s": round(setup_s, 1), "host_peak_gb_per_rank": host_peak, "host_rss_gb_rank0": rss_stages, "clocks": ck,
            "config": {"model": f"Mixtral-8x22B-shape layers ({a.layers} of 56, d=6144, 48/8 heads, 8 experts top-2, "
                                "FFN 16384)" + ("" if a.layers == 56 else " [NOT the full config]"),
                       "batch": f"{BATCH} x ({PROMPT} prompt + {NEW} decode)",
                       "parallelism": f"ep{world} " + ("dispatch/combine fused into the expert GEMMs"
                                                       if a.impl == "ours" else "NCCL all-to-all"),
                       "excluded": "embedding and LM head (both arms)"},
            "data": "synthetic (random-init weights, N(0,1) hidden states)"}))
    for e in ep.values():
        if hasattr(e, "close"):
            e.close()
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
