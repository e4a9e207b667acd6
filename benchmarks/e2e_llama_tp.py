"""End to end: Llama-3-70B-shape decoder layers at tensor parallelism, half of each rank's
weights offloaded to host memory (32 requests x (2048 prompt + 256 decode)).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        benchmarks/e2e_llama_tp.py [--impl ours|reference] [--decode-steps D] [--layers L]

Model: 80 layers, d=8192, 64 q / 8 KV heads, SwiGLU FFN 28672, RoPE theta 5e5, bf16 random-init
weights; each rank holds its 1/N shard of every layer (heads and FFN columns). The layers are
the offload units; 50 % of a rank's weight bytes may stay on its GPU, the rest streams from
host memory every forward. Embedding and LM head are not part of the timed work (the same for
both arms). Synthetic N(0,1) hidden states stand in for embedded tokens.

* ``ours``: ``flextensor_b200.models.llama.LlamaTP`` -- sequence-parallel residual stream, the
  all-gather fused into the column-parallel tcgen05 GEMMs and the reduce-scatter fused into the
  row-parallel GEMM epilogues over NVLink, split-KV decode attention.
* ``reference``: the unmodified reference runtime (``baseline/_ref``) offloading
  ``baseline/llama_torch.py`` (cuBLAS GEMMs, SDPA, NCCL all-reduce after each row-parallel
  projection: vLLM's TP layout).

Timed (CUDA events, max over ranks): one prefill of 32 x 2048 tokens filling the KV cache, then
``--decode-steps`` decode steps of one token per sequence. One JSON line from rank 0.
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

BATCH, PROMPT, NEW = 32, 2048, 256
RESIDENT = 0.5


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=80)
    ap.add_argument("--decode-steps", type=int, default=16)
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
    M = BATCH * PROMPT

    def host_fits(meta_model) -> bool:
        ok, why = bench.host_gate(pg, bench.host_need_bytes(meta_model, a.impl, 1 - RESIDENT, "layers."), world,
                                  bench.host_start_bytes(meta_model, a.impl))
        if not ok and rank == 0:
            print(json.dumps({"impl": a.impl, "n_gpus": world, "unavailable": why}))
        return ok

    if a.impl == "ours":
        from flextensor_b200.models.llama import LLAMA3_70B, LlamaTP, init_llama_params_, rope_tables_1d

        cfg = LLAMA3_70B
        with torch.device("meta"):
            model = LlamaTP(cfg, rank, world, layers=a.layers)
        if not host_fits(model):
            return bench.close_dist(pg)
        model = model.to(torch.bfloat16).to_empty(device=dev)  # bf16 before any bytes exist
        init_llama_params_(model, seed=rank)
        if world > 1:
            model.setup(M, collective="fused")
            model.add_rows(BATCH)
        cos, sin = rope_tables_1d(PROMPT + NEW, cfg.head_dim, cfg.rope_theta, dev)
        rows_pre, rows_dec = M // world, BATCH // world

        def fwd(x, S, cache, pos, c, s):
            return model(x, BATCH, S, (c, s), cache=cache, pos=pos)
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        from llama_torch import LlamaShape, LlamaShard, init_params_, rope_cos_sin

        cfg = LlamaShape()
        with torch.device("meta"):
            model = LlamaShard(cfg, world, layers=a.layers)
        if not host_fits(model):
            return bench.close_dist(pg)
        model = model.to(torch.bfloat16).to_empty(device=dev)  # bf16 before any bytes exist
        init_params_(model, seed=rank)
        bench.to_pageable(model)
        cos, sin = rope_cos_sin(PROMPT + NEW, cfg.head_dim, cfg.rope_theta, dev)
        rows_pre, rows_dec = M, BATCH

        def fwd(x, S, cache, pos, c, s):
            return model(x, BATCH, S, c, s, cache=cache, pos=pos)
    model.eval()
    model.requires_grad_(False)
    total = sum(p.numel() * p.element_size() for p in model.parameters())
    frac = RESIDENT * total / torch.cuda.get_device_properties(dev).total_memory
    om = ft.get_offload_manager()
    config = bench.make_config(ft, local, frac, a.profiling_iters)
    config = config.model_copy(update={"include_patterns": ["layers.*"]}) if hasattr(config, "model_copy") \
        else config
    rss_built = bench._rss_bytes()
    model = om.offload(model, config)
    rss_offloaded = bench._rss_bytes()
    cache = model.new_cache(BATCH, PROMPT + NEW, dev)
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    x_pre = torch.randn(rows_pre, cfg.dim, device=dev, generator=g).bfloat16()
    x_dec = torch.randn(rows_dec, cfg.dim, device=dev, generator=g).bfloat16()
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
        est = (pre_ms + NEW * dec_ms) / 1000.0
        print(json.dumps({
            "metric": "s/step (prefill, decode) & peak GPU GB, Llama-3-70B-shape layers at TP, 50% offloaded",
            "value": round(est, 3), "unit": "s per request batch (prefill + 256 decode steps, from measured steps)",
            "impl": a.impl, "n_gpus": world, "prefill_s": round(pre_ms / 1000, 4),
            "decode_ms_per_step": round(dec_ms, 3), "decode_steps_timed": a.decode_steps,
            "peak_gpu_gb": round(peak, 2), "transfer_hidden_pct": hidden, "weights_gb_per_rank": round(total / 1e9, 2),
            "setup_s": round(setup_s, 1), "host_peak_gb_per_rank": host_peak, "host_rss_gb_rank0": rss_stages, "clocks": ck,
            "config": {"model": f"Llama-3-70B-shape decoder layers ({a.layers} of 80, d=8192, 64/8 heads, FFN 28672)"
                                + ("" if a.layers == 80 else " [NOT the full config]"),
                       "batch": f"{BATCH} x ({PROMPT} prompt + {NEW} decode)",
                       "parallelism": f"tp{world} " + ("fused AG/RS GEMMs, sequence-parallel residual"
                                                       if a.impl == "ours" else "NCCL all-reduce (vLLM layout)"),
                       "excluded": "embedding and LM head (both arms)"},
            "data": "synthetic (random-init weights, N(0,1) hidden states)"}))
    if a.impl == "ours" and world > 1:
        model.close()
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
