"""Expert-parallel MoE layer at the Mixtral-8x22B shape: fused dispatch/combine vs NCCL.

    torchrun --nproc-per-node N benchmarks/ep_mixtral.py [--tokens 8192]

Each rank routes its own ``--tokens`` rows (top-2 of 8 experts, random router) and owns 8/N
experts (d=6144, FFN 16384). Times route+dispatch -> expert GEMMs -> combine (device time,
max over ranks) for ``ExpertParallel`` (dispatch pulled inside the gate/up GEMM, combine
stored from the down GEMM's epilogue) and ``NcclExpertParallel`` (all_to_all_single around
the same GEMM kernels). Roofline: max(expert FLOPs / measured bf16 peak, NVLink bytes / 770 GB/s).
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args()
    import torch.distributed as dist

    from flextensor_b200.models.mixtral import MIXTRAL_8X22B as cfg
    from flextensor_b200.parallel.ep import ExpertParallel, NcclExpertParallel, route_topk

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    T, d, f, E = a.tokens, cfg.dim, cfg.ffn_dim, cfg.n_experts
    el = E // W
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(T, d, device=dev, generator=g).bfloat16()
    router = torch.randn(E, d, device=dev, generator=g).bfloat16() * 0.02
    wgu = [(torch.randn(2 * f, d, device=dev, generator=g) * 0.02).bfloat16() for _ in range(el)]
    wdn = [(torch.randn(d, f, device=dev, generator=g) * 0.02).bfloat16() for _ in range(el)]
    ids, wts = route_topk(x, router, cfg.topk)
    peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("bf16_tflops", 1590.0)
    ep = ExpertParallel(T, d, f, E, cfg.topk)
    nccl = NcclExpertParallel(E)
    out = torch.empty_like(x)

    def fused():
        pos = ep.dispatch(x, ids)
        ep.experts(wgu, wdn)
        ep.combine(pos, wts, residual=x, out=out)

    def base():
        nccl(x, ids, wts, wgu, wdn, x)

    res = {}
    for name, fn in (("fused", fused), ("nccl", base)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name + "_ms"] = round(float(t.item()), 4)
    # work actually routed to this rank's experts (max over ranks sets the pace)
    counts = torch.bincount(ids.reshape(-1), minlength=E)
    allc = torch.empty(W, E, dtype=counts.dtype, device=dev)
    dist.all_gather_into_tensor(allc, counts)
    rows_per_rank = allc.sum(0).view(W, el).sum(1)
    rows_max = int(rows_per_rank.max())
    flops = 2.0 * rows_max * d * 3 * f
    sent = T * cfg.topk - int(counts.view(W, el)[rank].sum())
    nvlink = 2.0 * sent * d * 2  # dispatch + combine rows leaving / entering this rank
    t_nv = torch.tensor([nvlink], device=dev, dtype=torch.float64)
    dist.all_reduce(t_nv, op=dist.ReduceOp.MAX)
    roof = max(flops / (peak * 1e9), float(t_nv.item()) / 770e6)
    # per-phase device time of the fused path (max over ranks; cross-rank waits included)
    from flextensor_b200.ops import native

    lib = native.lib()
    P = ep.heap.ptrs
    tables = [p_ + ep.tbl_off for p_ in P]
    phases = {"route_pack_publish": [], "dispatch_gateup_gemm": [], "down_gemm_combine_stores": [], "reduce": []}
    for _ in range(a.iters):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        dist.barrier()
        ev[0].record()
        pos = ep.dispatch(x, ids)
        ev[1].record()
        lib.moe_gemm(True, ep.rank, ep.el, d, f, ep.max_rows, [p_ + ep.send_off for p_ in P], tables,
                     ep.send_flags[ep.rank], 1, [q + 8 * ep.rank for q in ep.send_acks], ep.a_local, ep.h_local,
                     wgu, [], [], ep.epoch, ep.counters)
        ev[2].record()
        lib.moe_gemm(False, ep.rank, ep.el, d, f, ep.max_rows, [], tables, ep.send_flags[ep.rank], 1, [],
                     ep.a_local, ep.h_local, wdn, [p_ + ep.comb_off for p_ in P],
                     [c + 8 * ep.rank for c in ep.comb_flags], ep.epoch, ep.counters)
        ev[3].record()
        ep.combine(pos, wts, residual=x, out=out)
        ev[4].record()
        torch.cuda.synchronize()
        for i, k in enumerate(phases):
            phases[k].append(ev[i].elapsed_time(ev[i + 1]))
    for k, v in phases.items():
        t = torch.tensor([sorted(v)[len(v) // 2]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res["fused_phase_ms_" + k] = round(float(t.item()), 4)
    res.update({"n_gpus": W, "tokens_per_rank": T, "max_rows_per_expert_rank": rows_max,
                "roofline_ms": round(roof, 4), "fused_frac_of_roofline": round(roof / res["fused_ms"], 3),
                "speedup_fused_vs_nccl": round(res["nccl_ms"] / res["fused_ms"], 3)})
    torch.cuda.synchronize()
    ep.close()
    if rank == 0:
        print(json.dumps(res))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
