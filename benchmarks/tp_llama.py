"""Tensor-parallel Llama-3-70B-shape decoder layers: fused collective GEMMs vs NCCL.

    torchrun --nproc-per-node N benchmarks/tp_llama.py [--tokens 16384] [--layers 4]

Each rank holds 1/N of the heads / FFN columns and 1/N of the token rows (sequence parallel).
Times one forward through ``--layers`` decoder layers (device time, max over ranks) with
``collective="fused"`` (all-gather inside the QKV / gate-up GEMMs, reduce-scatter from the
o_proj / down GEMM epilogues) and ``collective="nccl"`` (NCCL all_gather_into_tensor /
reduce_scatter_tensor around the same GEMMs). Reports per-layer ms, the collective bytes each
rank moves over NVLink and the roofline max(FLOPs / measured bf16 peak, bytes / 770 GB/s).
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
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--collectives", default="fused,nccl",
                    help="comma list of fused, nccl, fused_ag (fused all-gather only), fused_rs")
    ap.add_argument("--pair", action="store_true", help="experimental CTA-pair (cta_group::2) fused kernels")
    a = ap.parse_args()
    import torch.distributed as dist

    from flextensor_b200.models.llama import LLAMA3_70B, LlamaTP, rope_tables_1d

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = LLAMA3_70B
    M, S = a.tokens, a.seq
    B = M // S
    R = M // W
    tp = LlamaTP(cfg, rank, W, layers=a.layers).to(dev).to(torch.bfloat16)
    with torch.no_grad():
        for p in tp.parameters():
            p.normal_(0, 0.02)
    rope = rope_tables_1d(S, cfg.head_dim, cfg.rope_theta, dev)
    x0 = torch.randn(R, cfg.dim, device=dev).bfloat16()
    peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("bf16_tflops", 1590.0)
    res = {}
    for coll in a.collectives.split(","):
        tp.setup(M, collective=coll, pair=a.pair)
        x = x0.clone()

        def step():
            x.copy_(x0)
            with torch.no_grad():
                tp(x, B, S, rope)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            step()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters / a.layers], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[coll + "_ms_per_layer"] = round(float(t.item()), 4)
        tp.close()
    D, hq, hk, F = cfg.head_dim, cfg.n_heads // W, cfg.n_kv_heads // W, cfg.ffn_dim // W
    gemm_flops = 2.0 * M * cfg.dim * ((hq + 2 * hk) * D + hq * D + 2 * F + F)
    attn_flops = 4.0 * B * S * S * hq * D / 2  # causal
    nvlink = 4 * (W - 1) / W * M * cfg.dim * 2  # 2 all-gathers + 2 reduce-scatters of [M, d] bf16
    roof = max((gemm_flops + attn_flops) / (peak * 1e9), nvlink / 770e6)
    res.update({"n_gpus": W, "tokens": M, "layers_timed": a.layers, "flops_per_layer_per_rank": gemm_flops + attn_flops,
                "nvlink_bytes_per_layer_per_rank": nvlink, "roofline_ms_per_layer": round(roof, 4),
                })
    if "fused_ms_per_layer" in res:
        res["fused_frac_of_roofline"] = round(roof / res["fused_ms_per_layer"], 3)
        if "nccl_ms_per_layer" in res:
            res["speedup_fused_vs_nccl"] = round(res["nccl_ms_per_layer"] / res["fused_ms_per_layer"], 3)
    if rank == 0:
        print(json.dumps(res))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
