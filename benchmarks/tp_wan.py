"""Tensor-parallel Wan2.2-14B-shape DiT: fused collective kernels vs the NCCL all_reduce layout.

    torchrun --nproc-per-node N benchmarks/tp_wan.py [--layers 4] [--iters 3]

Every rank holds 1/N of the heads and FFN columns of ``--layers`` Wan-14B blocks. One forward
runs over the 32,760-token latent (81 frames at 480x832), batch 1. Both arms use the same
tcgen05 GEMM and attention kernels:

* ``fused``: sequence-parallel residual stream. The all-gather runs inside the Q / cross-Q /
  FFN-in GEMMs, the reduce-scatter leaves the output-projection GEMM epilogues, and the
  distributed Q/K RMSNorm exchanges its sums of squares over peer stores.
* ``nccl``: the reference driver's layout (``integrated_e2e.py:159-220``). The residual stream is
  replicated; NCCL ``all_reduce`` runs after each row-parallel projection and on the Q/K sums of
  squares.

Reports device ms per forward (max over ranks, CUDA events) and per layer, the NVLink bytes per
rank per layer, and the roofline max(FLOPs / measured bf16 peak, bytes / 770 GB/s).
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
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--frames", type=int, default=21, help="latent frames (21 = 81 video frames)")
    a = ap.parse_args()
    import torch.distributed as dist

    from flextensor_b200.models.wan import WAN_14B, WanConfig, WanDiT, init_wan_params_
    from flextensor_b200.models.wan_tp import WanTensorParallel

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = WanConfig(**{**WAN_14B.__dict__, "num_layers": a.layers})
    grid = (a.frames, 60, 104)  # latent 21 x 60 x 104 -> patches 21 x 30 x 52
    S = grid[0] * (grid[1] // 2) * (grid[2] // 2)
    g = torch.Generator(device=dev).manual_seed(0)
    lat = torch.randn(1, cfg.in_channels, *grid, device=dev, generator=g).bfloat16()
    ctx = torch.randn(1, cfg.text_len, cfg.text_dim, device=dev, generator=g).bfloat16()
    t = torch.tensor([500.0], device=dev)
    peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("bf16_tflops", 1590.0)
    res = {}
    for impl in ("fused", "nccl"):
        with torch.device("meta"):
            m = WanDiT(cfg)
        m = m.to(torch.bfloat16).to_empty(device=dev)
        init_wan_params_(m, seed=0)
        m.eval().requires_grad_(False)
        tp = WanTensorParallel(m, impl=impl, max_tokens=S)
        with torch.no_grad():
            for _ in range(2):
                tp(lat, t, ctx)
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(a.iters):
                tp(lat, t, ctx)
            e.record()
            torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / a.iters], device=dev, dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        res[impl + "_ms_per_forward"] = round(float(ms.item()), 3)
        res[impl + "_ms_per_layer"] = round(float(ms.item()) / a.layers, 3)
        tp.close()
        del tp, m
        torch.cuda.empty_cache()
    D, F, L = cfg.dim, cfg.ffn_dim, cfg.text_len
    gemm = 2.0 * S * (3 * D * D + D * D + D * D + D * D + 2 * D * F) / W + 2.0 * L * 2 * D * D / W
    attn = (4.0 * S * S * D + 4.0 * S * L * D) / W
    nvlink = 6 * (W - 1) / W * S * D * 2  # 3 all-gathers + 3 reduce-scatters of [S, D] bf16
    roof = max((gemm + attn) / (peak * 1e9), nvlink / 770e6)
    res.update({"n_gpus": W, "tokens": S, "layers": a.layers, "flops_per_layer_per_rank": gemm + attn,
                "nvlink_bytes_per_layer_per_rank": nvlink, "roofline_ms_per_layer": round(roof, 3),
                "fused_frac_of_roofline": round(roof / res["fused_ms_per_layer"], 3),
                "speedup_fused_vs_nccl": round(res["nccl_ms_per_forward"] / res["fused_ms_per_forward"], 3)})
    if rank == 0:
        print(json.dumps(res))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
