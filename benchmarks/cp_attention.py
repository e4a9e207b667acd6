"""Context-parallel self-attention at the LTX shape (40,480 tokens, 32 heads x 128, bf16).

Single process (``python benchmarks/cp_attention.py --emulate W``): W ranks are emulated on one
GPU -- separate full-sequence K|V buffers, peers' rows written and flagged before the launch --
so the fused kernel's gather runs from local HBM. Reports the fused kernel against plain
attention over already-local K/V (the compute-only floor).

Multi-GPU (``torchrun --nproc-per-node N benchmarks/cp_attention.py``): each rank holds 1/N of
the tokens. Times (CUDA events, max over ranks):
  * ``fused``   -- ContextParallel: publish + the fused K/V-gathering attention kernel;
  * ``ag_nccl`` -- NCCL all_gather of K|V, then plain attention (the unfused baseline);
  * ``ulysses`` -- all-to-all seq->heads, attention on H/N heads, all-to-all back (reference scheme).
Roofline of the fused kernel: max(FLOPs / measured bf16 peak, bytes pulled over NVLink /
770 GB/s per direction).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

S_TOT, H, D = 40480, 32, 128


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops", 1590.0)), float(d.get("hbm_gbs", 6650.0))
    except Exception:  # noqa: BLE001
        return 1590.0, 6650.0


def _time(fn, iters=10, warmup=3, pg=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    if pg is not None:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def emulate(W: int, iters: int):
    from flextensor_b200.ops import api as ops

    dev = torch.device("cuda", 0)
    S_loc = S_TOT // W
    torch.manual_seed(0)
    q = torch.randn(1, S_loc, H, D, device=dev).bfloat16()
    k = torch.randn(1, S_TOT, H, D, device=dev).bfloat16()
    v = torch.randn(1, S_TOT, H, D, device=dev).bfloat16()
    bufs = []
    for p in range(W):
        kv = torch.zeros(1, 2, S_TOT, H, D, device=dev, dtype=torch.bfloat16)
        rows = slice(p * S_loc, (p + 1) * S_loc)
        kv[:, 0, rows] = k[:, rows]
        kv[:, 1, rows] = v[:, rows]
        bufs.append(kv)
    rank = 0
    flags = torch.zeros(W, dtype=torch.int64, device=dev)
    acks = [torch.zeros(W, dtype=torch.int64, device=dev) for _ in range(W)]
    counters = torch.zeros(2 * W, dtype=torch.int32, device=dev)
    state = {"epoch": 0}

    def fused():
        state["epoch"] += 1
        flags.fill_(state["epoch"])
        ops.attention_cp(q, bufs[rank], peer_kv=[b.data_ptr() for b in bufs], flags_ptr=flags.data_ptr(),
                         flag_stride=1, peer_acks=[a.data_ptr() + 8 * rank for a in acks], rank=rank,
                         shard_rows=S_loc, epoch=state["epoch"], counters=counters)

    def local():
        ops.attention(q, k, v)

    flops = 4.0 * S_loc * S_TOT * H * D
    peak, _ = _peaks()
    t_f = _time(fused, iters)
    t_l = _time(local, iters)
    out = {"mode": f"emulated W={W} on 1 GPU", "S_loc": S_loc, "fused_ms": round(t_f, 4), "local_attn_ms": round(t_l, 4),
           "fused_tflops": round(flops / t_f / 1e9, 1), "local_tflops": round(flops / t_l / 1e9, 1),
           "gather_overhead_pct": round(100 * (t_f / t_l - 1), 2), "of_measured_peak": round(flops / t_f / 1e9 / peak, 3)}
    print(json.dumps(out))


def multi(iters: int):
    import datetime

    import torch.distributed as dist

    from flextensor_b200.ops import api as ops
    from flextensor_b200.parallel.cp import ContextParallel, UlyssesAttention

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    S_loc = S_TOT // W
    dev = torch.device("cuda", local)
    torch.manual_seed(rank)
    q = torch.randn(1, S_loc, H, D, device=dev).bfloat16()
    k = torch.randn(1, S_loc, H, D, device=dev).bfloat16()
    v = torch.randn(1, S_loc, H, D, device=dev).bfloat16()
    cp = ContextParallel(S_TOT, kv_heads=H)

    for _ in range(2):  # both slots hold this rank's rows; the timed calls only signal + attend
        kr, vr = cp.begin()
        kr.copy_(k.view(S_loc, H * D))
        vr.copy_(v.view(S_loc, H * D))
        cp.publish()
        cp.attention(q)

    def fused():
        cp.begin()
        cp.publish()
        cp.attention(q)

    k_all = torch.empty(1, S_TOT, H, D, device=dev, dtype=torch.bfloat16)
    v_all = torch.empty(1, S_TOT, H, D, device=dev, dtype=torch.bfloat16)

    def ag_nccl():
        dist.all_gather_into_tensor(k_all, k)
        dist.all_gather_into_tensor(v_all, v)
        ops.attention(q, k_all, v_all)

    uly = UlyssesAttention()

    def ulysses():
        uly(q, k, v, lambda a, b, c: ops.attention(a.contiguous(), b.contiguous(), c.contiguous()))

    flops = 4.0 * S_loc * S_TOT * H * D
    nvlink_bytes = (W - 1) * S_loc * 2 * H * D * 2
    peak, _ = _peaks()
    res = {}
    for name, fn in (("fused", fused), ("ag_nccl", ag_nccl), ("ulysses", ulysses)):
        res[name + "_ms"] = round(_time(fn, iters, pg=dist), 4)
    roof = max(flops / (peak * 1e9), nvlink_bytes / 770e6)
    res.update({"n_gpus": W, "S_loc": S_loc, "flops_per_rank": flops, "nvlink_bytes_per_rank": nvlink_bytes,
                "roofline_ms": round(roof, 4), "fused_frac_of_roofline": round(roof / res["fused_ms"], 3),
                "peak_bf16_tflops_measured": peak})
    torch.cuda.synchronize()
    cp.close()
    if rank == 0:
        print(json.dumps(res))
    dist.destroy_process_group()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--emulate", type=int, default=0)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    if a.emulate:
        emulate(a.emulate, a.iters)
    else:
        multi(a.iters)
