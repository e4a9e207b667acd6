"""Decode attention: one query per sequence over a KV cache, against the HBM roofline.

    python benchmarks/decode.py [--shapes llama70b,llama70b_tp8,mixtral] [--iters 20]

Shapes (B sequences, context, query heads, KV heads):
  llama70b      32 x 2304, 64 / 8   (BASELINE config: 2048 prompt + 256 decode tokens)
  llama70b_tp8  32 x 2304,  8 / 1   (one rank's heads at TP = 8)
  mixtral       64 x 1152, 48 / 8   (1024 prompt + 128 decode tokens)

For each: the split-KV decode kernel (``ops.decode_attention``), the prefill kernel given one
query per sequence (``ops.attention``, what the decode path used before), and PyTorch SDPA
(``enable_gqa``). Times are CUDA-event medians of device time (the GPU is given a head start so
host launch overhead is not counted); the L2 is flushed by reading 256 MB before each launch (a write flush would leave ~126 MB of dirty
lines whose write-back the timed kernel would pay for). Roofline: K + V bytes of the
context at the measured copy bandwidth (``MEASURED_PEAKS.json`` ``hbm_gbs``, else 6650 GB/s).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics as st
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

SHAPES = {"llama70b": (32, 2304, 64, 8), "llama70b_tp8": (32, 2304, 8, 1), "mixtral": (64, 1152, 48, 8)}


def hbm_gbs() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:  # noqa: BLE001
        return 6650.0


def timed(fn, iters, flush):
    """Device time of ``fn``: the GPU sleeps ~50 us after the L2 flush, before the start event, so
    the host has enqueued ``fn``'s launches when the start event fires (host-side launch overhead
    is not counted, for every timed op alike)."""
    ts = []
    for _ in range(3):
        fn()
    for _ in range(iters):
        flush.sum()  # read 256 MB: evicts the L2 without leaving dirty lines for fn to write back
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(100_000)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e) * 1000.0)
    return st.median(ts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="llama70b,llama70b_tp8,mixtral")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--n-split", type=int, default=0, help="0: the library's choice")
    a = ap.parse_args()
    from flextensor_b200 import ops
    from flextensor_b200.ops import native

    dev = torch.device("cuda", 0)
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=dev)
    bw = hbm_gbs()
    for name in a.shapes.split(","):
        B, L, Hq, Hk = SHAPES[name]
        torch.manual_seed(0)
        q = torch.randn(B, 1, Hq, 128, device=dev, dtype=torch.bfloat16)
        kc = torch.randn(B, L, Hk, 128, device=dev, dtype=torch.bfloat16)
        vc = torch.randn(B, L, Hk, 128, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(q)
        kv_bytes = 2 * B * L * Hk * 128 * 2
        roof_us = kv_bytes / (bw * 1e9) * 1e6
        t_dec = timed(lambda: ops.decode_attention(q, kc, vc, L, out=out, n_split=a.n_split), a.iters, flush)
        t_pre = timed(lambda: ops.attention(q, kc, vc), a.iters, flush)
        qt, kt, vt = q.transpose(1, 2), kc.transpose(1, 2), vc.transpose(1, 2)
        t_sdpa = timed(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, enable_gqa=True),
                       a.iters, flush)
        err = (ops.decode_attention(q, kc, vc, L).float() - ops.attention(q, kc, vc).float()).abs().max().item()
        assert native.device_error(reset=True) == 0
        print(json.dumps({"shape": name, "B": B, "ctx": L, "Hq": Hq, "Hk": Hk, "kv_MB": round(kv_bytes / 1e6, 1),
                          "roofline_us": round(roof_us, 1), "decode_us": round(t_dec, 1),
                          "n_split": a.n_split or native.lib().decode_splits(B, Hk, L, torch.cuda.get_device_properties(dev).multi_processor_count),
                          "decode_x_roofline": round(t_dec / roof_us, 2), "prefill_kernel_us": round(t_pre, 1),
                          "sdpa_us": round(t_sdpa, 1), "max_abs_diff_vs_prefill_kernel": err}))


if __name__ == "__main__":
    main()
