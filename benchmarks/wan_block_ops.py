"""Per-op device time inside Wan-14B-shape DiT blocks.

    python benchmarks/wan_block_ops.py [--layers 2]

Builds a ``--layers``-block Wan2.2-14B-shape DiT (random init, bf16, all weights on the GPU),
wraps every ``ops.*`` call (linear, layernorm_modulate, rmsnorm, qk_rmsnorm_rope, attention) in
CUDA events and runs 4 forwards over the 32,760-token latent; prints the last forward's total,
the summed time per op kind and shape, and the time outside the ops. The events themselves add a
little to each op.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    a = ap.parse_args()
    from flextensor_b200 import ops
    from flextensor_b200.models.wan import WAN_14B, WanConfig, WanDiT, init_wan_params_
    from flextensor_b200.ops import api

    cfg = WanConfig(**{**WAN_14B.__dict__, "num_layers": a.layers})
    with torch.device("meta"):
        m = WanDiT(cfg, impl="fused")
    m = m.to_empty(device="cuda").to(torch.bfloat16)
    init_wan_params_(m)
    lat = torch.randn(1, 16, 21, 60, 104, device="cuda", dtype=torch.bfloat16)
    ctx = torch.randn(1, 512, 4096, device="cuda", dtype=torch.bfloat16)
    ts = torch.tensor([500.0], device="cuda")
    rec = []

    def wrap(name, fn):
        def w(*args, **kw):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kw)
            e.record()
            rec.append((name, args, kw, s, e))
            return out
        return w

    for n in ("linear", "layernorm_modulate", "rmsnorm", "qk_rmsnorm_rope", "attention"):
        setattr(ops, n, wrap(n, getattr(api, n)))
    with torch.no_grad():
        for _ in range(4):
            rec.clear()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            m(lat, ts, ctx)
            t1.record()
            torch.cuda.synchronize()
    agg: dict[str, list[float]] = {}
    for name, args, kw, s, e in rec:
        key = name
        if name == "linear":
            key = f"linear {tuple(args[1].shape)} M={args[0].reshape(-1, args[0].shape[-1]).shape[0]} " \
                  f"epi={kw.get('epi', 'bias')}"
        elif name == "attention":
            key = f"attention q{tuple(args[0].shape)} k{tuple(args[1].shape)}"
        agg.setdefault(key, []).append(s.elapsed_time(e))
    total = t0.elapsed_time(t1)
    print(f"forward ({a.layers} blocks + embed/head): {total:.2f} ms")
    ssum = 0.0
    for k, v in agg.items():
        print(f"{sum(v):8.3f} ms  x{len(v):2d}  {k}")
        ssum += sum(v)
    print(f"sum of op times {ssum:.2f} ms; other {total - ssum:.2f} ms")


if __name__ == "__main__":
    main()
