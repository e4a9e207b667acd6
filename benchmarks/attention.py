"""sm_100a flash attention: timing, kernel-variant comparison, per-block timeline, accuracy.

    python benchmarks/attention.py [--seq 32760] [--heads 40] [--modes 0,100,102] [--trace]

``--modes`` are ``ops.attention``'s timing variants (``_diag_mode``): 0 = the default kernel,
100 + k = k exp2 pairs in 8 on the FMA pipe instead of MUFU, 200 / 201 = the experimental
one-tile kernel with double-buffered S (0 / 1 exp2 pair in 8 on the FMA pipe; not yet run on a
GPU), 300 + k = the split-row kernel (two warps per query row, k exp2 pairs in 8 on the FMA
pipe), 400 + k = P through shared memory with event-driven MMA issue. Each mode is timed with CUDA events
(5 launches after 2 warm-ups, median of ``--reps`` repetitions, all modes in one process)
against ``torch.nn.functional.scaled_dot_product_attention`` (cuDNN on B200). ``--trace``
prints the clock64 timeline of CTA 0, in cycles per 128-key block (median over blocks 4..57):
TMEM load, row max, the two halves of the exponentials, P publication, the MMA warp's handoff
and the period. Accuracy: max / mean abs error on 2 heads against fp32 SDPA.
"""

from __future__ import annotations

import argparse
import os
import statistics as st
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def timeline(t):
    J = range(4, 58)

    def d(a, b, off=0):
        return st.median([t[b][j + off] - t[a][j] for j in J])

    last = [max(t[7][j], t[16][j], t[17][j], t[3][j]) for j in range(64)]
    return {"ready->loaded": d(4, 5), "loaded->max": d(5, 12), "max->half": d(12, 13), "half->exp_done": d(13, 6),
            "exp_done->pub": d(6, 7), "warp pub offsets (w1,w2,w3)": (d(7, 16), d(7, 17), d(7, 3)),
            "last pub->MMA sees p_full": st.median([t[18][j] - last[j] for j in J]),
            "MMA sees p_full->S(j+1) issued": d(18, 1), "S(j+1) issued->next S ready": d(1, 4, 1),
            "period": d(4, 4, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=32760)
    ap.add_argument("--heads", type=int, default=40)
    ap.add_argument("--modes", default="0,100")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--trace", action="store_true")
    a = ap.parse_args()
    from flextensor_b200 import ops

    B, S, H = 1, a.seq, a.heads
    torch.manual_seed(0)
    q = torch.randn(B, S, H, 128, device="cuda", dtype=torch.bfloat16)
    k, v = torch.randn_like(q), torch.randn_like(q)
    modes = [int(m) for m in a.modes.split(",")]
    flops = 4.0 * B * S * S * H * 128
    if a.trace:
        for m in modes:
            tr = torch.zeros(20 * 64, dtype=torch.long, device="cuda")
            o = torch.empty_like(q)
            for _ in range(3):
                ops.attention(q, k, v, out=o, _trace=tr, _diag_mode=m)
            torch.cuda.synchronize()
            print(f"mode {m} timeline:", timeline(tr.view(20, 64).cpu().tolist()))
    res = {m: [] for m in modes + ["sdpa"]}
    for _ in range(a.reps):
        for m in modes + ["sdpa"]:
            o = torch.empty_like(q)
            if m == "sdpa":
                qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))
                f = lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)  # noqa: E731
            else:
                f = lambda m=m: ops.attention(q, k, v, out=o, _diag_mode=m)  # noqa: E731
            for _ in range(2):
                f()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(5):
                f()
            e.record()
            torch.cuda.synchronize()
            res[m].append(s.elapsed_time(e) / 5)
    for m, ts in res.items():
        ms = st.median(ts)
        print(f"{'mode ' + str(m) if m != 'sdpa' else 'SDPA'}: {ms:.3f} ms  {flops / ms / 1e9:.0f} TF/s")
    qf, kf, vf = (x[:, :, :2].float().transpose(1, 2) for x in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf).transpose(1, 2)
    for m in modes:
        o = ops.attention(q, k, v, _diag_mode=m)
        err = (o[:, :, :2].float() - ref).abs()
        print(f"mode {m}: max abs err {float(err.max()):.3e}, mean {float(err.mean()):.3e}")


if __name__ == "__main__":
    main()
