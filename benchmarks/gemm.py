"""tcgen05 GEMM on the Wan2.2-14B projection shapes against cuBLAS (``torch.matmul``).

    python benchmarks/gemm.py [--tokens 32760]

``C = A . W^T``, bf16 in, fp32 accumulation, bf16 out; the 1-SM 128x256 tile kernel
(``force_bn=256``) and the 2-SM 256x256 pair kernel (``force_bn=512``) against cuBLAS, CUDA
events, median of 10 launches after 3 warm-ups; also checks the outputs agree with cuBLAS.
"""

from __future__ import annotations

import argparse
import os
import statistics as st
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32760)
    a = ap.parse_args()
    from flextensor_b200 import ops

    def tm(f):
        for _ in range(3):
            f()
        ts = []
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            f()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        return st.median(ts)

    M = a.tokens
    for N, K, what in ((5120, 5120, "q/k/v/o"), (13824, 5120, "FFN in"), (5120, 13824, "FFN out")):
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
        fl = 2.0 * M * N * K
        row = []
        for bn in (256, 512):
            ms = tm(lambda bn=bn: ops.linear(x, w, None, epi="none", force_bn=bn))
            row.append(f"{'1-SM' if bn == 256 else '2-SM'} {fl / ms / 1e9:.0f} TF/s")
        ms = tm(lambda: torch.matmul(x, w.t()))
        row.append(f"cuBLAS {fl / ms / 1e9:.0f} TF/s")
        diff = (ops.linear(x, w, None, epi="none").float() - torch.matmul(x, w.t()).float()).abs().max()
        print(f"{M} x {N} x {K} ({what}): " + ", ".join(row) + f"; max |ours - cuBLAS| {float(diff):.3e}")


if __name__ == "__main__":
    main()
