"""Row-normalisation kernels against a device copy of the same bytes.

    python benchmarks/norms.py [--rows 32760] [--dim 5120]

Times ``ops.layernorm_modulate`` (adaLN modulation and affine forms), ``ops.qk_rmsnorm_rope``
and ``ops.rmsnorm`` on a ``[rows, dim]`` bf16 activation (read once, written once) and
``Tensor.copy_`` of the same tensor, CUDA events, best of 3 x 20 launches.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32760)
    ap.add_argument("--dim", type=int, default=5120)
    a = ap.parse_args()
    from flextensor_b200 import ops

    M, D = a.rows, a.dim
    x = torch.randn(M, D, device="cuda").bfloat16()
    sc, sh = torch.randn(1, D, device="cuda") * 0.1, torch.randn(1, D, device="cuda") * 0.1
    w = torch.randn(D, device="cuda")
    cos, sin = torch.randn(M, 64, device="cuda"), torch.randn(M, 64, device="cuda")
    out = torch.empty_like(x)

    def tm(f, n=20):
        for _ in range(3):
            f()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            f()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n

    nbytes = 2 * M * D * 2
    for name, f in (("layernorm_modulate", lambda: ops.layernorm_modulate(x, sc, sh, out=out)),
                    ("layernorm affine", lambda: ops.layernorm_modulate(x, weight=w, bias=w, out=out)),
                    ("qk_rmsnorm_rope", lambda: ops.qk_rmsnorm_rope(x, w, cos, sin, 128, M, out=out)),
                    ("rmsnorm", lambda: ops.rmsnorm(x, w, out=out)),
                    ("copy", lambda: out.copy_(x))):
        ms = min(tm(f) for _ in range(3))
        print(f"{name}: {ms * 1e3:.1f} us  {nbytes / ms / 1e9:.2f} TB/s")


if __name__ == "__main__":
    main()
