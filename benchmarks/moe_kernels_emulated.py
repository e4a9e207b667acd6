"""The fused expert-parallel MoE GEMMs on ONE GPU, emulating W ranks (every peer buffer is local):
the kernels' own structure without NVLink, at the Mixtral-8x7B expert shape (d 4096, f 14336,
8 experts, top-2, one expert per rank).

    python benchmarks/moe_kernels_emulated.py [--tokens 4096] [--iters 5]

Per emulated expert rank, one step launches the dispatch GEMM (pulls its routed rows from every
source's send buffer, gate/up projection with SwiGLU in the epilogue) and the combine GEMM (down
projection storing each row into its source's combine buffer); each source then reduces its
top-2 rows. Every source's flag is set before the expert kernels run, so no kernel waits on
another launch. Reports the mean device time per expert rank of each fused GEMM against the
plain tcgen05 GEMMs of the same row counts (``ops.linear_swiglu`` / ``ops.linear``).
"""

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

from flextensor_b200 import ops  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--tokens", type=int, default=4096, help="tokens per source rank")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--f", type=int, default=14336)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    W, T, d, f, k = a.world, a.tokens, a.d, a.f, 2
    E = W  # one expert per rank
    g = torch.Generator(device=dev).manual_seed(0)
    x = [torch.randn(T, d, device=dev, generator=g).bfloat16() for _ in range(W)]
    wgu = [(torch.randn(2 * f, d, device=dev, generator=g) / d ** 0.5).bfloat16() for _ in range(E)]
    wdn = [(torch.randn(d, f, device=dev, generator=g) / f ** 0.5).bfloat16() for _ in range(E)]
    rows = T * k
    max_rows = ((W * rows + 128) + 127) // 128 * 128
    send = [torch.zeros(rows, d, device=dev, dtype=torch.bfloat16) for _ in range(W)]
    comb = [torch.zeros(rows, d, device=dev, dtype=torch.bfloat16) for _ in range(W)]
    table = [torch.zeros(2 * E, device=dev, dtype=torch.int32) for _ in range(W)]
    send_flags = [torch.zeros(W, device=dev, dtype=torch.int64) for _ in range(W)]
    send_acks = [torch.zeros(W, device=dev, dtype=torch.int64) for _ in range(W)]
    comb_flags = [torch.zeros(W, device=dev, dtype=torch.int64) for _ in range(W)]
    a_local = torch.empty(max_rows, d, device=dev, dtype=torch.bfloat16)
    h_local = torch.empty(max_rows, f, device=dev, dtype=torch.bfloat16)
    counters = torch.zeros(2 * W + 1, device=dev, dtype=torch.int32)
    lib = native.lib()
    pos, wts, per_expert = [], [], torch.zeros(E, dtype=torch.int64)
    for p in range(W):  # routing + packing, once: the benchmark times the expert side
        e = torch.randint(0, E, (T, k), device=dev, generator=g)
        e[:, 1] = (e[:, 0] + 1 + torch.randint(0, E - 1, (T,), device=dev, generator=g)) % E
        wts.append(torch.softmax(torch.randn(T, k, device=dev, generator=g), -1))
        flat = e.reshape(-1)
        order = torch.argsort(flat, stable=True)
        cnt = torch.bincount(flat, minlength=E).to(torch.int32)
        per_expert += cnt.cpu().long()
        table[p][:E] = cnt
        table[p][E:] = torch.cumsum(cnt, 0, dtype=torch.int32) - cnt
        send[p].copy_(x[p].index_select(0, order // k))
        ps = torch.empty_like(order)
        ps[order] = torch.arange(order.numel(), device=dev)
        pos.append(ps.view(T, k).to(torch.int32))
    P = lambda ts: [t.data_ptr() for t in ts]  # noqa: E731
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    t_disp, t_comb, epoch = 0.0, 0.0, 0
    for it in range(2 + a.iters):
        epoch += 1
        for f_ in send_flags:
            f_.fill_(epoch)
        marks = []
        for r in range(W):
            e0, e1, e2 = ev(), ev(), ev()
            e0.record()
            lib.moe_gemm(True, r, 1, d, f, max_rows, P(send), P(table), send_flags[r].data_ptr(), 1,
                         [s.data_ptr() + 8 * r for s in send_acks], a_local, h_local, [wgu[r]], [], [], epoch, counters)
            e1.record()
            lib.moe_gemm(False, r, 1, d, f, max_rows, [], P(table), send_flags[r].data_ptr(), 1, [], a_local,
                         h_local, [wdn[r]], P(comb), [c.data_ptr() + 8 * r for c in comb_flags], epoch, counters)
            e2.record()
            marks.append((e0, e1, e2))
        for p in range(W):
            o = torch.empty(T, d, device=dev, dtype=torch.bfloat16)
            lib.moe_reduce(comb[p], pos[p], wts[p], x[p], o, comb_flags[p].data_ptr(), 1, W, p, epoch)
        torch.cuda.synchronize()
        if it >= 2:
            t_disp += sum(m[0].elapsed_time(m[1]) for m in marks) / W
            t_comb += sum(m[1].elapsed_time(m[2]) for m in marks) / W
    t_disp /= a.iters
    t_comb /= a.iters
    n_rows = int(per_expert.float().mean().item())  # the plain GEMMs run the mean rows per expert
    a_rows = torch.randn(n_rows, d, device=dev, generator=g).bfloat16()
    h_rows = torch.randn(n_rows, f, device=dev, generator=g).bfloat16()

    def tm(fn, n=a.iters):
        for _ in range(2):
            fn()
        s_, e_ = ev(), ev()
        s_.record()
        for _ in range(n):
            fn()
        e_.record()
        torch.cuda.synchronize()
        return s_.elapsed_time(e_) / n

    t_gu = tm(lambda: ops.linear_swiglu(a_rows, wgu[0]))
    t_dn = tm(lambda: ops.linear(h_rows, wdn[0], None, epi="none"))
    fl_gu, fl_dn = 2.0 * n_rows * d * 2 * f, 2.0 * n_rows * f * d
    print(json.dumps({
        "mode": f"emulated W={W} on 1 GPU", "tokens_per_source": T, "mean_rows_per_expert": n_rows,
        "dispatch_gemm_ms": round(t_disp, 4), "plain_gate_up_ms": round(t_gu, 4),
        "combine_gemm_ms": round(t_comb, 4), "plain_down_ms": round(t_dn, 4),
        "dispatch_tflops": round(fl_gu / t_disp / 1e9, 1), "combine_tflops": round(fl_dn / t_comb / 1e9, 1),
        "device_error": native.device_error(reset=True)}))


if __name__ == "__main__":
    main()
