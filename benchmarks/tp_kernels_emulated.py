"""The fused tensor-parallel kernels on ONE GPU, emulating W ranks (every peer buffer is local):
the kernels' own structure without NVLink. Times rank 0's all-gather GEMM / GEMM + reduce-scatter
launch against the plain GEMM of the same shape (Llama-3-70B layer shapes, 16,384 tokens).

    python benchmarks/tp_kernels_emulated.py [--pair]

``--pair``: the experimental CTA-pair (cta_group::2) kernels.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch
from flextensor_b200 import ops
dev = "cuda"
PAIR = "--pair" in sys.argv[1:]
def tm(f, n=10):
    for _ in range(3): f()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(n): f()
    e_.record(); torch.cuda.synchronize()
    return s_.elapsed_time(e_) / n
M = 16384
for W in (2, 8):
    R = M // W
    # GEMM -> RS: o_proj (K = 8192/W... per rank heads), down (K = 28672/W)
    for name, K, N in (("o_proj", 8192 // W, 8192), ("down", 28672 // W, 8192)):
        a = torch.randn(M, K, device=dev).bfloat16()
        w = (torch.randn(N, K, device=dev) / K ** 0.5).bfloat16()
        stage = [torch.zeros(W, R, N, device=dev, dtype=torch.bfloat16) for _ in range(W)]
        flags = [torch.zeros(W, dtype=torch.int64, device=dev) for _ in range(W)]
        counters = torch.zeros(1, dtype=torch.int32, device=dev)
        ep = [0]
        def rs():
            ep[0] += 1
            ops.tp_gemm_reducescatter(a, w, stage=[s.data_ptr() for s in stage],
                                      peer_flags=[f.data_ptr() for f in flags], rank=0, epoch=ep[0], counters=counters,
                                      _pair=PAIR)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        t_rs = tm(rs)
        t_lin = tm(lambda: ops.linear(a, w, None, epi="none", out=out))
        print(f"W={W} RS {name} M={M} K={K} N={N}: fused {t_rs:.3f} ms  plain GEMM {t_lin:.3f} ms  "
              f"({2*M*K*N/t_rs/1e9:.0f} vs {2*M*K*N/t_lin/1e9:.0f} TF/s)")
    # AG -> GEMM: qkv (N = 10240/W), gate_up (N = 2*28672/W, swiglu)
    for name, K, N, epi in (("qkv", 8192, 10240 // W, "none"), ("gate_up", 8192, 2 * 28672 // W, "swiglu")):
        a_full = torch.randn(M, K, device=dev).bfloat16()
        bufs = [a_full.clone() for _ in range(W)]
        w = (torch.randn(N, K, device=dev) / K ** 0.5).bfloat16()
        flags = torch.zeros(W, dtype=torch.int64, device=dev)
        acks = [torch.zeros(W, dtype=torch.int64, device=dev) for _ in range(W)]
        counters = torch.zeros(ops.api.tp_ag_counter_words(M, W), dtype=torch.int32, device=dev)
        ep = [0]
        def ag():
            ep[0] += 1
            flags.fill_(ep[0])
            ops.tp_allgather_gemm(bufs[0], w, peer_a=[b.data_ptr() for b in bufs], flags_ptr=flags.data_ptr(),
                                  flag_stride=1, peer_acks=[x.data_ptr() for x in acks], rank=0, epoch=ep[0],
                                  counters=counters, epi=epi, _pair=PAIR)
        t_ag = tm(ag)
        if epi == "swiglu":
            t_lin = tm(lambda: ops.linear_swiglu(a_full, w))
        else:
            t_lin = tm(lambda: ops.linear(a_full, w, None, epi="none"))
        print(f"W={W} AG {name} M={M} K={K} N={N}: fused {t_ag:.3f} ms  plain GEMM {t_lin:.3f} ms  "
              f"(gathers {(W-1)*R*K*2/1e6:.0f} MB locally)")
print("device error", __import__("flextensor_b200.ops", fromlist=["native"]).native.device_error(reset=True))
