"""Tensor-parallel fused GEMMs, ranks emulated on one GPU (every rank's buffers are separate
allocations; flags are set before the launches that read them, so no kernel waits on another
launch): all-gather -> GEMM (bias / SwiGLU) and GEMM -> reduce-scatter -> reduce, against fp32
references."""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.ops import api as ops  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("W,R,K,N,epi,rank", [(4, 200, 256, 384, "bias", 1), (2, 256, 512, 1024, "swiglu", 0),
                                              (8, 96, 128, 256, "none", 7), (3, 333, 192, 512, "swiglu", 2),
                                              (2, 150, 256, 640, "gelu", 1)])
def test_allgather_gemm(W, R, K, N, epi, rank):
    M = W * R
    g = torch.Generator(device=DEV).manual_seed(W * 10 + rank)
    a = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    bias = torch.randn(N, device=DEV, generator=g).bfloat16() if epi in ("bias", "gelu") else None
    bufs = []
    for p in range(W):
        b = torch.zeros(M, K, device=DEV, dtype=torch.bfloat16)
        b[p * R:(p + 1) * R] = a[p * R:(p + 1) * R]
        bufs.append(b)
    flags = torch.zeros(W, dtype=torch.int64, device=DEV)
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    counters = torch.zeros(ops.tp_ag_counter_words(M, W), dtype=torch.int32, device=DEV)
    for epoch in (1, 2):
        flags.fill_(epoch)
        out = ops.tp_allgather_gemm(bufs[rank], w, peer_a=[b.data_ptr() for b in bufs], flags_ptr=flags.data_ptr(),
                                    flag_stride=1, peer_acks=[x.data_ptr() + 8 * rank for x in acks], rank=rank,
                                    epoch=epoch, counters=counters, bias=bias, epi=epi)
        torch.cuda.synchronize()
        assert native.device_error(reset=True) == 0
        ref = a.float() @ w.float().t()
        if bias is not None:
            ref = ref + bias.float()
        if epi == "swiglu":
            ref = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
        if epi == "gelu":
            ref = torch.nn.functional.gelu(ref, approximate="tanh")
        assert _rel(out, ref) < 2e-2
        assert torch.equal(bufs[rank], a), "rows not gathered"
        for p in range(W):
            if p != rank:
                assert int(acks[p][rank]) == epoch
        for p in range(W):  # next epoch: clear the gathered rows again
            if p != rank:
                bufs[rank][p * R:(p + 1) * R].zero_()


@pytest.mark.parametrize("W,R,K,N", [(4, 200, 256, 384), (2, 256, 512, 512), (8, 64, 128, 256)])
def test_gemm_reducescatter(W, R, K, N):
    M = W * R
    g = torch.Generator(device=DEV).manual_seed(W + N)
    a = [torch.randn(M, K, device=DEV, generator=g).bfloat16() for _ in range(W)]
    w = [(torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).bfloat16() for _ in range(W)]
    res = [torch.randn(R, N, device=DEV, generator=g).bfloat16() for _ in range(W)]
    stage = [torch.zeros(W, R, N, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    flags = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]   # flags[owner][src]
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]    # acks[src][owner]
    counters = torch.zeros(1, dtype=torch.int32, device=DEV)
    for epoch in (1, 2):
        for r in range(W):
            ops.tp_gemm_reducescatter(a[r], w[r], stage=[s.data_ptr() for s in stage],
                                      peer_flags=[f.data_ptr() + 8 * r for f in flags], rank=r, epoch=epoch,
                                      counters=counters)
        outs = []
        for p in range(W):
            o = torch.empty(R, N, device=DEV, dtype=torch.bfloat16)
            ops.tp_reduce(stage[p], W, R, o, flags_ptr=flags[p].data_ptr(), flag_stride=1, epoch=epoch,
                          peer_acks=[x.data_ptr() + 8 * p for x in acks], rank=p, residual=res[p])
            outs.append(o)
        torch.cuda.synchronize()
        assert native.device_error(reset=True) == 0
        full = sum(a[r].float() @ w[r].float().t() for r in range(W))
        for p in range(W):
            ref = full[p * R:(p + 1) * R] + res[p].float()
            assert _rel(outs[p], ref) < 2e-2, f"owner {p}"
            for q in range(W):
                if q != p:
                    assert int(acks[q][p]) == epoch


@pytest.mark.parametrize("W,M,K,N", [(2, 37, 256, 256), (4, 300, 128, 512), (8, 5, 128, 256), (3, 3, 64, 256)])
def test_gemm_allreduce_uneven_rows(W, M, K, N):
    """GEMM -> reduce-scatter -> owner reduce broadcast into every rank's output (all-reduce),
    with row counts that do not divide evenly (some owners hold fewer or no rows)."""
    R = (M + W - 1) // W
    g = torch.Generator(device=DEV).manual_seed(W * 7 + M)
    a = [torch.randn(M, K, device=DEV, generator=g).bfloat16() for _ in range(W)]
    w = [(torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).bfloat16() for _ in range(W)]
    stage = [torch.zeros(W, R, N, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    outs = [torch.zeros(M, N, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    flags = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    counters = torch.zeros(1, dtype=torch.int32, device=DEV)
    for r in range(W):
        ops.tp_gemm_reducescatter(a[r], w[r], stage=[s.data_ptr() for s in stage],
                                  peer_flags=[f.data_ptr() + 8 * r for f in flags], rank=r, epoch=1, counters=counters)
    for p in range(W):
        rows = max(0, min(R, M - p * R))
        ops.tp_reduce(stage[p], W, rows, outs[p], flags_ptr=flags[p].data_ptr(), flag_stride=1, epoch=1,
                      peer_acks=[x.data_ptr() + 8 * p for x in acks], rank=p, out_peers=[o.data_ptr() for o in outs],
                      row_base=p * R, stage_rows=R)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    full = sum(a[r].float() @ w[r].float().t() for r in range(W))
    for q in range(W):
        assert _rel(outs[q], full) < 2e-2, f"rank {q}'s all-reduced output"
        for p in range(W):
            if p != q:
                assert int(acks[q][p]) == 1


@pytest.mark.parametrize("W,rows,D,rope", [(2, 77, 512, True), (4, 300, 1024, False), (8, 33, 5120, True), (1, 64, 256, True)])
def test_distributed_rmsnorm_emulated(W, rows, D, rope):
    """RMSNorm over a hidden dimension split across W emulated ranks (partial sums of squares to
    every rank's slot, then each rank scales its columns, optional RoPE), against the fp32 norm
    of the concatenated row. Phase 1 of every rank runs before any phase 2 (no launch waits on a
    launch that has not run)."""
    Dl, Dh = D // W, 128
    stage_rows = (rows + 31) // 32 * 32
    g = torch.Generator(device=DEV).manual_seed(W * 100 + rows)
    xs = [torch.randn(rows, Dl, device=DEV, generator=g).bfloat16() for _ in range(W)]
    w = torch.randn(D, device=DEV, generator=g)
    parts = [torch.zeros(W, stage_rows, device=DEV) for _ in range(W)]
    flags = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    cos = sin = None
    if rope:
        ang = torch.randn(rows, Dh // 2, device=DEV, generator=g)
        cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    outs = [torch.empty_like(x) for x in xs]
    for phase in (1, 2):
        for r in range(W):
            ops.tp_rmsnorm(xs[r], w[r * Dl:(r + 1) * Dl].contiguous(), d_full=D, part_peers=[p.data_ptr() for p in parts],
                           stage_rows=stage_rows, peer_flags=[f.data_ptr() + 8 * r for f in flags],
                           flags_ptr=flags[r].data_ptr(), flag_stride=1,
                           peer_acks=[a.data_ptr() + 8 * r for a in acks], rank=r, epoch=1, counter=counter,
                           eps=1e-6, cos=cos, sin=sin, head_dim=Dh if rope else 0, seq_len=rows if rope else 0,
                           out=outs[r], _phases=phase)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    xf = torch.cat([x.float() for x in xs], 1)
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    if rope:
        rr = ref.view(rows, D // Dh, Dh // 2, 2)
        re, im = rr[..., 0], rr[..., 1]
        c, s = cos[:, None, :], sin[:, None, :]
        ref = torch.stack([re * c - im * s, re * s + im * c], -1).view(rows, D)
    for r in range(W):
        assert _rel(outs[r], ref[:, r * Dl:(r + 1) * Dl]) < 1e-2, r
        for q in range(W):
            if q != r:
                assert int(acks[q][r]) == 1


def test_reduce_bias_gate_residual():
    """Owner reduce with bias, per-group fp32 gate and residual: out = res + gate * (sum + bias)."""
    W, M, K, N, S = 2, 64, 128, 256, 32
    R = M // W
    g = torch.Generator(device=DEV).manual_seed(3)
    a = [torch.randn(M, K, device=DEV, generator=g).bfloat16() for _ in range(W)]
    w = [(torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).bfloat16() for _ in range(W)]
    bias = torch.randn(N, device=DEV, generator=g).bfloat16()
    gate = torch.randn(M // S, N, device=DEV, generator=g)
    res = [torch.randn(R, N, device=DEV, generator=g).bfloat16() for _ in range(W)]
    stage = [torch.zeros(W, R, N, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    flags = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    counters = torch.zeros(1, dtype=torch.int32, device=DEV)
    for r in range(W):
        ops.tp_gemm_reducescatter(a[r], w[r], stage=[s.data_ptr() for s in stage],
                                  peer_flags=[f.data_ptr() + 8 * r for f in flags], rank=r, epoch=1, counters=counters)
    outs = [x.clone() for x in res]
    for p in range(W):
        ops.tp_reduce(stage[p], W, R, outs[p], flags_ptr=flags[p].data_ptr(), flag_stride=1, epoch=1,
                      peer_acks=[x.data_ptr() + 8 * p for x in acks], rank=p, residual=outs[p], bias=bias, gate=gate,
                      gate_rows=S, grow0=p * R)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    full = sum(a[r].float() @ w[r].float().t() for r in range(W)) + bias.float()
    full = full * gate.repeat_interleave(S, 0)
    for p in range(W):
        ref = res[p].float() + full[p * R:(p + 1) * R]
        assert _rel(outs[p], ref) < 2e-2, p


@pytest.mark.parametrize("W,R,K,N,epi", [(2, 256, 512, 1024, "none"), (4, 200, 256, 640, "swiglu"),
                                         (8, 96, 128, 384, "bias")])
def test_pair_kernels_emulated(W, R, K, N, epi):
    """The experimental cta_group::2 variants of the all-gather GEMM and the GEMM + reduce-scatter
    (``_pair=True``) on emulated ranks against fp32 references."""
    M = W * R
    g = torch.Generator(device=DEV).manual_seed(W + N)
    a = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).bfloat16()
    bias = torch.randn(N, device=DEV, generator=g).bfloat16() if epi == "bias" else None
    bufs = []
    for p in range(W):
        b = torch.zeros(M, K, device=DEV, dtype=torch.bfloat16)
        b[p * R:(p + 1) * R] = a[p * R:(p + 1) * R]
        bufs.append(b)
    flags = torch.ones(W, dtype=torch.int64, device=DEV)
    acks = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    counters = torch.zeros(ops.tp_ag_counter_words(M, W), dtype=torch.int32, device=DEV)
    out = ops.tp_allgather_gemm(bufs[0], w, peer_a=[b.data_ptr() for b in bufs], flags_ptr=flags.data_ptr(),
                                flag_stride=1, peer_acks=[x.data_ptr() for x in acks], rank=0, epoch=1,
                                counters=counters, bias=bias, epi=epi, _pair=True)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    ref = a.float() @ w.float().t() + (bias.float() if bias is not None else 0)
    if epi == "swiglu":
        ref = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
    assert _rel(out, ref) < 2e-2
    # GEMM -> reduce-scatter, every emulated rank with the pair kernel
    parts = [torch.randn(M, K, device=DEV, generator=g).bfloat16() for _ in range(W)]
    stage = [torch.zeros(W, R, N, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    rflags = [torch.zeros(W, dtype=torch.int64, device=DEV) for _ in range(W)]
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    for r in range(W):
        ops.tp_gemm_reducescatter(parts[r], w, stage=[s_.data_ptr() for s_ in stage],
                                  peer_flags=[f.data_ptr() + 8 * r for f in rflags], rank=r, epoch=1, counters=cnt,
                                  _pair=True)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    full = sum(parts[r].float() @ w.float().t() for r in range(W))
    for p in range(W):
        got = stage[p].float().sum(0)
        assert _rel(got, full[p * R:(p + 1) * R]) < 2e-2
        assert all(int(x) == 1 for x in rflags[p])
