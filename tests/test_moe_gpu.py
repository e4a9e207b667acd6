"""Expert-parallel MoE GEMMs with fused dispatch/combine, ranks emulated on one GPU.

Each emulated rank has its own send / combine buffers, routing table and flag words; every
source's flag is set before the expert kernels run and each expert's completion flag is set by
an earlier launch in stream order, so no kernel waits on another launch. The result of the
whole dispatch -> gate/up (SwiGLU) -> down -> combine chain must equal an fp32 reference."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("W,EL,T,d,f", [(2, 2, 300, 256, 512), (4, 1, 257, 128, 256), (8, 1, 64, 128, 128),
                                        (1, 4, 500, 256, 256)])
def test_moe_fused_ep(W, EL, T, d, f):
    E, k = W * EL, 2
    g = torch.Generator(device=DEV).manual_seed(W * 31 + EL)
    x = [torch.randn(T, d, device=DEV, generator=g).bfloat16() for _ in range(W)]
    wgu = [(torch.randn(2 * f, d, device=DEV, generator=g) / d ** 0.5).bfloat16() for _ in range(E)]
    wdn = [(torch.randn(d, f, device=DEV, generator=g) / f ** 0.5).bfloat16() for _ in range(E)]
    rows = T * k
    max_rows = ((W * rows + EL * 128) + 127) // 128 * 128
    send = [torch.zeros(rows, d, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    comb = [torch.zeros(rows, d, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    table = [torch.zeros(2 * E, device=DEV, dtype=torch.int32) for _ in range(W)]
    send_flags = [torch.zeros(W, device=DEV, dtype=torch.int64) for _ in range(W)]
    send_acks = [torch.zeros(W, device=DEV, dtype=torch.int64) for _ in range(W)]
    comb_flags = [torch.zeros(W, device=DEV, dtype=torch.int64) for _ in range(W)]
    a_local = torch.empty(max_rows, d, device=DEV, dtype=torch.bfloat16)
    h_local = torch.empty(max_rows, f, device=DEV, dtype=torch.bfloat16)
    counters = torch.zeros(2 * W + 1, device=DEV, dtype=torch.int32)
    lib = native.lib()
    for epoch in (1, 2):
        ids, wts, pos = [], [], []
        for p in range(W):  # source side: routing + packing
            e = torch.randint(0, E, (T, k), device=DEV, generator=g)
            e[:, 1] = (e[:, 0] + 1 + torch.randint(0, E - 1, (T,), device=DEV, generator=g)) % E if E > 1 else e[:, 0]
            w = torch.softmax(torch.randn(T, k, device=DEV, generator=g), -1)
            flat = e.reshape(-1)
            order = torch.argsort(flat, stable=True)
            cnt = torch.bincount(flat, minlength=E).to(torch.int32)
            table[p][:E] = cnt
            table[p][E:] = torch.cumsum(cnt, 0, dtype=torch.int32) - cnt
            send[p].copy_(x[p].index_select(0, order // k))
            ps = torch.empty_like(order)
            ps[order] = torch.arange(order.numel(), device=DEV)
            ids.append(e)
            wts.append(w)
            pos.append(ps.view(T, k).to(torch.int32))
        for f_ in send_flags:
            f_.fill_(epoch)
        P = lambda ts: [t.data_ptr() for t in ts]  # noqa: E731
        for r in range(W):  # expert side of every emulated rank
            lib.moe_gemm(True, r, EL, d, f, max_rows, P(send), P(table), send_flags[r].data_ptr(), 1,
                         [a.data_ptr() + 8 * r for a in send_acks], a_local, h_local, wgu[r * EL:(r + 1) * EL],
                         [], [], epoch, counters)
            lib.moe_gemm(False, r, EL, d, f, max_rows, [], P(table), send_flags[r].data_ptr(), 1, [], a_local,
                         h_local, wdn[r * EL:(r + 1) * EL], P(comb), [c.data_ptr() + 8 * r for c in comb_flags],
                         epoch, counters)
        outs = []
        for p in range(W):
            o = torch.empty(T, d, device=DEV, dtype=torch.bfloat16)
            lib.moe_reduce(comb[p], pos[p], wts[p], x[p], o, comb_flags[p].data_ptr(), 1, W, p, epoch)
            outs.append(o)
        torch.cuda.synchronize()
        assert native.device_error(reset=True) == 0
        for p in range(W):
            ref = x[p].float().clone()
            for kk in range(k):
                for ex in range(E):
                    m = ids[p][:, kk] == ex
                    if m.any():
                        hh = x[p][m].float() @ wgu[ex].float().t()
                        y = (torch.nn.functional.silu(hh[:, 0::2]) * hh[:, 1::2]) @ wdn[ex].float().t()
                        ref[m] += wts[p][m, kk:kk + 1] * y
            err = float((outs[p].float() - ref).abs().max() / ref.abs().max())
            assert err < 3e-2, f"source {p}: rel err {err}"
            for q in range(W):
                if q != p:
                    assert int(send_acks[p][q]) == epoch, f"expert {q} did not ack source {p}"
