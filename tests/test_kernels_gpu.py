"""Numerics of the sm_100a kernels against plain PyTorch fp32 references (GPU only)."""

import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU collection
    pytest.skip("CUDA device required", allow_module_level=True)

from flextensor_b200 import ops  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _lin_ref(x, w, b=None):
    y = x.float() @ w.float().t()
    return y + b.float() if b is not None else y


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 320), (1000, 384, 512), (4096, 5120, 5120),
                                   (257, 64, 128), (130, 136, 72)])
def test_gemm_plain(M, N, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    y = ops.linear(x, w, None, epi="none")
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(y, _lin_ref(x, w)) < 1e-2


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths(bn):
    torch.manual_seed(1)
    x = torch.randn(700, 1024, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(768, 1024, device=DEV, dtype=torch.bfloat16) / 32
    y = ops.linear(x, w, None, epi="none", force_bn=bn)
    assert rel_err(y, _lin_ref(x, w)) < 1e-2


def test_gemm_epilogues():
    torch.manual_seed(2)
    M, N, K = 513, 1024, 768
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    b = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    ref = _lin_ref(x, w, b)
    assert rel_err(ops.linear(x, w, b, epi="bias"), ref) < 1e-2
    g = torch.nn.functional.gelu(ref, approximate="tanh")
    assert rel_err(ops.linear(x, w, b, epi="gelu"), g) < 1e-2
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    gate = torch.randn(N, device=DEV, dtype=torch.float32)
    assert rel_err(ops.linear(x, w, b, epi="gate_res", residual=res, gate=gate), res.float() + gate * ref) < 1e-2
    assert rel_err(ops.linear(x, w, b, epi="res", residual=res), res.float() + ref) < 1e-2
    # in place: out aliases residual
    r2 = res.clone()
    ops.linear(x, w, b, epi="gate_res", residual=r2, gate=gate, out=r2)
    assert rel_err(r2, res.float() + gate * ref) < 1e-2
    # per-sample gates
    gate2 = torch.randn(2, N, device=DEV, dtype=torch.float32)
    rows = (M + 1) // 2
    y = ops.linear(x, w, b, epi="gate_res", residual=res, gate=gate2, gate_rows=rows)
    gfull = torch.cat([gate2[0].expand(rows, N), gate2[1].expand(M - rows, N)])
    assert rel_err(y, res.float() + gfull * ref) < 1e-2


def test_gemm_strided_views():
    torch.manual_seed(3)
    big = torch.randn(400, 3 * 512, device=DEV, dtype=torch.bfloat16)
    x = big[:, 512:1024]                      # strided A (row stride 1536)
    w = torch.randn(256, 512, device=DEV, dtype=torch.bfloat16) / 22
    out = torch.zeros(400, 3 * 256, device=DEV, dtype=torch.bfloat16)
    ops.linear(x, w, None, epi="none", out=out[:, 256:512])
    assert rel_err(out[:, 256:512], _lin_ref(x, w)) < 1e-2
    assert out[:, :256].abs().sum().item() == 0 and out[:, 512:].abs().sum().item() == 0


def test_layernorm_modulate():
    torch.manual_seed(4)
    M, D = 777, 5120
    x = (torch.randn(M, D, device=DEV) * 3 + 1).bfloat16()
    sc = torch.randn(D, device=DEV) * 0.1
    sh = torch.randn(D, device=DEV) * 0.1
    ref = torch.nn.functional.layer_norm(x.float(), (D,), eps=1e-6) * (1 + sc) + sh
    assert rel_err(ops.layernorm_modulate(x, sc, sh), ref) < 1e-2
    w = torch.randn(D, device=DEV)
    b = torch.randn(D, device=DEV)
    ref2 = torch.nn.functional.layer_norm(x.float(), (D,), w, b, eps=1e-6)
    assert rel_err(ops.layernorm_modulate(x, weight=w, bias=b), ref2) < 1e-2


def test_rmsnorm_and_rope():
    torch.manual_seed(5)
    S, H, Dh = 300, 8, 128
    x = torch.randn(2 * S, H * Dh, device=DEV).bfloat16()
    w = torch.randn(H * Dh, device=DEV)
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert rel_err(ops.rmsnorm(x, w), ref) < 1e-2
    ang = torch.randn(S, Dh // 2, device=DEV)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    y = ops.qk_rmsnorm_rope(x, w, cos, sin, Dh, S)
    r = ref.view(2, S, H, Dh // 2, 2)
    re, im = r[..., 0], r[..., 1]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    rot = torch.stack([re * c - im * s, re * s + im * c], -1).view(2 * S, H * Dh)
    assert rel_err(y, rot) < 1e-2


def test_layernorm_large_mean():
    """Rows with |mean| >> std (mean 40, std 1; a bf16 step at 40 is 0.25): the block-merged
    per-thread centred statistics match fp32 LayerNorm of the same bf16 values."""
    torch.manual_seed(7)
    M, D = 64, 5120
    x = (torch.randn(M, D, device=DEV) + 40).bfloat16()
    ref = torch.nn.functional.layer_norm(x.float(), (D,), eps=1e-6)
    y = ops.layernorm_modulate(x)
    assert float((y.float() - ref).abs().max()) < 0.05


@pytest.mark.parametrize("D", [1000, 4096, 5120, 6144, 8192, 12288])
def test_norm_vector_shapes_and_scalar_fallback(D):
    """Every launch shape of the row kernels (1..8 vectors per thread at 128 threads, wider CTAs
    past 8192 columns) with 16-byte-aligned parameters (vector loads), and the scalar-load
    variant on parameters that start one element off a 16-byte boundary."""
    torch.manual_seed(D)
    M = 300
    x = (torch.randn(M, D, device=DEV) * 2 + 0.5).bfloat16()
    buf = torch.randn(4, D + 8, device=DEV) * 0.1
    for off in (0, 1):
        sc, sh = buf[0, off:off + D], buf[1, off:off + D]
        ref = torch.nn.functional.layer_norm(x.float(), (D,), eps=1e-6) * (1 + sc) + sh
        assert rel_err(ops.layernorm_modulate(x, sc, sh), ref) < 1e-2, off
        wb = (buf[2] + 1).bfloat16()[off:off + D]
        bb = buf[3].bfloat16()[off:off + D]
        ref2 = torch.nn.functional.layer_norm(x.float(), (D,), wb.float(), bb.float(), eps=1e-6)
        assert rel_err(ops.layernorm_modulate(x, weight=wb, bias=bb), ref2) < 1e-2, off
        w = buf[2, off:off + D] + 1
        ref3 = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w
        assert rel_err(ops.rmsnorm(x, w), ref3) < 1e-2, off
    if D % 128 == 0:
        Dh, S = 128, M // 2
        ang = torch.randn(S * Dh // 2 + 1, device=DEV)
        w = buf[2, :D] + 1
        for off in (0, 1):  # tables at a 16-byte boundary, and one float past it (scalar loads)
            cos = ang.cos()[off:off + S * Dh // 2].view(S, Dh // 2)
            sin = ang.sin()[off:off + S * Dh // 2].view(S, Dh // 2)
            y = ops.qk_rmsnorm_rope(x, w, cos, sin, Dh, S)
            r = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w)
            r = r.view(2, S, D // Dh, Dh // 2, 2)
            re, im = r[..., 0], r[..., 1]
            c, s = cos[None, :, None, :], sin[None, :, None, :]
            rot = torch.stack([re * c - im * s, re * s + im * c], -1).view(M, D)
            assert rel_err(y, rot) < 1e-2, off


def _attn_ref(q, k, v, causal=False):
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    if kf.shape[1] != qf.shape[1]:
        rep = qf.shape[1] // kf.shape[1]
        kf = kf.repeat_interleave(rep, 1)
        vf = vf.repeat_interleave(rep, 1)
    o = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=causal)
    return o.transpose(1, 2)


@pytest.mark.parametrize("B,Sq,Sk,H,Hk", [(1, 128, 128, 1, 1), (2, 300, 300, 4, 4), (1, 256, 512, 2, 2),
                                          (2, 200, 77, 3, 3), (1, 384, 384, 8, 2), (1, 1000, 1000, 2, 2)])
def test_attention(B, Sq, Sk, H, Hk):
    torch.manual_seed(6)
    q = torch.randn(B, Sq, H, 128, device=DEV).bfloat16()
    k = torch.randn(B, Sk, Hk, 128, device=DEV).bfloat16()
    v = torch.randn(B, Sk, Hk, 128, device=DEV).bfloat16()
    o = ops.attention(q, k, v)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(o, _attn_ref(q, k, v)) < 2e-2


def test_attention_causal():
    torch.manual_seed(7)
    q = torch.randn(2, 500, 4, 128, device=DEV).bfloat16()
    k = torch.randn(2, 500, 4, 128, device=DEV).bfloat16()
    v = torch.randn(2, 500, 4, 128, device=DEV).bfloat16()
    o = ops.attention(q, k, v, causal=True)
    assert rel_err(o, _attn_ref(q, k, v, causal=True)) < 2e-2


def test_attention_large_logits():
    # exercises the deferred-rescale path: logits grow along the key axis
    torch.manual_seed(8)
    q = torch.randn(1, 256, 2, 128, device=DEV).bfloat16()
    k = (torch.randn(1, 1024, 2, 128, device=DEV) * torch.linspace(0.2, 3, 1024, device=DEV)[None, :, None, None]
         ).bfloat16()
    v = torch.randn(1, 1024, 2, 128, device=DEV).bfloat16()
    o = ops.attention(q, k, v)
    assert rel_err(o, _attn_ref(q, k, v)) < 2e-2


@pytest.mark.parametrize("mode", [200, 201])
@pytest.mark.parametrize("B,Sq,Sk,H,Hk,causal", [(1, 128, 128, 1, 1, False), (2, 300, 300, 4, 4, False),
                                                 (1, 384, 1000, 8, 2, False), (2, 500, 500, 4, 4, True)])
def test_attention_one_tile_kernel(mode, B, Sq, Sk, H, Hk, causal):
    """The experimental one-tile kernel with double-buffered S (``_diag_mode`` 200/201) against the
    fp32 reference and the default kernel; includes the deferred-rescale path."""
    torch.manual_seed(9)
    q = torch.randn(B, Sq, H, 128, device=DEV).bfloat16()
    k = (torch.randn(B, Sk, Hk, 128, device=DEV) * torch.linspace(0.2, 3, Sk, device=DEV)[None, :, None, None]
         ).bfloat16()
    v = torch.randn(B, Sk, Hk, 128, device=DEV).bfloat16()
    o = ops.attention(q, k, v, causal=causal, _diag_mode=mode)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(o, _attn_ref(q, k, v, causal=causal)) < 2e-2
    assert rel_err(o, ops.attention(q, k, v, causal=causal)) < 1e-2


@pytest.mark.parametrize("mode", [100, 102, 103, 104, 300, 301, 302, 400, 401, 402])
@pytest.mark.parametrize("B,Sq,Sk,H,Hk,causal", [(1, 128, 128, 1, 1, False), (2, 300, 300, 4, 4, False),
                                                 (1, 384, 1000, 8, 2, False), (2, 500, 500, 4, 4, True),
                                                 (1, 1024, 2048, 2, 1, False)])
def test_attention_split_row_kernel(mode, B, Sq, Sk, H, Hk, causal):
    """The split-row kernel (two warps per query row, ``_diag_mode`` 300-302) and the
    P-through-shared-memory kernel (event-driven MMA issue, modes 400-402) against the fp32
    reference and the default kernel; keys with growing scale exercise the rescale path."""
    torch.manual_seed(11)
    q = torch.randn(B, Sq, H, 128, device=DEV).bfloat16()
    k = (torch.randn(B, Sk, Hk, 128, device=DEV) * torch.linspace(0.2, 3, Sk, device=DEV)[None, :, None, None]
         ).bfloat16()
    v = torch.randn(B, Sk, Hk, 128, device=DEV).bfloat16()
    o = ops.attention(q, k, v, causal=causal, _diag_mode=mode)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(o, _attn_ref(q, k, v, causal=causal)) < 2e-2
    assert rel_err(o, ops.attention(q, k, v, causal=causal)) < 1e-2


@pytest.mark.parametrize("M,N,K", [(512, 256, 64), (1000, 768, 512), (4096, 5120, 5120), (777, 384, 1024)])
def test_gemm_pair_kernel(M, N, K):
    """2-SM (cta_group::2, 256x256 tiles) kernel, forced."""
    torch.manual_seed(9)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    b = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    gate = torch.randn(N, device=DEV, dtype=torch.float32)
    ref = _lin_ref(x, w, b)
    y = ops.linear(x, w, b, epi="gate_res", residual=res, gate=gate, force_bn=512)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(y, res.float() + gate * ref) < 1e-2


def _decode_ref(q, kc, vc, lens):
    """fp32 SDPA of one query per sequence over keys [0, len_b)."""
    B, Hq = q.shape[0], q.shape[1]
    rep = Hq // kc.shape[2]
    out = torch.empty(B, Hq, 128, device=q.device)
    for b in range(B):
        n = int(lens[b])
        k = kc[b, :n].float().repeat_interleave(rep, 1).transpose(0, 1)  # [Hq, n, 128]
        v = vc[b, :n].float().repeat_interleave(rep, 1).transpose(0, 1)
        if n == 0:
            out[b] = 0
            continue
        out[b] = torch.nn.functional.scaled_dot_product_attention(q[b].float()[:, None], k, v)[:, 0]
    return out


@pytest.mark.parametrize("B,L,Hq,Hk,n_split", [(2, 300, 8, 1, 0), (4, 2304, 64, 8, 0), (3, 1000, 48, 8, 0),
                                               (2, 777, 8, 8, 1), (1, 5000, 16, 1, 7), (5, 130, 4, 2, 0)])
def test_decode_attention(B, L, Hq, Hk, n_split):
    """Split-KV decode kernel against fp32 SDPA: uniform and ragged lengths, GQA groups 1-16,
    single split (direct bf16 output) and merged splits."""
    torch.manual_seed(B * 131 + L)
    q = torch.randn(B, Hq, 128, device=DEV).bfloat16()
    kc = (torch.randn(B, L, Hk, 128, device=DEV) * torch.linspace(0.3, 2.5, L, device=DEV)[None, :, None, None]
          ).bfloat16()
    vc = torch.randn(B, L, Hk, 128, device=DEV).bfloat16()
    o = ops.decode_attention(q, kc, vc, L, n_split=n_split)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(o, _decode_ref(q, kc, vc, [L] * B)) < 1e-2
    lens = torch.randint(0, L + 1, (B,), device=DEV, dtype=torch.int32)
    lens[0] = L
    # cache rows past each length hold garbage (NaN / Inf) that must not reach the output
    for b in range(B):
        kc[b, int(lens[b]):] = float("nan")
        vc[b, int(lens[b]):] = float("inf")
    o2 = ops.decode_attention(q.view(B, 1, Hq, 128), kc, vc, lens, max_len=L, n_split=n_split).view(B, Hq, 128)
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(o2, _decode_ref(q, kc, vc, lens.tolist())) < 1e-2


def test_decode_attention_strided_cache_prefix():
    """A prefix view of a larger cache (the decode path's kc[:, :pos+1]) and a timed comparison
    baseline: the prefill kernel with one query per sequence gives the same result."""
    torch.manual_seed(5)
    B, Lmax, Hq, Hk, n = 4, 4096, 32, 8, 2049
    q = torch.randn(B, 1, Hq, 128, device=DEV).bfloat16()
    kc = torch.randn(B, Lmax, Hk, 128, device=DEV).bfloat16()
    vc = torch.randn(B, Lmax, Hk, 128, device=DEV).bfloat16()
    o = ops.decode_attention(q, kc, vc, n)
    ref = ops.attention(q, kc[:, :n], vc[:, :n])
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert rel_err(o, ref) < 1e-2
