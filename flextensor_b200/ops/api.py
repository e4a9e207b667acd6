"""Python entry points of the native kernels.

All ops run on the caller's current CUDA stream, take bf16 activations and
return bf16; reductions and epilogues are computed in fp32 inside the kernels.
They require the native extension on CUDA tensors (no silent fallback).
"""

from __future__ import annotations

import math

import torch

from flextensor_b200.ops import native

EPI = {"none": 0, "bias": 1, "gelu": 2, "gate_res": 3, "res": 4}

# Number of native kernel launches issued through these entry points (each call = one launch).
_launches = 0


def launch_count() -> int:
    return _launches


def _count(n: int = 1) -> None:
    global _launches
    _launches += n


def _2d(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, epi: str = "bias",
           residual: torch.Tensor | None = None, gate: torch.Tensor | None = None, gate_rows: int = 0,
           out: torch.Tensor | None = None, force_bn: int = 0) -> torch.Tensor:
    """``epi(x @ weight.T + bias)`` on tcgen05 tensor cores.

    epi: ``none`` | ``bias`` | ``gelu`` (tanh GELU) | ``res`` (residual + y) |
    ``gate_res`` (residual + gate * y; gate fp32 ``[N]`` or ``[M/gate_rows, N]``).
    ``out`` may alias ``residual`` (in-place residual update).
    """
    lead = x.shape[:-1]
    a = _2d(x)
    if a.stride(-1) != 1:
        a = a.contiguous()
    n = weight.shape[0]
    if out is None:
        out = torch.empty(*lead, n, dtype=torch.bfloat16, device=x.device)
    o2 = _2d(out)
    r2 = _2d(residual) if residual is not None else None
    e = EPI[epi]
    if e in (1, 2) and bias is None:
        e = EPI["none"] if e == 1 else e
    native.lib().gemm(a, weight, o2, bias, r2, gate, int(gate_rows), e, int(force_bn))
    _count()
    return out


def layernorm_modulate(x: torch.Tensor, scale: torch.Tensor | None = None, shift: torch.Tensor | None = None, *,
                       weight: torch.Tensor | None = None, bias: torch.Tensor | None = None, mod_rows: int = 0,
                       eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """``LN(x) [*w+b] [*(1+scale)+shift]`` per row; scale/shift fp32 ``[D]`` or ``[M/mod_rows, D]``."""
    x2 = _2d(x)
    if out is None:
        out = torch.empty_like(x)
    native.lib().ln_modulate(x2, _2d(out), weight, bias, scale, shift, int(mod_rows), float(eps))
    _count()
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor | None = None, *, eps: float = 1e-6,
            out: torch.Tensor | None = None) -> torch.Tensor:
    x2 = _2d(x)
    if out is None:
        out = torch.empty(x2.shape, dtype=x.dtype, device=x.device).view(x.shape)
    native.lib().rmsnorm(x2, _2d(out), weight, None, None, 0, 0, float(eps))
    _count()
    return out


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, head_dim: int, seq_len: int, *,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """Interleaved-pair rotary embedding per head (row position = row index mod ``seq_len``)."""
    x2 = _2d(x)
    if out is None:
        out = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    native.lib().rmsnorm(x2, _2d(out), None, cos, sin, int(head_dim), int(seq_len), -1.0)
    _count()
    return out


def qk_rmsnorm_rope(x: torch.Tensor, weight: torch.Tensor | None, cos: torch.Tensor, sin: torch.Tensor,
                    head_dim: int, seq_len: int, *, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the full row, then interleaved-pair RoPE per head (tables ``[seq_len, head_dim/2]``)."""
    x2 = _2d(x)
    if out is None:
        out = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    native.lib().rmsnorm(x2, _2d(out), weight, cos, sin, int(head_dim), int(seq_len), float(eps))
    _count()
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float | None = None,
              causal: bool = False, out: torch.Tensor | None = None, _diag_mode: int = 0,
              _trace: torch.Tensor | None = None) -> torch.Tensor:
    """Softmax attention on ``[B, S, H, 128]`` bf16 tensors (GQA when k/v have fewer heads)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    native.lib().attention(q, k, v, out, float(scale), bool(causal), int(_diag_mode), _trace)
    _count()
    return out


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: int | torch.Tensor, *,
                     max_len: int | None = None, scale: float | None = None, out: torch.Tensor | None = None,
                     n_split: int = 0) -> torch.Tensor:
    """One decode step of attention: ``q [B, Hq, 128]`` (or ``[B, 1, Hq, 128]``), one query per
    sequence, over the KV cache ``k_cache`` / ``v_cache [B, L, Hk, 128]`` (GQA when Hk < Hq).
    ``kv_len``: keys per sequence, an int (every sequence) or an int32 CUDA tensor ``[B]`` (then
    ``max_len`` bounds it, default L). Keys are split over CTAs and the splits merged in a second
    pass (``n_split``: 0 = about one CTA per SM)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if isinstance(kv_len, torch.Tensor):
        seqlens, n = kv_len, 0
        ml = int(max_len) if max_len is not None else int(k_cache.shape[1])
    else:
        seqlens, n = None, int(kv_len)
        ml = n
    if n_split <= 0:
        sms = torch.cuda.get_device_properties(q.device).multi_processor_count
        n_split = native.lib().decode_splits(int(k_cache.shape[0]), int(k_cache.shape[2]), ml, sms)
    native.lib().decode_attention(q, k_cache, v_cache, out, seqlens, n, ml, float(scale), int(n_split))
    _count(1 if n_split == 1 else 2)  # the split kernel, plus the combine pass when split
    return out


def attention_cp(q: torch.Tensor, kv_local: torch.Tensor, *, peer_kv: list[int], flags_ptr: int, flag_stride: int,
                 peer_acks: list[int], rank: int, shard_rows: int, epoch: int, counters: torch.Tensor,
                 scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Context-parallel attention: local queries ``q [B, Sq, Hq, 128]`` over the keys of every
    rank. ``kv_local [B, 2, Sk, Hk, 128]`` is this rank's full-sequence K/V buffer with its own
    rows ``[rank*shard_rows, (rank+1)*shard_rows)`` written and published (epoch flag) before
    the call; the kernel pulls the other ranks' rows from ``peer_kv`` over NVLink while it
    computes (see ``attention_sm100.cu``)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    native.lib().attention_cp(q, kv_local, out, float(scale), [int(p) for p in peer_kv], int(flags_ptr),
                              int(flag_stride), [int(p) for p in peer_acks], int(rank), int(shard_rows), int(epoch),
                              counters)
    _count()
    return out


TP_EPI = {"none": 0, "bias": 1, "swiglu": 2, "gelu": 3}


def tp_allgather_gemm(a_full: torch.Tensor, weight: torch.Tensor, *, peer_a: list[int], flags_ptr: int,
                      flag_stride: int, peer_acks: list[int], rank: int, epoch: int, counters: torch.Tensor,
                      bias: torch.Tensor | None = None, epi: str = "none", out: torch.Tensor | None = None,
                      _pair: bool = False):
    """All-gather -> GEMM: ``a_full [M, K]`` is this rank's full-row buffer with its own rows
    written and published; the kernel pulls peers' rows over NVLink while multiplying.
    ``epi="swiglu"``: weight rows interleaved (gate, up) -> ``[M, N/2]``. ``_pair``: the
    experimental CTA-pair (cta_group::2) kernel (tested on emulated ranks)."""
    n_out = weight.shape[0] // 2 if epi == "swiglu" else weight.shape[0]
    if out is None:
        out = torch.empty(a_full.shape[0], n_out, dtype=torch.bfloat16, device=a_full.device)
    native.lib().tp_ag_gemm(a_full, weight, out, bias, TP_EPI[epi], [int(p) for p in peer_a], int(flags_ptr),
                            int(flag_stride), [int(p) for p in peer_acks], int(rank), int(epoch), counters,
                            bool(_pair))
    _count()
    return out


def tp_ag_counter_words(rows_total: int, world: int) -> int:
    """int32 scratch words ``tp_allgather_gemm`` needs for ``rows_total`` rows over ``world``
    ranks: per-peer tickets plus a landed-byte count per 128-row block of every peer."""
    return world * (2 + (rows_total // world + 127) // 128) if world > 1 else 2 * world


def tp_gemm_reducescatter(a: torch.Tensor, weight: torch.Tensor, *, stage: list[int], peer_flags: list[int],
                          rank: int, epoch: int, counters: torch.Tensor, _pair: bool = False) -> None:
    """GEMM -> reduce-scatter, sender side: partial ``a @ weight.T`` rows go straight into the
    owning rank's staging slot ``[world, M/world, N]`` (``stage[p]``); then flags. ``_pair``:
    the experimental CTA-pair (cta_group::2) kernel (tested on emulated ranks)."""
    native.lib().tp_gemm_rs(a, weight, [int(p) for p in stage], [int(p) for p in peer_flags], int(rank), int(epoch),
                            counters, bool(_pair))
    _count()


def tp_reduce(stage: torch.Tensor, world: int, rows: int, out: torch.Tensor, *, flags_ptr: int, flag_stride: int,
              epoch: int, peer_acks: list[int], rank: int, residual: torch.Tensor | None = None,
              out_peers: list[int] | None = None, row_base: int = 0, stage_rows: int = 0,
              bias: torch.Tensor | None = None, gate: torch.Tensor | None = None, gate_rows: int = 0,
              grow0: int = 0) -> torch.Tensor:
    """Owner side: ``out = residual + gate * (sum of the world partial rows + bias)`` once every
    sender flagged (``gate``: fp32 ``[groups, N]``, one row per ``gate_rows`` global rows, the
    first owned row being global row ``grow0``). ``out_peers`` (all-reduce): write the reduced
    rows at ``row_base`` of every rank's output instead; the acknowledgements that follow also
    certify that the rows arrived."""
    native.lib().tp_reduce(stage, int(world), int(rows), out, residual, int(flags_ptr), int(flag_stride), int(epoch),
                           [int(p) for p in peer_acks], int(rank), [int(p) for p in (out_peers or [])],
                           int(row_base), int(stage_rows), bias, gate, int(gate_rows), int(grow0))
    _count(2)
    return out


def tp_rmsnorm(x: torch.Tensor, weight: torch.Tensor | None, *, d_full: int, part_peers: list[int], stage_rows: int,
               peer_flags: list[int], flags_ptr: int, flag_stride: int, peer_acks: list[int], rank: int, epoch: int,
               counter: torch.Tensor, eps: float = 1e-6, cos: torch.Tensor | None = None,
               sin: torch.Tensor | None = None, head_dim: int = 0, seq_len: int = 0,
               out: torch.Tensor | None = None, _phases: int = 3) -> torch.Tensor:
    """RMSNorm over a hidden dimension whose columns are split across tensor-parallel ranks:
    per-row partial sums of squares go to every rank over peer stores, each rank then scales its
    own columns (weight shard, optional interleaved-pair RoPE per head). ``_phases`` (tests that
    emulate several ranks on one GPU): 1 = partial sums and publish only, 2 = wait and scale only."""
    x2 = _2d(x)
    if out is None:
        out = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    native.lib().tp_rmsnorm(x2, _2d(out), weight, cos, sin, int(head_dim), int(seq_len), float(eps), int(d_full),
                            [int(p) for p in part_peers], int(stage_rows), [int(p) for p in peer_flags],
                            int(flags_ptr), int(flag_stride), [int(p) for p in peer_acks], int(rank), int(epoch),
                            counter, int(_phases))
    _count((1 if _phases & 1 else 0) + (2 if _phases & 2 else 0))
    return out


_swiglu_dummies: dict = {}


def linear_swiglu(x: torch.Tensor, weight_gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(x @ Wg.T) * (x @ Wu.T)`` with gate/up rows interleaved in ``weight_gate_up`` ``[2F, K]``
    (one tcgen05 GEMM, SwiGLU in the epilogue; the all-gather GEMM kernel with one rank)."""
    a = x if x.is_contiguous() else x.contiguous()
    key = a.device
    d = _swiglu_dummies.get(key)
    if d is None:
        d = (torch.zeros(2, dtype=torch.int64, device=a.device), torch.zeros(2, dtype=torch.int32, device=a.device))
        _swiglu_dummies[key] = d
    flags, counters = d
    return tp_allgather_gemm(a, weight_gate_up, peer_a=[a.data_ptr()], flags_ptr=flags.data_ptr(), flag_stride=1,
                             peer_acks=[flags.data_ptr() + 8], rank=0, epoch=0, counters=counters, epi="swiglu",
                             out=out)
