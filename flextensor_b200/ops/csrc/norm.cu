// Row-wise normalisation kernels (memory-bound; one CTA per row, values kept in
// registers between the statistics pass and the write pass so each row is read
// from HBM exactly once):
//
//   ln_modulate     y = LN(x) [* w + b] [* (1 + scale) + shift]     (adaLN modulate)
//   rmsnorm         y = x * rsqrt(mean(x^2) + eps) * w
//   qk_norm_rope    y = rope(rmsnorm(x) * w)  per head, interleaved pairs
//                   (RMSNorm over the full H*Dh row, then complex rotation by
//                   cos/sin tables indexed by token position)
//
// The row stays in registers as packed bf16. LayerNorm statistics are per-thread two-pass
// (mean, then centred M2) merged across the block in one reduction (Chan et al.), which
// avoids the cancellation of the one-pass E[x^2]-E[x]^2 form.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ft_ops_norm.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(norm_device_error)

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) t += red[i];
  return t;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int e = 0; e < 8; e++) f[e] = __bfloat162float(b[e]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float ldf(const void* p, int i, bool is_bf16) {
  return is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                 : reinterpret_cast<const float*>(p)[i];
}

// Eight consecutive per-column parameters starting at column c (c % 8 == 0). VEC: the pointer is
// 16-byte aligned, so one 16-byte load (bf16) or two (fp32) through the read-only path; otherwise
// eight scalar loads.
template <bool VEC>
__device__ __forceinline__ void ldp8(const void* p, int c, bool is_bf16, float (&f)[8]) {
  if constexpr (VEC) {
    if (is_bf16) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + c));
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; e++) f[e] = __bfloat162float(b[e]);
    } else {
      const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + c);
      const float4 lo = __ldg(q), hi = __ldg(q + 1);
      f[0] = lo.x, f[1] = lo.y, f[2] = lo.z, f[3] = lo.w, f[4] = hi.x, f[5] = hi.y, f[6] = hi.z, f[7] = hi.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; e++) f[e] = ldf(p, c + e, is_bf16);
  }
}

// Four consecutive fp32 values (RoPE cos/sin of four pairs).
template <bool VEC>
__device__ __forceinline__ float4 ld4f(const float* p) {
  if constexpr (VEC) return __ldg(reinterpret_cast<const float4*>(p));
  return make_float4(p[0], p[1], p[2], p[3]);
}

// Row statistics in one block reduction: every thread holds (count, mean, M2) of its own
// elements (exact two-pass over its registers), and the pairs merge by Chan et al.'s parallel
// update, n = na + nb, d = mb - ma, mean = ma + d nb / n, M2 = Ma + Mb + d^2 na nb / n, which
// keeps the centred form (no E[x^2] - E[x]^2 cancellation) with half the barriers of two sums.
__device__ __forceinline__ void chan_merge(float& n, float& m, float& M, float nb, float mb, float Mb) {
  const float tot = n + nb;
  if (nb > 0.f) {
    const float d = mb - m;
    const float f = nb / tot;
    m = fmaf(d, f, m);
    M = M + Mb + d * d * n * f;
    n = tot;
  }
}

template <int NT>
__device__ __forceinline__ void block_mean_m2(float n, float m, float M, float* red, float& mean, float& m2) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float nb = __shfl_xor_sync(0xffffffff, n, o);
    const float mb = __shfl_xor_sync(0xffffffff, m, o);
    const float Mb = __shfl_xor_sync(0xffffffff, M, o);
    if (n == 0.f) {
      n = nb, m = mb, M = Mb;
    } else {
      chan_merge(n, m, M, nb, mb, Mb);
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[3 * w] = n, red[3 * w + 1] = m, red[3 * w + 2] = M;
  __syncthreads();
  float tn = red[0], tm = red[1], tM = red[2];
#pragma unroll
  for (int i = 1; i < NT / 32; i++) {
    if (tn == 0.f) {
      tn = red[3 * i], tm = red[3 * i + 1], tM = red[3 * i + 2];
    } else {
      chan_merge(tn, tm, tM, red[3 * i], red[3 * i + 1], red[3 * i + 2]);
    }
  }
  mean = tm;
  m2 = tM;
}

// Marks the packed row registers as rewritten, so each pass converts them again instead of
// keeping a second, fp32 copy of the row live (the point of holding it packed).
template <int VPT>
__device__ __forceinline__ void refresh(uint4 (&raw)[VPT]) {
#pragma unroll
  for (int i = 0; i < VPT; i++) asm volatile("" : "+r"(raw[i].x), "+r"(raw[i].y), "+r"(raw[i].z), "+r"(raw[i].w));
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int e = 0; e < 8; e++) f[e] = __bfloat162float(b[e]);
}

// VPT = 8-element vectors per thread, held in registers as packed bf16 (D <= NT*8*VPT). VEC =
// every per-column parameter array is 16-byte aligned (vector loads; the parameter traffic is
// otherwise the limiter of these HBM-bound kernels, not the row itself).
template <int NT, int VPT, bool VEC>
__global__ void __launch_bounds__(NT) ln_modulate_kernel(LnArgs a) {
  __shared__ float red[3 * (NT / 32)];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = a.x + (size_t)row * a.ldx;
  __nv_bfloat16* y = a.y + (size_t)row * a.ldy;
  const int nvec = a.D / 8;
  uint4 raw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) raw[i] = *reinterpret_cast<const uint4*>(x + vi * 8);
  }
  // this thread's (count, mean, M2), two passes over its registers
  float cnt = 0.f, s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    if (threadIdx.x + i * NT < nvec) {
      float f[8];
      unpack8(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; e++) s += f[e];
      cnt += 8.f;
    }
  }
  const float tmean = cnt > 0.f ? s / cnt : 0.f;
  refresh(raw);
  float tm2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    if (threadIdx.x + i * NT < nvec) {
      float f[8];
      unpack8(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const float d = f[e] - tmean;
        tm2 = fmaf(d, d, tm2);
      }
    }
  }
  float mean, m2;
  block_mean_m2<NT>(cnt, tmean, tm2, red, mean, m2);
  const float rstd = rsqrtf(m2 / a.D + a.eps);
  refresh(raw);
  const int mrow = a.mod_rows > 0 ? row / a.mod_rows : 0;
  const float* sc = a.scale ? a.scale + (size_t)mrow * a.mod_stride : nullptr;
  const float* sh = a.shift ? a.shift + (size_t)mrow * a.mod_stride : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
      const int c0 = vi * 8;
      float o[8], p[8];
      unpack8(raw[i], o);
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] = (o[e] - mean) * rstd;
      if (a.weight) {
        ldp8<VEC>(a.weight, c0, a.affine_bf16, p);
#pragma unroll
        for (int e = 0; e < 8; e++) o[e] *= p[e];
      }
      if (a.bias) {
        ldp8<VEC>(a.bias, c0, a.affine_bf16, p);
#pragma unroll
        for (int e = 0; e < 8; e++) o[e] += p[e];
      }
      if (sc) {
        ldp8<VEC>(sc, c0, false, p);
#pragma unroll
        for (int e = 0; e < 8; e++) o[e] = fmaf(o[e], p[e], o[e]);
      }
      if (sh) {
        ldp8<VEC>(sh, c0, false, p);
#pragma unroll
        for (int e = 0; e < 8; e++) o[e] += p[e];
      }
      store8(y + c0, o);
    }
  }
}

template <int NT, int VPT, bool VEC>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(RmsArgs a) {
  __shared__ float red[NT / 32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = a.x + (size_t)row * a.ldx;
  __nv_bfloat16* y = a.y + (size_t)row * a.ldy;
  const int nvec = a.D / 8;
  uint4 raw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) raw[i] = *reinterpret_cast<const uint4*>(x + vi * 8);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    if (threadIdx.x + i * NT < nvec) {
      float f[8];
      unpack8(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; e++) ss = fmaf(f[e], f[e], ss);
    }
  }
  const float r = a.no_norm ? 1.f : rsqrtf(block_sum<NT>(ss, red) / a.D + a.eps);
  // optional rotary embedding on interleaved pairs, per head of size a.head_dim (a multiple of 8,
  // so one 8-element vector is four pairs of one head)
  const int pos = a.seq_len > 0 ? row % a.seq_len : 0;
  const int half = a.head_dim / 2;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
      const int c0 = vi * 8;
      float o[8];
      unpack8(raw[i], o);
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] *= r;
      if (a.weight) {
        float w[8];
        ldp8<VEC>(a.weight, c0, a.weight_bf16, w);
#pragma unroll
        for (int e = 0; e < 8; e++) o[e] *= w[e];
      }
      if (a.cos != nullptr) {
        const size_t t = (size_t)pos * half + (c0 % a.head_dim) / 2;
        const float4 cs = ld4f<VEC>(a.cos + t), sn = ld4f<VEC>(a.sin + t);
        const float cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float re = o[2 * q], im = o[2 * q + 1];
          o[2 * q] = re * cv[q] - im * sv[q];
          o[2 * q + 1] = re * sv[q] + im * cv[q];
        }
      }
      store8(y + c0, o);
    }
  }
}

// Launch shape: 128 threads and the fewest vectors per thread that cover the row (no idle lanes
// at D = 5120: 640 vectors = 128 x 5), wider CTAs past 8192 columns. The scalar-parameter
// variant keeps three shapes only.
#define FT_LAUNCH_ROWS(KER, ARGS, ROWS, D, VEC, ST)                                      \
  do {                                                                                   \
    const int nvec = (D) / 8;                                                            \
    if (VEC && nvec <= 128 * 8) {                                                        \
      switch ((nvec + 127) / 128) {                                                      \
        case 1: KER<128, 1, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        case 2: KER<128, 2, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        case 3: KER<128, 3, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        case 4: KER<128, 4, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        case 5: KER<128, 5, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        case 6: KER<128, 6, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        case 7: KER<128, 7, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;                \
        default: KER<128, 8, true><<<(ROWS), 128, 0, (ST)>>>(ARGS); break;               \
      }                                                                                  \
    } else if (VEC && nvec <= 256 * 8) KER<256, 8, true><<<(ROWS), 256, 0, (ST)>>>(ARGS);  \
    else if (VEC && nvec <= 512 * 8) KER<512, 8, true><<<(ROWS), 512, 0, (ST)>>>(ARGS);    \
    else if (nvec <= 128 * 4) KER<128, 4, false><<<(ROWS), 128, 0, (ST)>>>(ARGS);        \
    else if (nvec <= 256 * 4) KER<256, 4, false><<<(ROWS), 256, 0, (ST)>>>(ARGS);        \
    else if (nvec <= 512 * 8) KER<512, 8, false><<<(ROWS), 512, 0, (ST)>>>(ARGS);        \
    else return cudaErrorInvalidValue;                                                   \
  } while (0)

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaError_t ln_modulate(const LnArgs& a, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (a.D % 8 || a.ldx % 8 || a.ldy % 8) return cudaErrorInvalidValue;
  const bool vec = al16(a.weight) && al16(a.bias) && al16(a.scale) && al16(a.shift) && a.mod_stride % 4 == 0;
  FT_LAUNCH_ROWS(ln_modulate_kernel, a, rows, a.D, vec, st);
  return cudaGetLastError();
}

cudaError_t rmsnorm(const RmsArgs& a, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (a.D % 8 || a.ldx % 8 || a.ldy % 8) return cudaErrorInvalidValue;
  if (a.cos != nullptr && (a.head_dim % 8 || a.D % a.head_dim || a.seq_len <= 0)) return cudaErrorInvalidValue;
  const bool vec = al16(a.weight) && al16(a.cos) && al16(a.sin);
  FT_LAUNCH_ROWS(rmsnorm_kernel, a, rows, a.D, vec, st);
  return cudaGetLastError();
}

}  // namespace ft
