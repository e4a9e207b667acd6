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
// Statistics are two-pass in fp32 (mean, then centred variance) from the
// register copy, which is exact-enough for bf16 activations and avoids the
// cancellation of the one-pass E[x^2]-E[x]^2 form.
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

// VPT = 8-element vectors per thread held in registers (D <= NT*8*VPT).
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) ln_modulate_kernel(LnArgs a) {
  __shared__ float red[NT / 32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = a.x + (size_t)row * a.ldx;
  __nv_bfloat16* y = a.y + (size_t)row * a.ldy;
  const int nvec = a.D / 8;
  float v[VPT][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
      load8(x + vi * 8, v[i]);
#pragma unroll
      for (int e = 0; e < 8; e++) s += v[i][e];
    }
  }
  const float mean = block_sum<NT>(s, red) / a.D;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
#pragma unroll
      for (int e = 0; e < 8; e++) {
        float d = v[i][e] - mean;
        ss += d * d;
      }
    }
  }
  const float rstd = rsqrtf(block_sum<NT>(ss, red) / a.D + a.eps);
  const int mrow = a.mod_rows > 0 ? row / a.mod_rows : 0;
  const float* sc = a.scale ? a.scale + (size_t)mrow * a.mod_stride : nullptr;
  const float* sh = a.shift ? a.shift + (size_t)mrow * a.mod_stride : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int c = vi * 8 + e;
        float t = (v[i][e] - mean) * rstd;
        if (a.weight) t = t * ldf(a.weight, c, a.affine_bf16) + (a.bias ? ldf(a.bias, c, a.affine_bf16) : 0.f);
        if (sc) t = t * (1.f + sc[c]);
        if (sh) t = t + sh[c];
        o[e] = t;
      }
      store8(y + vi * 8, o);
    }
  }
}

template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(RmsArgs a) {
  __shared__ float red[NT / 32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = a.x + (size_t)row * a.ldx;
  __nv_bfloat16* y = a.y + (size_t)row * a.ldy;
  const int nvec = a.D / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
      load8(x + vi * 8, v[i]);
#pragma unroll
      for (int e = 0; e < 8; e++) ss += v[i][e] * v[i][e];
    }
  }
  const float r = a.no_norm ? 1.f : rsqrtf(block_sum<NT>(ss, red) / a.D + a.eps);
  // optional rotary embedding on interleaved pairs, per head of size a.head_dim
  const int pos = a.seq_len > 0 ? row % a.seq_len : 0;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int vi = threadIdx.x + i * NT;
    if (vi < nvec) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int c = vi * 8 + e;
        o[e] = v[i][e] * r * (a.weight ? ldf(a.weight, c, a.weight_bf16) : 1.f);
      }
      if (a.cos != nullptr) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const int c = vi * 8 + e;
          const int pair = (c % a.head_dim) >> 1;
          const float cs = a.cos[(size_t)pos * (a.head_dim / 2) + pair];
          const float sn = a.sin[(size_t)pos * (a.head_dim / 2) + pair];
          const float re = o[e], im = o[e + 1];
          o[e] = re * cs - im * sn;
          o[e + 1] = re * sn + im * cs;
        }
      }
      store8(y + vi * 8, o);
    }
  }
}

#define FT_LAUNCH_ROWS(KER, ARGS, ROWS, D, ST)                                           \
  do {                                                                                   \
    const int nvec = (D) / 8;                                                            \
    if (nvec <= 128 * 4) KER<128, 4><<<(ROWS), 128, 0, (ST)>>>(ARGS);                    \
    else if (nvec <= 256 * 4) KER<256, 4><<<(ROWS), 256, 0, (ST)>>>(ARGS);               \
    else if (nvec <= 512 * 4) KER<512, 4><<<(ROWS), 512, 0, (ST)>>>(ARGS);               \
    else return cudaErrorInvalidValue;                                                   \
  } while (0)

cudaError_t ln_modulate(const LnArgs& a, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (a.D % 8 || a.ldx % 8 || a.ldy % 8) return cudaErrorInvalidValue;
  FT_LAUNCH_ROWS(ln_modulate_kernel, a, rows, a.D, st);
  return cudaGetLastError();
}

cudaError_t rmsnorm(const RmsArgs& a, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (a.D % 8 || a.ldx % 8 || a.ldy % 8) return cudaErrorInvalidValue;
  if (a.cos != nullptr && (a.head_dim % 8 || a.D % a.head_dim || a.seq_len <= 0)) return cudaErrorInvalidValue;
  FT_LAUNCH_ROWS(rmsnorm_kernel, a, rows, a.D, st);
  return cudaGetLastError();
}

}  // namespace ft
