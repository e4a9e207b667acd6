// Decode attention (one query per sequence over a KV cache), split over the keys
// ("flash-decoding"), GQA, head_dim 128, bf16, for sm_100a.
//
// A decode step reads every cached key and value once and does ~2 FLOPs per byte: the kernel is
// bound by HBM bandwidth, not by a tensor core (the G <= 16 query heads of a KV group would fill
// at most 1/8 of a 128-row tcgen05 tile). So it streams the cache with TMA and computes on the
// FMA pipe:
//   * grid = (key split, KV head, sequence); each CTA covers a contiguous run of 64-key tiles of
//     one sequence's cache for one KV head and ALL G query heads that share it (the K/V bytes
//     are read once per group, not once per query head);
//   * warp 8 (one elected lane) loads K and V tiles with 4-D tensor maps ([B, L, Hk, 128]
//     cache, 128-byte swizzle, no multicast) into a 2-stage ring guarded by mbarriers;
//   * warps 0-7: S = q K^T with four threads per key (each G/4 of the heads, fp32 pairs on the
//     FMA pipe), an online softmax per head (warp h owns head h: tile max and sum by shuffles,
//     exp2 on MUFU, running max / sum in registers), and O += P V with warp w owning keys
//     8w..8w+7 of the tile and lane l owning dims 4l..4l+3 of every head;
//   * after the last tile the eight warps' partial O are summed in shared memory; a single split
//     writes bf16 output directly, otherwise (O, max, sum) per split go to a caller-provided
//     fp32 scratch and decode_combine_kernel merges them (weights 2^(m_s - M)).
// Keys at or past a sequence's length are masked. All waits are bounded: a timeout records the
// device error word, the producer drains its own loads, and the consumers fall through their
// remaining tiles without computing.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ft_ops.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(decode_device_error)

namespace {

constexpr int DHD = 128;              // head dim
constexpr int KT = 64;                // keys per tile
constexpr int DSTAGES = 2;
constexpr int DCONS = 256;            // consumer threads (warps 0-7)
constexpr int DTHREADS = DCONS + 32;  // + producer warp
constexpr int BOX_BYTES = KT * 128;   // one [64 keys x 64 dims] bf16 box (8 KB)
constexpr int QSTRIDE = DHD + 4;      // padded fp32 q rows (bank spread across heads)

struct DecArgs {
  int B, Hq, Hk, L;            // L: cache capacity (tokens)
  const __nv_bfloat16* q;      // [B, Hq, 128]
  long long q_b;               // elements between sequences
  __nv_bfloat16* o;            // [B, Hq, 128]
  long long o_b;
  const int* seqlens;          // [B] keys per sequence, or null: every sequence has kv_len keys
  int kv_len;
  float scale_log2;            // softmax scale * log2(e)
  int n_split, tiles_per_split;
  float* part_o;               // [n_split, B, Hq, 128] unnormalised partial outputs
  float* part_ml;              // [n_split, B, Hq, 2]   running max (log2 units) and sum
};

template <int G>
struct DecSmem {
  uint8_t k[DSTAGES][2 * BOX_BYTES];
  uint8_t v[DSTAGES][2 * BOX_BYTES];
  alignas(16) float q[G][QSTRIDE];
  float s[G][KT + 1];
  alignas(16) float p[KT][(G + 3) / 4 * 4];  // P per key, all heads (float4 reads)
  float alpha[G];
  float ml[G][2];
  uint64_t full[DSTAGES], empty[DSTAGES];
};

// 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled box
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void bf16x8_to_f32(const uint4& w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int G>
__global__ void __launch_bounds__(DTHREADS, G <= 8 ? 2 : 1)
    decode_split_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, DecArgs a) {
  constexpr int HPT = (G + 3) / 4;  // heads per thread in q K^T
  constexpr int GP = (G + 3) / 4 * 4;
  extern __shared__ uint8_t smem_raw[];
  DecSmem<G>& sm = *reinterpret_cast<DecSmem<G>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int len = a.seqlens ? min(a.seqlens[b], a.L) : a.kv_len;
  const int t_begin = split * a.tiles_per_split;
  const int t_end = min(t_begin + a.tiles_per_split, (len + KT - 1) / KT);
  const int n_tiles = max(0, t_end - t_begin);

  if (tid == 0) {
    for (int s = 0; s < DSTAGES; s++) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 8);  // lane 0 of every consumer warp
    }
    fence_barrier_init();
  }
  // q of the group, pre-scaled into log2 units
  for (int i = tid; i < G * DHD; i += DTHREADS) {
    const int g = i / DHD, d = i % DHD;
    sm.q[g][d] = __bfloat162float(a.q[(long long)b * a.q_b + (long long)(hk * G + g) * DHD + d]) * a.scale_log2;
  }
  __syncthreads();

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t pend = 0, pph = 0;
      bool ok = true;
      for (int i = 0; i < n_tiles && ok; i++) {
        const int s = i % DSTAGES;
        const uint32_t ph = (i / DSTAGES) & 1;
        if (!mbar_wait(&sm.empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        const int key0 = (t_begin + i) * KT;
        mbar_arrive_expect_tx(&sm.full[s], 4 * BOX_BYTES);
        for (int c = 0; c < 2; c++) {
          tma_load_4d(sm.k[s] + c * BOX_BYTES, &tmK, &sm.full[s], c * 64, hk, key0, b);
          tma_load_4d(sm.v[s] + c * BOX_BYTES, &tmV, &sm.full[s], c * 64, hk, key0, b);
        }
        pend |= 1u << s;
        pph = (pph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {
        const long long t0 = clock64();
        for (int s = 0; s < DSTAGES; s++)
          if (pend >> s & 1)
            while (!mbar_try_wait(smem_u32(&sm.full[s]), (pph >> s) & 1) &&
                   (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
            }
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    const int key = tid & (KT - 1), hg = tid >> 6;      // q K^T: thread = (key, head group)
    const int hs = warp;                                // softmax: warp = head (and head + 8)
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    unsigned long long acc[G][2];  // (dims 4l, 4l+1) and (4l+2, 4l+3) of every head, fp32 pairs
#pragma unroll
    for (int g = 0; g < G; g++) acc[g][0] = acc[g][1] = 0ull;
    bool ok = true;
    for (int i = 0; i < n_tiles; i++) {
      const int s = i % DSTAGES;
      const uint32_t ph = (i / DSTAGES) & 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.full[s], ph));
      const int key0 = (t_begin + i) * KT;
      // ---- S = q K^T for this thread's key and heads
      if (ok) {
        const uint8_t* kt = sm.k[s];
        unsigned long long accp[HPT];
#pragma unroll
        for (int u = 0; u < HPT; u++) accp[u] = 0ull;
#pragma unroll 4
        for (int c = 0; c < 16; c++) {
          const uint4 w = *reinterpret_cast<const uint4*>(kt + (c >> 3) * BOX_BYTES + swz(key, c & 7));
          float kf[8];
          bf16x8_to_f32(w, kf);
#pragma unroll
          for (int u = 0; u < HPT; u++) {
            const int g = hg * HPT + u;
            if (g < G) {
              const float4 q0 = *reinterpret_cast<const float4*>(&sm.q[g][c * 8]);
              const float4 q1 = *reinterpret_cast<const float4*>(&sm.q[g][c * 8 + 4]);
              unsigned long long x = accp[u];
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(x) : "l"(((unsigned long long)__float_as_uint(kf[1]) << 32) | __float_as_uint(kf[0])),
                  "l"(((unsigned long long)__float_as_uint(q0.y) << 32) | __float_as_uint(q0.x)));
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(x) : "l"(((unsigned long long)__float_as_uint(kf[3]) << 32) | __float_as_uint(kf[2])),
                  "l"(((unsigned long long)__float_as_uint(q0.w) << 32) | __float_as_uint(q0.z)));
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(x) : "l"(((unsigned long long)__float_as_uint(kf[5]) << 32) | __float_as_uint(kf[4])),
                  "l"(((unsigned long long)__float_as_uint(q1.y) << 32) | __float_as_uint(q1.x)));
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(x) : "l"(((unsigned long long)__float_as_uint(kf[7]) << 32) | __float_as_uint(kf[6])),
                  "l"(((unsigned long long)__float_as_uint(q1.w) << 32) | __float_as_uint(q1.z)));
              accp[u] = x;
            }
          }
        }
        const bool valid = key0 + key < len;
#pragma unroll
        for (int u = 0; u < HPT; u++) {
          const int g = hg * HPT + u;
          if (g < G) {
            const float sv = __uint_as_float((uint32_t)accp[u]) + __uint_as_float((uint32_t)(accp[u] >> 32));
            sm.s[g][key] = valid ? sv : -INFINITY;
          }
        }
      }
      cons_sync();
      // ---- online softmax, one warp per head
      if (ok) {
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          const int g = hs + 8 * hh;
          if (g < G) {
            const float s0 = sm.s[g][lane], s1 = sm.s[g][lane + 32];
            float mx = fmaxf(s0, s1);
#pragma unroll
            for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[hh], mx);
            const float msub = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = m_run[hh] == -INFINITY ? 0.f : ex2f(m_run[hh] - msub);
            const float p0 = ex2f(s0 - msub), p1 = ex2f(s1 - msub);
            float ps = p0 + p1;
#pragma unroll
            for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l_run[hh] = l_run[hh] * alpha + ps;
            m_run[hh] = m_new;
            sm.p[lane][g] = p0;
            sm.p[lane + 32][g] = p1;
            if (lane == 0) sm.alpha[g] = alpha;
          }
        }
        if (G < GP && warp == 0 && lane < KT / 2) {  // padded heads read as zero
#pragma unroll
          for (int g = G; g < GP; g++) {
            sm.p[lane][g] = 0.f;
            sm.p[lane + 32][g] = 0.f;
          }
        }
      }
      cons_sync();
      // ---- O += P V: warp owns keys 8w..8w+7, lane owns dims 4l..4l+3 of every head
      if (ok) {
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float al = sm.alpha[g];
          const unsigned long long al2 = ((unsigned long long)__float_as_uint(al) << 32) | __float_as_uint(al);
#pragma unroll
          for (int e = 0; e < 2; e++) asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(acc[g][e]) : "l"(al2));
        }
        const uint8_t* vt = sm.v[s] + (lane >> 4) * BOX_BYTES;
        const int cc = (lane & 15) >> 1, sub = (lane & 1) * 8;
        const int nvalid = len - key0;  // keys past the length: P is 0, but their V rows may be
                                        // uninitialised cache memory (0 * NaN = NaN), so skip them
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
          const int kr = warp * 8 + kk;
          if (kr >= nvalid) break;
          const uint2 w = *reinterpret_cast<const uint2*>(vt + swz(kr, cc) + sub);
          const unsigned long long v01 =
              ((unsigned long long)(w.x & 0xffff0000u) << 32) | (unsigned long long)(w.x << 16);
          const unsigned long long v23 =
              ((unsigned long long)(w.y & 0xffff0000u) << 32) | (unsigned long long)(w.y << 16);
#pragma unroll
          for (int g4 = 0; g4 < GP; g4 += 4) {
            const float4 pp = *reinterpret_cast<const float4*>(&sm.p[kr][g4]);
            const float pv[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
              if (g4 + u < G) {
                const unsigned long long p2 =
                    ((unsigned long long)__float_as_uint(pv[u]) << 32) | __float_as_uint(pv[u]);
                asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[g4 + u][0]) : "l"(p2), "l"(v01));
                asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc[g4 + u][1]) : "l"(p2), "l"(v23));
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);
    }
    // ---- sum the eight warps' partial O in the K/V ring: every tile loaded has been consumed
    // and the producer issues nothing more
    cons_sync();
    float* red = reinterpret_cast<float*>(&sm.k[0][0]);  // [8 warps][G][128]
#pragma unroll
    for (int g = 0; g < G; g++)
      *reinterpret_cast<float4*>(&red[(warp * G + g) * DHD + lane * 4]) =
          make_float4(__uint_as_float((uint32_t)acc[g][0]), __uint_as_float((uint32_t)(acc[g][0] >> 32)),
                      __uint_as_float((uint32_t)acc[g][1]), __uint_as_float((uint32_t)(acc[g][1] >> 32)));
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int g = hs + 8 * hh;
      if (g < G && lane == 0) {
        sm.ml[g][0] = m_run[hh];
        sm.ml[g][1] = l_run[hh];
      }
    }
    cons_sync();
    for (int i = tid; i < G * DHD; i += DCONS) {
      const int g = i / DHD, d = i % DHD;
      float o = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) o += red[(w * G + g) * DHD + d];
      const int hq = hk * G + g;
      if (a.n_split == 1) {
        const float l = sm.ml[g][1];
        a.o[(long long)b * a.o_b + (long long)hq * DHD + d] = __float2bfloat16(ok && l > 0.f ? o / l : 0.f);
      } else {
        const long long row = ((long long)split * a.B + b) * a.Hq + hq;
        a.part_o[row * DHD + d] = ok ? o : 0.f;
        if (d == 0) {
          a.part_ml[row * 2] = ok ? sm.ml[g][0] : -INFINITY;
          a.part_ml[row * 2 + 1] = ok ? sm.ml[g][1] : 0.f;
        }
      }
    }
  }
}

// Merge the splits: O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s. One CTA per (b, q head),
// thread = dim.
__global__ void __launch_bounds__(DHD) decode_combine_kernel(DecArgs a) {
  const int row = blockIdx.x;  // b * Hq + hq
  const int b = row / a.Hq, hq = row % a.Hq;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < a.n_split; s++) M = fmaxf(M, a.part_ml[((long long)s * a.B * a.Hq + row) * 2]);
  float num = 0.f, den = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < a.n_split; s++) {
      const long long r = (long long)s * a.B * a.Hq + row;
      const float ms = a.part_ml[r * 2];
      if (ms == -INFINITY) continue;
      const float w = ex2f(ms - M);
      den += w * a.part_ml[r * 2 + 1];
      num += w * a.part_o[r * DHD + d];
    }
  }
  a.o[(long long)b * a.o_b + (long long)hq * DHD + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

bool make_tmap_cache(CUtensorMap* map, const void* base, int Hk, int L, int B, long long tok_stride,
                     long long batch_stride) {
  return make_tmap_4d_bf16(map, base, DHD, (uint64_t)Hk, (uint64_t)L, (uint64_t)B, DHD, (uint64_t)tok_stride,
                           (uint64_t)batch_stride, 64, 1, KT, 1);
}

template <int G>
cudaError_t launch_g(const CUtensorMap& tk, const CUtensorMap& tv, const DecArgs& a, dim3 grid, cudaStream_t st) {
  const int smem = (int)sizeof(DecSmem<G>) + 1024;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  decode_split_kernel<G><<<grid, DTHREADS, smem, st>>>(tk, tv, a);
  return cudaGetLastError();
}

}  // namespace

int decode_splits(int B, int Hk, int max_len, int num_sms) {
  const int tiles = (max(max_len, 1) + KT - 1) / KT;
  const int base = max(1, B * Hk);
  int n = (2 * max(num_sms, 1) + base - 1) / base;  // about two CTAs per SM
  n = max(1, min(n, (tiles + 1) / 2));               // at least two tiles per split where possible
  return n;
}

size_t decode_scratch_floats(int B, int Hq, int n_split) {
  return n_split > 1 ? (size_t)n_split * B * Hq * (DHD + 2) : 0;
}

cudaError_t decode_attention(const DecodeProblem& p, cudaStream_t stream) {
  if (p.B == 0) return cudaSuccess;
  if (p.Hk <= 0 || p.Hq % p.Hk || p.L <= 0) return cudaErrorInvalidValue;
  const int G = p.Hq / p.Hk;
  if ((reinterpret_cast<uintptr_t>(p.k) & 15) || (reinterpret_cast<uintptr_t>(p.v) & 15)) return cudaErrorMisalignedAddress;
  CUtensorMap tk, tv;
  if (!make_tmap_cache(&tk, p.k, p.Hk, p.L, p.B, p.k_tok, p.k_batch)) return cudaErrorInvalidValue;
  if (!make_tmap_cache(&tv, p.v, p.Hk, p.L, p.B, p.v_tok, p.v_batch)) return cudaErrorInvalidValue;
  DecArgs a;
  a.B = p.B;
  a.Hq = p.Hq;
  a.Hk = p.Hk;
  a.L = p.L;
  a.q = p.q;
  a.q_b = p.q_b;
  a.o = p.o;
  a.o_b = p.o_b;
  a.seqlens = p.seqlens;
  a.kv_len = p.kv_len;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.n_split = max(1, p.n_split);
  const int tiles = (max(p.max_len, 1) + KT - 1) / KT;
  a.tiles_per_split = (tiles + a.n_split - 1) / a.n_split;
  a.part_o = p.scratch;
  a.part_ml = p.scratch ? p.scratch + (size_t)a.n_split * p.B * p.Hq * DHD : nullptr;
  if (a.n_split > 1 && p.scratch == nullptr) return cudaErrorInvalidValue;
  if (p.B > 65535 || p.Hk > 65535) return cudaErrorInvalidValue;
  const dim3 grid(a.n_split, p.Hk, p.B);
  cudaError_t e;
  switch (G) {
    case 1: e = launch_g<1>(tk, tv, a, grid, stream); break;
    case 2: e = launch_g<2>(tk, tv, a, grid, stream); break;
    case 4: e = launch_g<4>(tk, tv, a, grid, stream); break;
    case 6: e = launch_g<6>(tk, tv, a, grid, stream); break;
    case 8: e = launch_g<8>(tk, tv, a, grid, stream); break;
    case 16: e = launch_g<16>(tk, tv, a, grid, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || a.n_split == 1) return e;
  decode_combine_kernel<<<p.B * p.Hq, DHD, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace ft
