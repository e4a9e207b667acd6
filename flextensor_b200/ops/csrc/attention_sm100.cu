// Flash attention forward on 5th-generation tensor cores (sm_100a), head_dim 128, bf16.
//
// One CTA per (batch, query head, 128-query tile); 192 threads:
//   warp 0     TMA: Q once (2 x [128 x 64] swizzled boxes), then K_j and V_j
//              tiles of 128 keys into a 2-stage ring (3-D tensor maps, so keys
//              past the sequence end are zero-filled, never read from the next batch).
//   warp 1     TMEM owner + MMA issuer:  S = Q K_j^T  (M=128, N=128, K=128) into
//              TMEM, then O += P_j V_j with P from shared memory (K-major) and
//              V as an MN-major operand (no transpose pass).
//   warps 2-5  softmax + epilogue, one query row per thread (TMEM lane = row):
//              row max / exp2 / row sum entirely in registers, O rescaled in
//              TMEM only when the running max grows by more than 2^8
//              (stale-max trick: exp2 stays <= 256 and the final 1/l fixes it),
//              P written back as bf16 in the 128-byte-swizzled layout the MMA reads.
// Every mbarrier wait is bounded; a timeout sets the device error word and the
// CTA unwinds (waits for its own MMAs, frees TMEM) instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ft_attn.h"
#include "ft_ops.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(attn_device_error)

namespace {

constexpr int AT_M = 128;   // queries per CTA
constexpr int AT_N = 128;   // keys per block
constexpr int AT_D = 128;   // head dim
constexpr int CHUNK = 128 * 64 * 2;  // one [128 rows x 64] bf16 swizzled box = 16 KB
constexpr int STAGES = 2;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

struct AttnArgs {
  int B, Sq, Sk, Hq, Hk;
  __nv_bfloat16* o;
  long long o_row, o_batch;
  float scale_log2;
  int causal;
  int n_qtiles;
};

struct Smem {
  uint8_t q[2 * CHUNK];
  uint8_t k[STAGES][2 * CHUNK];
  uint8_t v[STAGES][2 * CHUNK];
  uint8_t p[2 * CHUNK];
  uint64_t q_full, k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  uint64_t s_full, p_full, o_done, drain;
  uint32_t tmem_base;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int qt = blockIdx.x % a.n_qtiles;
  const int h = (blockIdx.x / a.n_qtiles) % a.Hq;
  const int b = blockIdx.x / (a.n_qtiles * a.Hq);
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qt * AT_M;
  int n_kv = (a.Sk + AT_N - 1) / AT_N;
  if (a.causal) n_kv = min(n_kv, (q0 + AT_M + AT_N - 1) / AT_N);

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.o_done, 1);
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = sm.tmem_base;        // columns [0,128): S
  const uint32_t tO = sm.tmem_base + 128;  // columns [128,256): O

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&sm.q_full, 2 * CHUNK);
      tma_load_3d(sm.q, &tmQ, &sm.q_full, h * AT_D, q0, b);
      tma_load_3d(sm.q + CHUNK, &tmQ, &sm.q_full, h * AT_D + 64, q0, b);
      uint32_t pend = 1u << 8, pend_ph = 0;  // bit 8: q; bits 0..: stages
      bool ok = true;
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&sm.kv_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.k_full[s], 2 * CHUNK);
        tma_load_3d(sm.k[s], &tmK, &sm.k_full[s], hk * AT_D, j * AT_N, b);
        tma_load_3d(sm.k[s] + CHUNK, &tmK, &sm.k_full[s], hk * AT_D + 64, j * AT_N, b);
        mbar_arrive_expect_tx(&sm.v_full[s], 2 * CHUNK);
        tma_load_3d(sm.v[s], &tmV, &sm.v_full[s], hk * AT_D, j * AT_N, b);
        tma_load_3d(sm.v[s] + CHUNK, &tmV, &sm.v_full[s], hk * AT_D + 64, j * AT_N, b);
        pend |= 1u << s;
        pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {
        const long long t0 = clock64();
        auto left = [&] { return (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4; };
        while (!mbar_try_wait(smem_u32(&sm.q_full), 0) && left()) {
        }
        for (int s = 0; s < STAGES; s++) {
          if (!(pend >> s & 1)) continue;
          while (!mbar_try_wait(smem_u32(&sm.k_full[s]), (pend_ph >> s) & 1) && left()) {
          }
          while (!mbar_try_wait(smem_u32(&sm.v_full[s]), (pend_ph >> s) & 1) && left()) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(AT_M, AT_N);
      constexpr uint32_t idO = umma_idesc_bf16_f32(AT_M, AT_D, false, true);  // B (V) is MN-major
      bool ok = mbar_wait(&sm.q_full, 0);
      const uint32_t qa = smem_u32(sm.q);
      for (int j = 0; ok && j < n_kv; j++) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        // S_j = Q K_j^T   (S buffer is free: softmax signalled p_full for j-1 before we got here)
        if (!mbar_wait(&sm.k_full[s], ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(sm.k[s]);
#pragma unroll
        for (int kk = 0; kk < AT_D / 16; kk++) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          umma_bf16_ss(tS, umma_desc_kmajor_sw128(qa + off), umma_desc_kmajor_sw128(ka + off), idS, kk > 0);
        }
        umma_commit(&sm.s_full);
        // O += P_j V_j  once softmax published P_j
        if (!mbar_wait(&sm.p_full, j & 1) || !mbar_wait(&sm.v_full[s], ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t pa = smem_u32(sm.p);
        const uint32_t va = smem_u32(sm.v[s]);
#pragma unroll
        for (int kk = 0; kk < AT_N / 16; kk++) {
          const uint32_t poff = (kk >> 2) * CHUNK + (kk & 3) * 32;  // keys 16kk.. in P (K-major)
          const uint32_t voff = kk * 16 * 128;                       // 16 key rows of 128 B in V (MN-major)
          umma_bf16_ss(tO, umma_desc_kmajor_sw128(pa + poff), umma_desc_mnmajor_sw128(va + voff, CHUNK), idO,
                       (j | kk) != 0);
        }
        umma_commit(&sm.kv_empty[s]);
        umma_commit(&sm.o_done);
      }
      if (!ok) {
        umma_commit(&sm.drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(&sm.drain), 0) &&
               (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
        }
      }
    }
  } else {
    // softmax / epilogue warpgroup
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int qpos = q0 + r;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; j++) {
      // tcgen05.ld/st are warp-collective (.sync.aligned): every branch that guards
      // one must be warp-uniform, so wait results are combined with a vote.
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full, j & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[AT_N];
#pragma unroll
      for (int c = 0; c < AT_N / 32; c++) {
        uint32_t t[32];
        tmem_ld_32x32b_x32(tS + lane_off + c * 32, t);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e++) sv[c * 32 + e] = __uint_as_float(t[e]) * a.scale_log2;
      }
      const int kbase = j * AT_N;
      float mx = m;
#pragma unroll
      for (int e = 0; e < AT_N; e++) {
        const int kpos = kbase + e;
        const bool valid = kpos < a.Sk && (!a.causal || kpos <= qpos);
        if (!valid) sv[e] = -INFINITY;
        mx = fmaxf(mx, sv[e]);
      }
      // P_j may only overwrite the P buffer after PV_{j-1} finished; the same wait
      // makes it safe to rescale O.
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&sm.o_done, (j - 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float m_use = m;
      // Rescale decision is taken per warp: if any row's max grew past the threshold
      // (or is still -inf), every row of the warp moves to its exact new max
      // (alpha == 1 for rows whose max did not change).
      const bool need = (mx > m + RESCALE_THRESHOLD) || (m == -INFINITY);
      if (__any_sync(0xffffffffu, need)) {
        m_use = fmaxf(m, mx);
        if (j > 0) {
          const float alpha = (m == -INFINITY) ? 0.f : ex2(m - m_use);
          l *= alpha;
#pragma unroll
          for (int c = 0; c < AT_D / 32; c++) {
            uint32_t t[32];
            tmem_ld_32x32b_x32(tO + lane_off + c * 32, t);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; e++) t[e] = __float_as_uint(__uint_as_float(t[e]) * alpha);
            tmem_st_32x32b_x32(tO + lane_off + c * 32, t);
          }
          tmem_st_wait();
        }
        m = m_use;
      }
      const float msub = (m_use == -INFINITY) ? 0.f : m_use;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 2; c++) {          // key halves -> P chunks
        uint8_t* pbase = sm.p + c * CHUNK + r * 128;
#pragma unroll
        for (int u = 0; u < 8; u++) {        // 16-byte units of 8 keys
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; e++) {
            pv[e] = ex2(sv[c * 64 + u * 8 + e] - msub);
            rs += pv[e];
          }
          uint4 w;
          w.x = pack_bf16x2(pv[0], pv[1]);
          w.y = pack_bf16x2(pv[2], pv[3]);
          w.z = pack_bf16x2(pv[4], pv[5]);
          w.w = pack_bf16x2(pv[6], pv[7]);
          *reinterpret_cast<uint4*>(pbase + ((u ^ (r & 7)) << 4)) = w;
        }
      }
      l += rs;
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }
    if (ok && n_kv > 0 && __all_sync(0xffffffffu, mbar_wait(&sm.o_done, (n_kv - 1) & 1))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * AT_D;
#pragma unroll
      for (int c = 0; c < AT_D / 32; c++) {
        uint32_t t[32];
        tmem_ld_32x32b_x32(tO + lane_off + c * 32, t);
        tmem_ld_wait();
        if (qpos < a.Sq) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(t[u * 8 + 0]) * inv, __uint_as_float(t[u * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(t[u * 8 + 2]) * inv, __uint_as_float(t[u * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(t[u * 8 + 4]) * inv, __uint_as_float(t[u * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(t[u * 8 + 6]) * inv, __uint_as_float(t[u * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + u * 8) = w;
          }
        }
      }
    } else if (n_kv == 0 && qpos < a.Sq) {
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * AT_D;
      for (int d = 0; d < AT_D; d++) out[d] = __float2bfloat16(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(sm.tmem_base, 256);
  }
}

bool make_tmap_3d(CUtensorMap* map, const void* base, int H, int S, int B, long long row_stride,
                  long long batch_stride) {
  // dims (inner->outer): head*dim columns, sequence rows, batch; box 64 x 128 x 1, 128-byte swizzle
  return make_tmap_3d_bf16(map, base, (uint64_t)H * AT_D, (uint64_t)S, (uint64_t)B, (uint64_t)row_stride,
                           (uint64_t)batch_stride, 64, 128);
}

}  // namespace

cudaError_t attention_fwd(const AttnProblem& p, cudaStream_t stream) {
  if (p.B == 0 || p.Sq == 0) return cudaSuccess;
  if (p.Hq % p.Hk) return cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  if (!make_tmap_3d(&tq, p.q, p.Hq, p.Sq, p.B, p.q_row, p.q_batch)) return cudaErrorInvalidValue;
  if (!make_tmap_3d(&tk, p.k, p.Hk, p.Sk, p.B, p.k_row, p.k_batch)) return cudaErrorInvalidValue;
  if (!make_tmap_3d(&tv, p.v, p.Hk, p.Sk, p.B, p.v_row, p.v_batch)) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(p.o) & 15 || p.o_row % 8 || p.o_batch % 8) return cudaErrorMisalignedAddress;
  AttnArgs a;
  a.B = p.B;
  a.Sq = p.Sq;
  a.Sk = p.Sk;
  a.Hq = p.Hq;
  a.Hk = p.Hk;
  a.o = p.o;
  a.o_row = p.o_row;
  a.o_batch = p.o_batch;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.causal = p.causal ? 1 : 0;
  a.n_qtiles = (p.Sq + AT_M - 1) / AT_M;
  const int smem = (int)sizeof(Smem) + 1024;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const long long grid = (long long)a.n_qtiles * p.Hq * p.B;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  attn_fwd_kernel<<<(int)grid, 192, smem, stream>>>(tq, tk, tv, a);
  return cudaGetLastError();
}

}  // namespace ft
