// Persistent, warp-specialised tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M,N] = epilogue( A[M,K] . W[N,K]^T )      (nn.Linear layout, bf16 in, fp32 accumulate)
//
// Roles per CTA (192 threads, one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0      TMA producer: A (128 x 64) and W (BN x 64) tiles, 128-byte
//               swizzle, into a STAGES-deep shared-memory ring (full/empty mbarriers).
//   warp 1      TMEM owner + MMA issuer: one elected lane issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) x4 per
//               64-wide k-block; tcgen05.commit releases the smem stage; a second
//               commit hands the finished accumulator to the epilogue.
//   warps 2..5  Epilogue: tcgen05.ld 32x32b.x32 (each warp owns its 32-lane TMEM
//               quadrant), fused bias / GELU / gate*x + residual, bf16 stores.
// The accumulator is double-buffered in TMEM (2 x BN columns), so the epilogue
// of tile i overlaps the MMAs of tile i+1. Tiles are walked in grouped order
// (8 M-tiles per group) so concurrently running CTAs share A and W tiles in L2.
//
// Every wait is bounded (sm100_common.cuh); on timeout each role stops issuing,
// the CTA drains in-flight TMA loads (bounded) and frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "sm100_common.cuh"
#include "ft_ops.h"

namespace ft {

FT_DEFINE_ERROR_READER(gemm_device_error)

struct GemmArgs {
  int M, N, K;
  __nv_bfloat16* C;
  int ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int ldr;
  const float* gate;
  int gate_rows;  // rows per gate vector (0: one gate vector for every row)
  int num_m_tiles, num_n_tiles, num_tiles;
  int epi;
};

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int GROUP_M = 8;

__device__ __forceinline__ void tile_coords(int tile, const GemmArgs& p, int& mt, int& nt) {
  const int per_group = GROUP_M * p.num_n_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int first = g * GROUP_M;
  const int gsz = min(GROUP_M, p.num_m_tiles - first);
  mt = first + r % gsz;
  nt = r / gsz;
}

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int TMEM_COLS = (2 * BN) < 32 ? 32 : 2 * BN;
  static constexpr int SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + 256;
};

__device__ __forceinline__ void epi_store32(const GemmArgs& p, int row, int col0, float (&v)[32]) {
  const int N = p.N;
  const bool full = col0 + 32 <= N;
  if (p.epi != EPI_NONE && p.bias != nullptr) {
    if (full) {
      const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint4 u = __ldg(b4 + j);
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int e = 0; e < 8; e++) v[j * 8 + e] += __bfloat162float(b[e]);
      }
    } else {
      for (int e = 0; e < 32; e++)
        if (col0 + e < N) v[e] += __bfloat162float(p.bias[col0 + e]);
    }
  }
  if (p.epi == EPI_BIAS_GELU) {
#pragma unroll
    for (int e = 0; e < 32; e++) v[e] = gelu_tanh(v[e]);
  }
  if (p.epi == EPI_BIAS_GATE_RES || p.epi == EPI_BIAS_RES) {
    const __nv_bfloat16* res = p.residual + (size_t)row * p.ldr + col0;
    const float* g = nullptr;
    if (p.epi == EPI_BIAS_GATE_RES) g = p.gate + (p.gate_rows > 0 ? (size_t)(row / p.gate_rows) * N : 0) + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint4 u = *reinterpret_cast<const uint4*>(res + j * 8);
        const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          float gv = g ? __ldg(g + j * 8 + e) : 1.f;
          v[j * 8 + e] = __bfloat162float(r[e]) + gv * v[j * 8 + e];
        }
      }
    } else {
      for (int e = 0; e < 32; e++)
        if (col0 + e < N) v[e] = __bfloat162float(res[e]) + (g ? g[e] : 1.f) * v[e];
    }
  }
  __nv_bfloat16* out = p.C + (size_t)row * p.ldc + col0;
  if (full) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      uint4 u;
      u.x = pack_bf16x2(v[j * 8 + 0], v[j * 8 + 1]);
      u.y = pack_bf16x2(v[j * 8 + 2], v[j * 8 + 3]);
      u.z = pack_bf16x2(v[j * 8 + 4], v[j * 8 + 5]);
      u.w = pack_bf16x2(v[j * 8 + 6], v[j * 8 + 7]);
      *reinterpret_cast<uint4*>(out + j * 8) = u;
    }
  } else {
    for (int e = 0; e < 32; e++)
      if (col0 + e < N) out[e] = __float2bfloat16(v[e]);
  }
}

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t pend = 0, pend_ph = 0;  // per-stage: load issued / parity it completes with
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(tile, p, mt, nt);
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::A_BYTES + Cfg::B_BYTES);
          tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, &full[s], kb * BK, mt * BM);
          tma_load_2d(sB + s * Cfg::B_BYTES, &tmB, &full[s], kb * BK, nt * BN);
          pend |= 1u << s;
          pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {
        // unwinding after a timeout: let every issued load land before the CTA exits
        for (int st = 0; st < STAGES; st++) {
          if (!(pend >> st & 1)) continue;
          const long long t0 = clock64();
          while (!mbar_try_wait(smem_u32(&full[st]), (pend_ph >> st) & 1) &&
                 (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(BM, BN);
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {
            umma_bf16_ss(d, umma_desc_kmajor_sw128(a0 + k * 32), umma_desc_kmajor_sw128(b0 + k * 32), idesc,
                         (kb | k) != 0);
          }
          umma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
      if (!ok) {
        // unwinding: every MMA issued so far must finish before TMEM is freed
        umma_commit(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(drain), 0) &&
               (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
        }
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int mt, nt;
      tile_coords(tile, p, mt, nt);
      // tcgen05.ld below is warp-collective: leave the loop as a whole warp
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph))) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + c * 32, r);
        tmem_ld_wait();
        const int col0 = nt * BN + c * 32;
        if (row < p.M && col0 < p.N) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; e++) v[e] = __uint_as_float(r[e]);
          epi_store32(p, row, col0, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ 2-SM (CTA pair) variant
// Cluster of 2 CTAs computes a 256 x 256 tile with tcgen05.mma.cta_group::2 (M=256):
// CTA r loads A rows [m0 + 128r, +128) and W rows [n0 + 128r, +128) into its own
// shared memory; both halves' TMA bytes are counted on the leader's (rank 0) full
// barrier; the leader's single MMA thread issues M=256 x N=256 x K=16 MMAs reading
// both CTAs' tiles, and each CTA's TMEM receives its 128 rows x 256 columns.
// Commits are multicast to both CTAs (stage free / accumulator ready); epilogue warps
// of both CTAs arrive on the leader's accumulator-empty barrier.
// Per CTA per k-block: 32 KB of shared-memory traffic for 2x the math of the 1-SM
// 128x256 tile, which halves L2->SM bandwidth per FLOP.
struct Gemm2Cfg {
  static constexpr int BN = 256;  // pair tile N
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = BM * BK * 2;         // this CTA's 128 A rows
  static constexpr int B_BYTES = (BN / 2) * BK * 2;   // this CTA's 128 W rows
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + 256;
};

__device__ __forceinline__ void tile_coords_pair(int tile, const GemmArgs& p, int& mt2, int& nt) {
  // mt2 indexes 256-row tiles
  const int num_m2 = (p.num_m_tiles + 1) / 2;
  const int per_group = 4 * p.num_n_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int first = g * 4;
  const int gsz = min(4, num_m2 - first);
  mt2 = first + r % gsz;
  nt = r / gsz;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_bf16_tcgen05_2sm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          GemmArgs p) {
  using Cfg = Gemm2Cfg;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int kblocks = (p.K + BK - 1) / BK;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_tiles = ((p.num_m_tiles + 1) / 2) * p.num_n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps x 2 CTAs (leader's copy is the one used)
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive / TMA completion
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t pend = 0, pend_ph = 0;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        int mt2, nt;
        tile_coords_pair(tile, p, mt2, nt);
        const int arow = mt2 * 256 + (int)rank * 128;
        const int brow = nt * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
          tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, &full[s], kb * BK, arow);
          tma_load_2d_pair(sB + s * Cfg::B_BYTES, &tmB, &full[s], kb * BK, brow);
          pend |= 1u << s;
          pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok && leader) {
        for (int st = 0; st < STAGES; st++) {
          if (!(pend >> st & 1)) continue;
          const long long t0 = clock64();
          while (!mbar_try_wait(smem_u32(&full[st]), (pend_ph >> st) & 1) &&
                 (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(256, BN);
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES);
          const uint32_t b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {
            umma_bf16_ss_pair(d, umma_desc_kmajor_sw128(a0 + k * 32), umma_desc_kmajor_sw128(b0 + k * 32), idesc,
                              (kb | k) != 0);
          }
          umma_commit_pair(&empty[s], 0x3);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
      if (!ok) {
        umma_commit_pair(drain, 0x1);
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(drain), 0) &&
               (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
        }
      }
    }
  } else {
    const int q = warp & 3;
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      int mt2, nt;
      tile_coords_pair(tile, p, mt2, nt);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph))) break;
      tc_fence_after();
      const int row = mt2 * 256 + (int)rank * 128 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + c * 32, r);
        tmem_ld_wait();
        const int col0 = nt * BN + c * 32;
        if (row < p.M && col0 < p.N) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; e++) v[e] = __uint_as_float(r[e]);
          epi_store32(p, row, col0, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty0 + acc * 8);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
  }

  tc_fence_before();
  cluster_sync();  // no remote arrive / MMA may target a CTA that has left
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

static cudaError_t launch_gemm_2sm(const GemmArgs& a, const __nv_bfloat16* A, int lda, const __nv_bfloat16* W,
                                   int ldw, int num_sms, cudaStream_t stream) {
  using Cfg = Gemm2Cfg;
  CUtensorMap tmA, tmB;
  if (!make_tmap_2d_bf16(&tmA, A, a.K, a.M, lda, BK, BM)) return cudaErrorInvalidValue;
  if (!make_tmap_2d_bf16(&tmB, W, a.K, a.N, ldw, BK, Cfg::BN / 2)) return cudaErrorInvalidValue;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tcgen05_2sm, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int tiles = ((a.num_m_tiles + 1) / 2) * a.num_n_tiles;
  int clusters = tiles < num_sms / 2 ? tiles : num_sms / 2;
  gemm_bf16_tcgen05_2sm<<<2 * clusters, 192, Cfg::SMEM, stream>>>(tmA, tmB, a);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ host side
template <int BN>
static cudaError_t launch_gemm(const GemmArgs& a, const __nv_bfloat16* A, int lda, const __nv_bfloat16* W, int ldw,
                               int num_sms, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap tmA, tmB;
  if (!make_tmap_2d_bf16(&tmA, A, a.K, a.M, lda, BK, BM)) return cudaErrorInvalidValue;
  if (!make_tmap_2d_bf16(&tmB, W, a.K, a.N, ldw, BK, BN)) return cudaErrorInvalidValue;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tcgen05<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  int grid = a.num_tiles < num_sms ? a.num_tiles : num_sms;
  gemm_bf16_tcgen05<BN><<<grid, 192, Cfg::SMEM, stream>>>(tmA, tmB, a);
  return cudaGetLastError();
}

cudaError_t gemm_bf16(const GemmProblem& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaSuccess;
  if ((g.K % 8) || (g.lda % 8) || (g.ldw % 8) || (g.ldc % 8) || (g.N % 8)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.W) | reinterpret_cast<uintptr_t>(g.C)) & 15)
    return cudaErrorMisalignedAddress;
  if ((g.epi == EPI_BIAS_GATE_RES || g.epi == EPI_BIAS_RES) && (g.residual == nullptr || (g.ldr % 8)))
    return cudaErrorInvalidValue;
  if (g.epi == EPI_BIAS_GATE_RES && g.gate == nullptr) return cudaErrorInvalidValue;
  GemmArgs a{};
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.C = g.C;
  a.ldc = g.ldc;
  a.bias = g.bias;
  a.residual = g.residual;
  a.ldr = g.ldr;
  a.gate = g.gate;
  a.gate_rows = g.gate_rows;
  a.epi = g.epi;
  if (a.bias != nullptr && (reinterpret_cast<uintptr_t>(a.bias) & 15)) return cudaErrorMisalignedAddress;
  int bn = g.N >= 256 ? 256 : (g.N > 64 ? 128 : 64);
  if (g.force_bn) bn = g.force_bn;
  const bool pair = (g.force_bn == 512) || (g.force_bn == 0 && g.M >= 512 && g.N >= 256 && g.pair_ok);
  if (pair) {
    a.num_m_tiles = (g.M + BM - 1) / BM;
    a.num_n_tiles = (g.N + 255) / 256;
    a.num_tiles = a.num_m_tiles * a.num_n_tiles;
    return launch_gemm_2sm(a, g.A, g.lda, g.W, g.ldw, g.num_sms > 0 ? g.num_sms : 148, stream);
  }
  a.num_m_tiles = (g.M + BM - 1) / BM;
  a.num_n_tiles = (g.N + bn - 1) / bn;
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  int num_sms = g.num_sms > 0 ? g.num_sms : 148;
  switch (bn) {
    case 256:
      return launch_gemm<256>(a, g.A, g.lda, g.W, g.ldw, num_sms, stream);
    case 128:
      return launch_gemm<128>(a, g.A, g.lda, g.W, g.ldw, num_sms, stream);
    default:
      return launch_gemm<64>(a, g.A, g.lda, g.W, g.ldw, num_sms, stream);
  }
}

}  // namespace ft
