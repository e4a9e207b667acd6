// Expert-parallel MoE expert GEMMs with the token dispatch and combine fused in (sm_100a).
//
// Each rank is a token source and owns E_l experts. A source packs the rows it routes to each
// expert contiguously in its send buffer (expert order) and publishes {cnt[E], off[E]} plus an
// epoch flag. On the expert side:
//
// moe_dispatch_gemm -- gate/up projection of the routed rows, SwiGLU in the epilogue. Every CTA
//   reads all sources' tables (NVLink loads of a few hundred bytes) and derives the same row
//   layout: one group per local expert (padded to 128 rows, so an M tile never mixes experts),
//   and inside a group one segment per source, own rows first. Warp 6 of every CTA pulls the
//   segments' rows from the sources' send buffers into the local A buffer (12 KB bulk copies
//   peer -> smem -> HBM; pieces claimed per source from a ticket counter, so any resident CTA
//   can finish a source and nothing waits on a CTA that is not running) and acknowledges the
//   source once all its rows are local. The TMA producer waits, per M tile, until every source
//   with rows in the tile is complete, then streams A and that expert's weight tiles; the
//   tcgen05 MMA / TMEM / epilogue structure is the persistent GEMM of gemm_sm100.cu.
//
// moe_combine_gemm -- down projection; the epilogue stores each output row straight into the
//   combine buffer of the source that routed it, at the row the source packed it from (plain
//   16-byte stores over NVLink), and the last CTA stores the epoch into every source's flag.
//   The source's moe_combine_reduce adds the top-k expert rows with their router weights.
//
// Every wait is bounded (device error word on timeout). No TMA multicast anywhere.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "ft_moe.h"
#include "ft_ops.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(moe_device_error)

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int PIECE = 12288;
constexpr int NTHREADS = 224;  // warp 0 TMA, 1 MMA, 2-5 epilogue, 6 gather
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int RING = STAGES * (A_BYTES + B_BYTES);
constexpr int TMEM_COLS = 2 * BN;
constexpr int W_ = kMoeMaxRanks;
constexpr int E_ = kMoeMaxLocalExperts;

struct MoeArgs {
  int rank, world, el, d, f, max_rows, N, K, num_n_tiles;
  const uint8_t* peer_send[W_];
  const int* peer_table[W_];
  const uint64_t* flags;
  int flag_stride;
  uint64_t* send_acks[W_];
  uint8_t* a_local;
  __nv_bfloat16* out;       // dispatch: h_local
  int ldo;
  __nv_bfloat16* peer_comb[W_];
  uint64_t* comb_flags[W_];
  uint64_t epoch;
  unsigned int* claim;
  unsigned int* done;
  unsigned int* cta_done;
};

struct Layout {
  int ok;
  int m_tiles;
  int group_start[E_], group_rows[E_];
  int seg_start[E_][W_], seg_cnt[E_][W_], seg_off[E_][W_];  // [j][d], source = (rank + d) % world
  int src_pieces[W_];                                        // indexed by source rank
};

struct Smem {
  uint8_t ring[RING];
  uint8_t stage[2][PIECE];
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2], drain, stage_full[2];
  uint32_t tmem;
  Layout L;
};

__device__ bool wait_u64(const uint64_t* f, uint64_t target) {
  const long long t0 = clock64();
  while (ld_acquire_sys_u64(f) < target) {
    if ((unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES) {
      record_error(kErrPeerTimeout);
      return false;
    }
    if (error_raised()) return false;
    __nanosleep(128);
  }
  return true;
}

__device__ bool wait_done(const unsigned int* d, unsigned int target) {
  const long long t0 = clock64();
  while (ld_acquire_gpu_u32(d) < target) {
    if ((unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES) {
      record_error(kErrWaitTimeout);
      return false;
    }
    if (error_raised()) return false;
    __nanosleep(64);
  }
  fence_proxy_async_global();
  return true;
}

// Thread 0: wait for every source's flag, read the tables, build the expert-side row layout.
__device__ void build_layout(Layout& L, const MoeArgs& a) {
  L.ok = 1;
  const int E = a.el * a.world;
  const long long row_bytes = (long long)a.d * 2;
  int row = 0;
  for (int p = 0; p < a.world; p++) L.src_pieces[p] = 0;
  for (int d = 0; d < a.world && L.ok; d++) {
    const int p = (a.rank + d) % a.world;
    if (!wait_u64(a.flags + (size_t)p * a.flag_stride, a.epoch)) L.ok = 0;
  }
  for (int j = 0; j < a.el && L.ok; j++) {
    const int e = a.rank * a.el + j;
    L.group_start[j] = row;
    int rows = 0;
    for (int d = 0; d < a.world; d++) {
      const int p = (a.rank + d) % a.world;
      const volatile int* t = a.peer_table[p];
      const int cnt = t[e], off = t[E + e];
      L.seg_start[j][d] = row + rows;
      L.seg_cnt[j][d] = cnt;
      L.seg_off[j][d] = off;
      rows += cnt;
      L.src_pieces[p] += (int)((cnt * row_bytes + PIECE - 1) / PIECE);
    }
    L.group_rows[j] = rows;
    row += (rows + BM - 1) / BM * BM;
  }
  if (row > a.max_rows) {  // more routed rows than the buffers hold: refuse to run
    record_error(kErrBadArgs);
    L.ok = 0;
  }
  L.m_tiles = L.ok ? row / BM : 0;
}

// Linear tile index -> (expert group j, M tile, N tile). Tiles go expert group by expert group;
// inside a group, GROUP_M M tiles share each N tile before moving on, so an expert's weight
// tile is read from HBM once per GROUP_M M tiles instead of once per M tile (an expert's
// gate/up weight is 400 MB at the Mixtral shape, far larger than L2).
constexpr int GROUP_M = 16;

__device__ __forceinline__ void tile_coords(const Layout& L, int el, int n_tiles, int tile, int& j, int& mt,
                                            int& nt) {
  j = 0;
  for (; j < el; j++) {
    const int mtj = (L.group_rows[j] + BM - 1) / BM;
    if (tile < mtj * n_tiles) break;
    tile -= mtj * n_tiles;
  }
  const int mtj = (L.group_rows[j] + BM - 1) / BM;
  const int per_group = GROUP_M * n_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int first = g * GROUP_M;
  const int gsz = min(GROUP_M, mtj - first);
  mt = L.group_start[j] / BM + first + r % gsz;
  nt = r / gsz;
}

// Gather lane: claim pieces source by source (own rows first) and move them into a_local.
__device__ void gather(Smem& sm, const MoeArgs& a) {
  const Layout& L = sm.L;
  const long long row_bytes = (long long)a.d * 2;
  uint32_t ph[2] = {0, 0};
  int issued = 0, pend_p = -1;
  bool ok = true;
  auto finish = [&](int p) {
    fence_proxy_async_global();
    const unsigned int old = atom_add_release_gpu_u32(a.done + p, 1u);
    if (old + 1 == (unsigned int)L.src_pieces[p] && p != a.rank) {
      __threadfence_system();
      st_release_sys_u64(a.send_acks[p], a.epoch);
    }
  };
  if (blockIdx.x == 0) {  // sources with nothing for us are acknowledged at once
    for (int p = 0; p < a.world; p++)
      if (p != a.rank && L.src_pieces[p] == 0) st_release_sys_u64(a.send_acks[p], a.epoch);
  }
  for (int d = 0; d < a.world && ok; d++) {
    const int p = (a.rank + d) % a.world;
    const unsigned int np = (unsigned int)L.src_pieces[p];
    for (;;) {
      unsigned int idx = atomicAdd(a.claim + p, 1u);
      if (idx >= np) break;
      int j = 0;  // which local expert's segment of source p holds piece idx
      long long seg_bytes = 0;
      for (; j < a.el; j++) {
        seg_bytes = L.seg_cnt[j][d] * row_bytes;
        const unsigned int pj = (unsigned int)((seg_bytes + PIECE - 1) / PIECE);
        if (idx < pj) break;
        idx -= pj;
      }
      const long long off = (long long)idx * PIECE;
      const uint32_t n = (uint32_t)min((long long)PIECE, seg_bytes - off);
      const uint8_t* src = a.peer_send[p] + (long long)L.seg_off[j][d] * row_bytes + off;
      uint8_t* dst = a.a_local + (long long)L.seg_start[j][d] * row_bytes + off;
      const int st = issued & 1;
      mbar_arrive_expect_tx(&sm.stage_full[st], n);
      bulk_load_g2s(sm.stage[st], src, n, &sm.stage_full[st]);
      if (!mbar_wait(&sm.stage_full[st], ph[st])) {
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(&sm.stage_full[st]), ph[st]) &&
               (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
        }
        ok = false;
        break;
      }
      ph[st] ^= 1;
      bulk_store_s2g(dst, sm.stage[st], n);
      bulk_commit();
      issued++;
      if (pend_p >= 0) {
        bulk_wait<1>();
        finish(pend_p);
      }
      pend_p = p;
    }
  }
  bulk_wait<0>();
  if (ok && pend_p >= 0) finish(pend_p);
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

struct WeightMaps {
  CUtensorMap w[E_];
};

template <bool DISPATCH>
__global__ void __launch_bounds__(NTHREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ WeightMaps wm,
                    const __grid_constant__ MoeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = sm.ring;
  uint8_t* sB = sm.ring + STAGES * A_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = (a.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&sm.tfull[b], 1);
      mbar_init(&sm.tempty[b], 4);
      mbar_init(&sm.stage_full[b], 1);
    }
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
    build_layout(sm.L, a);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sm.tmem;
  const Layout& L = sm.L;
  const int num_tiles = L.m_tiles * a.num_n_tiles;

  if (warp == 6) {
    if constexpr (DISPATCH) {
      if (lane == 0 && L.ok) gather(sm, a);
    }
  } else if (warp == 0) {
    if (elect_one() && L.ok) {
      tma_prefetch_desc(&tmA);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t pend = 0, pend_ph = 0, ready = 0;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int j, mt, nt;
        tile_coords(L, a.el, a.num_n_tiles, tile, j, mt, nt);
        if constexpr (DISPATCH) {
          const int r0 = mt * BM, r1 = r0 + BM;
          for (int dd = 0; dd < a.world && ok; dd++) {
            const int p = (a.rank + dd) % a.world;
            const int s0 = L.seg_start[j][dd], s1 = s0 + L.seg_cnt[j][dd];
            if (s1 <= r0 || s0 >= r1 || (ready >> p & 1u)) continue;
            ok = wait_done(a.done + p, (unsigned int)L.src_pieces[p]);
            ready |= 1u << p;
          }
          if (!ok) break;
        }
        const CUtensorMap* tmB = &wm.w[j];
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&sm.empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[s], A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmA, &sm.full[s], kb * BK, mt * BM);
          tma_load_2d(sB + s * B_BYTES, tmB, &sm.full[s], kb * BK, nt * BN);
          pend |= 1u << s;
          pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {
        for (int st = 0; st < STAGES; st++) {
          if (!(pend >> st & 1)) continue;
          const long long t0 = clock64();
          while (!mbar_try_wait(smem_u32(&sm.full[st]), (pend_ph >> st) & 1) &&
                 (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one() && L.ok) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(BM, BN);
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&sm.tempty[acc], acc_ph ^ 1)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + acc * BN;
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&sm.full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            umma_bf16_ss(dt, umma_desc_kmajor_sw128(a0 + k * 32), umma_desc_kmajor_sw128(b0 + k * 32), idesc,
                         (kb | k) != 0);
          umma_commit(&sm.empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&sm.tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
      if (!ok) {
        umma_commit(&sm.drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(&sm.drain), 0) &&
               (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
        }
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int tile = blockIdx.x; L.ok && tile < num_tiles; tile += gridDim.x) {
      int j, mt, nt;
      tile_coords(L, a.el, a.num_n_tiles, tile, j, mt, nt);
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.tfull[acc], acc_ph))) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      __nv_bfloat16* rowp = nullptr;
      if (row < L.group_start[j] + L.group_rows[j]) {
        if constexpr (DISPATCH) {
          rowp = a.out + (size_t)row * a.ldo;
        } else {
          for (int dd = 0; dd < a.world; dd++) {
            const int s0 = L.seg_start[j][dd];
            if (row >= s0 && row < s0 + L.seg_cnt[j][dd]) {
              const int p = (a.rank + dd) % a.world;
              rowp = a.peer_comb[p] + (size_t)(L.seg_off[j][dd] + row - s0) * a.N;
              break;
            }
          }
        }
      }
      if constexpr (DISPATCH) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + c * 32, r);
          tmem_ld_wait();
          const int col0 = nt * BN + c * 32;
          if (rowp != nullptr && col0 < a.N) {  // SwiGLU: (gate, up) column pairs -> 16 outputs
            __nv_bfloat16* dst = rowp + col0 / 2;
#pragma unroll
            for (int h = 0; h < 2; h++) {
              float o[8];
#pragma unroll
              for (int e = 0; e < 8; e++)
                o[e] = silu(__uint_as_float(r[h * 16 + 2 * e])) * __uint_as_float(r[h * 16 + 2 * e + 1]);
              uint4 u;
              u.x = pack_bf16x2(o[0], o[1]);
              u.y = pack_bf16x2(o[2], o[3]);
              u.z = pack_bf16x2(o[4], o[5]);
              u.w = pack_bf16x2(o[6], o[7]);
              *reinterpret_cast<uint4*>(dst + h * 8) = u;
            }
          }
        }
      } else {
        // Combine: the rows go to their token's rank over NVLink. As in the tensor-parallel
        // reduce-scatter, each warp turns 64 columns of its 32 rows around in shared memory (the
        // gather staging, idle in this GEMM; 4 KB per warp, 16-byte segments XOR-swizzled by row)
        // and stores 128 contiguous bytes per row, 4 rows per instruction; a row's destination
        // comes from the lane that owns it.
        uint8_t* ws = &sm.stage[0][0] + q * 4096;
        const unsigned long long mydst = reinterpret_cast<unsigned long long>(rowp);
#pragma unroll 1
        for (int c2 = 0; c2 < BN / 64; c2++) {
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + (c2 * 2 + hh) * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int v = 0; v < 4; v++) {
              uint4 u;
              u.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
              u.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
              u.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
              u.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
              const int seg = hh * 4 + v;
              *reinterpret_cast<uint4*>(ws + lane * 128 + ((seg ^ (lane & 7)) * 16)) = u;
            }
          }
          __syncwarp();
          const int col0 = nt * BN + c2 * 64;
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const int rr = k * 4 + (lane >> 3), seg = lane & 7;
            const unsigned long long d = __shfl_sync(0xffffffffu, mydst, rr);
            const int col = col0 + seg * 8;
            if (d != 0ull && col < a.N)
              *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d) + col) =
                  *reinterpret_cast<const uint4*>(ws + rr * 128 + ((seg ^ (rr & 7)) * 16));
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
    if constexpr (!DISPATCH) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (!DISPATCH) {
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned int old = atomicAdd(a.cta_done, 1u);
      if (old == gridDim.x - 1 && L.ok) {
        __threadfence_system();
        for (int p = 0; p < a.world; p++) st_release_sys_u64(a.comb_flags[p], a.epoch);
      }
    }
  }
}

__global__ void __launch_bounds__(256)
    moe_reduce_kernel(const __nv_bfloat16* comb, const int* pos, const float* wts, const __nv_bfloat16* residual,
                      __nv_bfloat16* out, int tokens, int topk, int d, const uint64_t* flags, int flag_stride,
                      int world, uint64_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int q = 0; q < world && ok; q++)
      if (!wait_u64(flags + (size_t)q * flag_stride, epoch)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;
  const int vec = d / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)tokens * vec;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / vec), c = (int)(i % vec) * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; e++) acc[e] = 0.f;
    if (residual != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(residual + (size_t)t * d + c);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] = __bfloat162float(b[e]);
    }
    for (int k = 0; k < topk; k++) {
      const int r = pos[(size_t)t * topk + k];
      const float w = wts[(size_t)t * topk + k];
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(comb + (size_t)r * d + c));
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] += w * __bfloat162float(b[e]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + (size_t)t * d + c) = o;
  }
}

cudaError_t launch(const MoeProblem& p, bool dispatch, cudaStream_t stream) {
  if (p.world < 1 || p.world > W_ || p.rank < 0 || p.rank >= p.world || p.local_experts < 1 ||
      p.local_experts > E_ || p.d % 64 || p.f % 64 || p.max_rows % BM || p.max_rows <= 0 || p.counters == nullptr ||
      p.flags == nullptr || p.a_local == nullptr || p.h_local == nullptr)
    return cudaErrorInvalidValue;
  MoeArgs a{};
  a.rank = p.rank;
  a.world = p.world;
  a.el = p.local_experts;
  a.d = p.d;
  a.f = p.f;
  a.max_rows = p.max_rows;
  a.N = dispatch ? 2 * p.f : p.d;
  a.K = dispatch ? p.d : p.f;
  a.num_n_tiles = (a.N + BN - 1) / BN;
  for (int r = 0; r < p.world; r++) {
    if (p.peer_table[r] == nullptr) return cudaErrorInvalidValue;
    a.peer_send[r] = static_cast<const uint8_t*>(p.peer_send[r]);
    a.peer_table[r] = p.peer_table[r];
    a.send_acks[r] = p.send_acks[r];
    a.peer_comb[r] = static_cast<__nv_bfloat16*>(p.peer_comb[r]);
    a.comb_flags[r] = p.comb_flags[r];
    if (dispatch && (a.peer_send[r] == nullptr || (r != p.rank && a.send_acks[r] == nullptr)))
      return cudaErrorInvalidValue;
    if (!dispatch && (a.peer_comb[r] == nullptr || a.comb_flags[r] == nullptr)) return cudaErrorInvalidValue;
  }
  a.flags = p.flags;
  a.flag_stride = p.flag_stride;
  a.a_local = static_cast<uint8_t*>(p.a_local);
  a.out = static_cast<__nv_bfloat16*>(p.h_local);
  a.ldo = p.f;
  a.epoch = p.epoch;
  a.claim = p.counters;
  a.done = p.counters + p.world;
  a.cta_done = p.counters + 2 * p.world;
  cudaError_t e = cudaMemsetAsync(p.counters, 0, sizeof(unsigned int) * (2 * p.world + 1), stream);
  if (e != cudaSuccess) return e;
  CUtensorMap tA;
  WeightMaps wm;
  memset(&wm, 0, sizeof(wm));
  if (dispatch) {
    if (!make_tmap_2d_bf16(&tA, p.a_local, p.d, p.max_rows, p.d, BK, BM)) return cudaErrorInvalidValue;
  } else {
    if (!make_tmap_2d_bf16(&tA, p.h_local, p.f, p.max_rows, p.f, BK, BM)) return cudaErrorInvalidValue;
  }
  for (int j = 0; j < p.local_experts; j++) {
    const void* w = dispatch ? p.w_gate_up[j] : p.w_down[j];
    if (w == nullptr) return cudaErrorInvalidValue;
    if (!make_tmap_2d_bf16(&wm.w[j], w, a.K, a.N, a.K, BK, BN)) return cudaErrorInvalidValue;
  }
  const int smem = (int)sizeof(Smem) + 1024;
  const int sms = p.num_sms > 0 ? p.num_sms : 148;
  const int max_tiles = (p.max_rows / BM) * a.num_n_tiles;
  const int grid = max_tiles < sms ? max_tiles : sms;
  if (dispatch) {
    static bool attr = false;
    if (!attr) {
      e = cudaFuncSetAttribute(moe_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      attr = true;
    }
    moe_gemm_kernel<true><<<grid, NTHREADS, smem, stream>>>(tA, wm, a);
  } else {
    static bool attr = false;
    if (!attr) {
      e = cudaFuncSetAttribute(moe_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      attr = true;
    }
    moe_gemm_kernel<false><<<grid, NTHREADS, smem, stream>>>(tA, wm, a);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t moe_dispatch_gemm(const MoeProblem& p, cudaStream_t stream) { return launch(p, true, stream); }
cudaError_t moe_combine_gemm(const MoeProblem& p, cudaStream_t stream) { return launch(p, false, stream); }

cudaError_t moe_combine_reduce(const MoeCombineProblem& p, cudaStream_t stream) {
  if (p.tokens <= 0) return cudaSuccess;
  if (p.d % 8 || p.topk < 1 || p.comb == nullptr || p.pos == nullptr || p.weight == nullptr || p.out == nullptr ||
      p.flags == nullptr)
    return cudaErrorInvalidValue;
  const long long work = (long long)p.tokens * (p.d / 8);
  int grid = (int)((work + 255) / 256);
  if (grid > 4 * 148) grid = 4 * 148;
  moe_reduce_kernel<<<grid, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(p.comb), p.pos, p.weight, static_cast<const __nv_bfloat16*>(p.residual),
      static_cast<__nv_bfloat16*>(p.out), p.tokens, p.topk, p.d, p.flags, p.flag_stride, p.world, p.epoch);
  return cudaGetLastError();
}

}  // namespace ft
