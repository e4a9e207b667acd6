// Tensor-parallel GEMMs with the collective fused in (sm_100a, NVLink peer memory).
//
// Both kernels are the persistent warp-specialised tcgen05 GEMM of gemm_sm100.cu (TMA ring of
// A 128x64 and W BNx64 tiles, one elected MMA thread, double-buffered TMEM accumulator, four
// epilogue warps reading TMEM), with the collective built into the data path:
//
// all-gather -> GEMM (column-parallel layer, sequence-parallel input):
//   A is the full [M, K] activation; each rank owns rows [rank*R, (rank+1)*R) of it (R = M /
//   world) in its own copy of the buffer (symmetric heap) and has published an epoch flag.
//   Warp 6 of every CTA pulls peers' rows into the local copy (12 KB bulk copies peer -> smem
//   -> HBM, pieces claimed from a per-peer ticket counter, so any running CTA can finish a
//   peer's rows and nothing waits on a CTA that is not resident) and acknowledges each peer
//   when its rows are local. M tiles are walked starting at this rank's own rows; before the
//   first load of an A tile the producer waits until every rank owning rows of the tile is
//   complete locally. Epilogue: bias, or SwiGLU over interleaved (gate, up) weight rows.
//
// GEMM -> reduce-scatter (row-parallel layer): every rank computes its partial product of all
//   M rows; the epilogue stores each output row straight into the staging buffer of the rank
//   that owns the row (slot [source rank] of that rank's [world, R, N] staging area, plain
//   16-byte stores over NVLink). M tiles start with the next rank's rows so remote traffic
//   begins early and the own rows come last. After its last tile each CTA fences; the last
//   CTA stores the epoch into every owner's flag. The owner's reduce kernel (tp_reduce) waits
//   for all flags, sums the world partials (+ residual) in fp32 and acknowledges the senders.
//
// Every wait is bounded (device error word on timeout); no TMA multicast anywhere.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ft_ops.h"
#include "ft_tp.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(tp_device_error)

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int GROUP_M = 8;
constexpr int TP_PIECE = 12288;
constexpr int NTHREADS = 224;  // warp 0 TMA, 1 MMA, 2-5 epilogue, 6 gather (AG) / idle (RS)

struct TpArgs {
  int M, N, K;
  int num_m_tiles, num_n_tiles, num_tiles, m_rot;
  int epi;  // TP_EPI_NONE / TP_EPI_BIAS / TP_EPI_SWIGLU / TP_EPI_BIAS_GELU
  const __nv_bfloat16* bias;
  __nv_bfloat16* C;
  int ldc;
  int rank, world, rows;
  // all-gather side
  const uint8_t* peer_a[kTpMaxRanks];
  uint8_t* local_a;
  long long row_bytes;
  const uint64_t* flags;
  int flag_stride;
  uint64_t* peer_acks[kTpMaxRanks];
  uint64_t epoch;
  unsigned int* claim;
  unsigned int* done;
  unsigned int* done_blk;  // [world][nblk]: bytes of each BM-row block of each peer's rows landed
  int nblk;                // BM-row blocks per rank
  int pieces;  // per rank
  // reduce-scatter side
  __nv_bfloat16* stage[kTpMaxRanks];  // rank p's staging base for this slot: [world][rows][N]
  uint64_t* peer_flags[kTpMaxRanks];  // where rank p learns our partial rows are complete
  unsigned int* cta_done;
};

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int SMEM = 1024 + RING + 2 * TP_PIECE + 512;
};

__device__ __forceinline__ void tile_coords(int tile, const TpArgs& p, int& mt, int& nt) {
  const int per_group = GROUP_M * p.num_n_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int first = g * GROUP_M;
  const int gsz = min(GROUP_M, p.num_m_tiles - first);
  mt = (first + r % gsz + p.m_rot) % p.num_m_tiles;
  nt = r / gsz;
}

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

// One lane of warp 6: pull peers' A rows into the local copy (see the file comment). Two pieces
// are in flight: piece i's peer load is issued before piece i-1's load is waited on and stored,
// so the NVLink read of one piece overlaps the local write of the previous one.
__device__ void gather_rows(const TpArgs& c, uint8_t* stage, uint64_t* stage_full) {
  const unsigned int npieces = (unsigned int)c.pieces;
  const long long rank_bytes = c.row_bytes * c.rows;
  uint32_t ph[2] = {0, 0};
  bool loading[2] = {false, false};
  bool ok = true;
  // pieces in the pipeline: [0] = the one being loaded, [1] = loaded and being stored
  struct Piece {
    int p;
    long long at;  // byte offset in the full buffer
    uint32_t n;
    int st;
  };
  const long long blk_bytes = (long long)BM * c.row_bytes;
  // a landed piece: its bytes count toward the (one or two) BM-row blocks it covers, so a tile
  // can start as soon as its own rows are in; the last piece of a peer acknowledges the peer
  auto finish = [&](const Piece& q) {
    fence_proxy_async_global();
    const long long off = q.at - (long long)q.p * rank_bytes;
    const int b0 = (int)(off / blk_bytes), b1 = (int)((off + q.n - 1) / blk_bytes);
    for (int b = b0; b <= b1; b++) {
      const long long lo = max(off, (long long)b * blk_bytes), hi = min(off + (long long)q.n, (long long)(b + 1) * blk_bytes);
      atom_add_release_gpu_u32(c.done_blk + q.p * c.nblk + b, (unsigned int)(hi - lo));
    }
    const unsigned int old = atom_add_release_gpu_u32(c.done + q.p, 1u);
    if (old + 1 == npieces) {
      __threadfence_system();
      st_release_sys_u64(c.peer_acks[q.p], c.epoch);
    }
  };
  Piece prev{-1, 0, 0, 0};
  Piece stored{-1, 0, 0, 0};  // the piece whose store was committed last (finished one step later)
  int issued = 0;
  int d = 1;
  bool flagged = false;
  while (ok) {
    // claim the next piece, moving to the next peer when this one is exhausted
    Piece cur{-1, 0, 0, 0};
    while (d < c.world) {
      const int p = (c.rank + d) % c.world;
      const unsigned int idx = atomicAdd(c.claim + p, 1u);
      if (idx >= npieces) {
        d++;
        flagged = false;
        continue;
      }
      if (!flagged) {
        if (!wait_u64(c.flags + (size_t)p * c.flag_stride, c.epoch)) {
          ok = false;
          break;
        }
        flagged = true;
      }
      const long long off = (long long)idx * TP_PIECE;
      cur = Piece{p, (long long)p * rank_bytes + off, (uint32_t)min((long long)TP_PIECE, rank_bytes - off),
                  issued & 1};
      break;
    }
    if (!ok) break;
    if (cur.p >= 0) {
      bulk_wait_read<0>();  // the store that last read this buffer (two pieces ago) is done with it
      uint8_t* buf = stage + cur.st * TP_PIECE;
      mbar_arrive_expect_tx(&stage_full[cur.st], cur.n);
      bulk_load_g2s(buf, c.peer_a[cur.p] + cur.at, cur.n, &stage_full[cur.st]);
      loading[cur.st] = true;
      issued++;
    }
    if (prev.p >= 0) {
      if (!mbar_wait(&stage_full[prev.st], ph[prev.st])) {
        ok = false;
        break;
      }
      loading[prev.st] = false;
      ph[prev.st] ^= 1;
      bulk_store_s2g(c.local_a + prev.at, stage + prev.st * TP_PIECE, prev.n);
      bulk_commit();
      bulk_wait<1>();  // the store committed one step earlier has landed
      if (stored.p >= 0) finish(stored);
      stored = prev;
    }
    if (cur.p < 0) break;
    prev = cur;
  }
  if (!ok) {  // never leave with a load in flight
    for (int st = 0; st < 2; st++) {
      if (!loading[st]) continue;
      const long long t0 = clock64();
      while (!mbar_try_wait(smem_u32(&stage_full[st]), ph[st]) &&
             (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
      }
    }
  }
  bulk_wait<0>();
  if (ok && stored.p >= 0) finish(stored);
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// 32 accumulator columns of one row -> bias / SwiGLU -> bf16 store to dst (a row pointer
// already offset to the tile's first output column).
__device__ __forceinline__ void epi_row32(const TpArgs& p, float (&v)[32], int col0, __nv_bfloat16* dst,
                                          int n_out) {
  if ((p.epi == TP_EPI_BIAS || p.epi == TP_EPI_BIAS_GELU) && p.bias != nullptr) {
#pragma unroll
    for (int e = 0; e < 32; e++) v[e] += (col0 + e < p.N) ? __bfloat162float(p.bias[col0 + e]) : 0.f;
  }
  if (p.epi == TP_EPI_BIAS_GELU) {
#pragma unroll
    for (int e = 0; e < 32; e++) v[e] = gelu_tanh(v[e]);
  }
  if (p.epi == TP_EPI_SWIGLU) {  // columns (2j, 2j+1) = (gate_j, up_j) -> 16 outputs
    const int o0 = col0 / 2;
    if (o0 + 16 <= n_out) {
#pragma unroll
      for (int j = 0; j < 2; j++) {
        uint4 u;
        u.x = pack_bf16x2(silu(v[j * 16 + 0]) * v[j * 16 + 1], silu(v[j * 16 + 2]) * v[j * 16 + 3]);
        u.y = pack_bf16x2(silu(v[j * 16 + 4]) * v[j * 16 + 5], silu(v[j * 16 + 6]) * v[j * 16 + 7]);
        u.z = pack_bf16x2(silu(v[j * 16 + 8]) * v[j * 16 + 9], silu(v[j * 16 + 10]) * v[j * 16 + 11]);
        u.w = pack_bf16x2(silu(v[j * 16 + 12]) * v[j * 16 + 13], silu(v[j * 16 + 14]) * v[j * 16 + 15]);
        *reinterpret_cast<uint4*>(dst + j * 8) = u;
      }
    } else {
      for (int j = 0; j < 16; j++)
        if (o0 + j < n_out) dst[j] = __float2bfloat16(silu(v[2 * j]) * v[2 * j + 1]);
    }
    return;
  }
  if (col0 + 32 <= n_out) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      uint4 u;
      u.x = pack_bf16x2(v[j * 8 + 0], v[j * 8 + 1]);
      u.y = pack_bf16x2(v[j * 8 + 2], v[j * 8 + 3]);
      u.z = pack_bf16x2(v[j * 8 + 4], v[j * 8 + 5]);
      u.w = pack_bf16x2(v[j * 8 + 6], v[j * 8 + 7]);
      *reinterpret_cast<uint4*>(dst + j * 8) = u;
    }
  } else {
    for (int e = 0; e < 32; e++)
      if (col0 + e < n_out) dst[e] = __float2bfloat16(v[e]);
  }
}

template <int BN, bool AG>
__global__ void __launch_bounds__(NTHREADS, 1)
    tp_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ TpArgs p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* stage = smem + C::RING;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage + 2 * TP_PIECE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* stage_full = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stage_full + 2);

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
      mbar_init(&stage_full[b], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 6) {
    if constexpr (AG) {
      if (lane == 0) gather_rows(p, stage, stage_full);
    }
  } else if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t pend = 0, pend_ph = 0;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(tile, p, mt, nt);
        if constexpr (AG) {
          // wait for the BM-row blocks of each owner that this tile's rows fall in
          const int r0 = mt * BM, r1 = min(mt * BM + BM, p.M);  // rows [r0, r1)
          for (int q = r0 / p.rows; q <= (r1 - 1) / p.rows && ok; q++) {
            if (q == p.rank) continue;
            const long long qb = (long long)q * p.rows;
            const int lo = (int)(max((long long)r0, qb) - qb), hi = (int)(min((long long)r1, qb + p.rows) - qb);
            for (int b = lo / BM; b <= (hi - 1) / BM && ok; b++) {
              const long long bytes = (long long)(min((b + 1) * BM, p.rows) - b * BM) * p.row_bytes;
              ok = wait_done(p.done_blk + q * p.nblk + b, (unsigned int)bytes);
            }
          }
          if (!ok) break;
        }
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::A_BYTES + C::B_BYTES);
          tma_load_2d(sA + s * C::A_BYTES, &tmA, &full[s], kb * BK, mt * BM);
          tma_load_2d(sB + s * C::B_BYTES, &tmB, &full[s], kb * BK, nt * BN);
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
          const uint32_t a0 = smem_u32(sA + s * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++)
            umma_bf16_ss(d, umma_desc_kmajor_sw128(a0 + k * 32), umma_desc_kmajor_sw128(b0 + k * 32), idesc,
                         (kb | k) != 0);
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
        umma_commit(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(drain), 0) &&
               (unsigned long long)(clock64() - t0) < FT_WAIT_LIMIT_CYCLES / 4) {
        }
      }
    }
  } else {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_ph = 0;
    const int n_out = p.epi == TP_EPI_SWIGLU ? p.N / 2 : p.N;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int mt, nt;
      tile_coords(tile, p, mt, nt);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph))) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      if constexpr (!AG) {
        // Reduce-scatter: the partial rows go to their owners over NVLink. A thread holds one
        // row, so direct stores would scatter 16-byte writes over 32 rows per instruction;
        // instead each warp turns 64 columns of its 32 rows around in shared memory (the idle
        // gather staging, 4 KB per warp, 16-byte segments XOR-swizzled by row) and stores
        // 128 contiguous bytes per row, 4 rows per instruction.
        uint8_t* ws = stage + q * 4096;
#pragma unroll 1
        for (int c2 = 0; c2 < BN / 64; c2++) {
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + (c2 * 2 + hh) * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int v = 0; v < 4; v++) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
              w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
              w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
              w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
              const int seg = hh * 4 + v;
              *reinterpret_cast<uint4*>(ws + lane * 128 + ((seg ^ (lane & 7)) * 16)) = w;
            }
          }
          __syncwarp();
          const int col0 = nt * BN + c2 * 64;
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const int rr = k * 4 + (lane >> 3), seg = lane & 7;
            const int grow = mt * BM + q * 32 + rr;
            const int col = col0 + seg * 8;
            if (grow < p.M && col < p.N) {
              const uint4 w = *reinterpret_cast<const uint4*>(ws + rr * 128 + ((seg ^ (rr & 7)) * 16));
              const int owner = grow / p.rows;
              *reinterpret_cast<uint4*>(p.stage[owner] + ((size_t)p.rank * p.rows + (grow - owner * p.rows)) * p.N +
                                        col) = w;
            }
          }
          __syncwarp();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
        continue;
      }
      __nv_bfloat16* rowp = row < p.M ? p.C + (size_t)row * p.ldc : nullptr;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + c * 32, r);
        tmem_ld_wait();
        const int col0 = nt * BN + c * 32;
        if (rowp != nullptr && col0 < p.N) {
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; e++) v[e] = __uint_as_float(r[e]);
          epi_row32(p, v, col0, rowp + (p.epi == TP_EPI_SWIGLU ? col0 / 2 : col0), n_out);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
    if constexpr (!AG) __threadfence_system();  // this thread's peer stores before the completion flag
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if constexpr (!AG) {
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned int old = atomicAdd(p.cta_done, 1u);
      if (old == gridDim.x - 1) {  // last CTA: every partial row of every CTA is stored
        __threadfence_system();
        for (int r = 0; r < p.world; r++) st_release_sys_u64(p.peer_flags[r], p.epoch);
      }
    }
  }
}

// Owner side of the reduce-scatter: out[r] = (residual[r] +) sum_src stage[src][r], fp32 sum.
struct OutList {
  __nv_bfloat16* ptr[kTpMaxRanks];  // every rank's output buffer (all-reduce broadcast), or ptr[0] only
  int n;
};

struct ReduceEpi {
  const __nv_bfloat16* bias;  // [N] or null
  const float* gate;          // rows of gate_stride, one per gate_rows global rows, or null
  long long gate_stride;
  int gate_rows;
  long long grow0;            // global row of local row 0
};

__global__ void __launch_bounds__(256)
    tp_reduce_kernel(const __nv_bfloat16* stage, int world, int rows, int stage_rows, int N,
                     const __nv_bfloat16* residual, int ldr, OutList outs, long long row_base, int ldo,
                     const uint64_t* flags, int flag_stride, uint64_t epoch, ReduceEpi ep) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int q = 0; q < world && ok; q++)
      if (!wait_u64(flags + (size_t)q * flag_stride, epoch)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;
  const int vec = N / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)rows * vec;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / vec), c = (int)(i % vec) * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; e++) acc[e] = 0.f;
    for (int s = 0; s < world; s++) {
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(stage + ((size_t)s * stage_rows + r) * N + c));
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] += __bfloat162float(b[e]);
    }
    if (ep.bias != nullptr) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(ep.bias + c));
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] += __bfloat162float(b[e]);
    }
    if (ep.gate != nullptr) {
      const float* g = ep.gate + ((ep.grow0 + r) / ep.gate_rows) * ep.gate_stride + c;
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] *= __ldg(g + e);
    }
    if (residual != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(residual + (size_t)r * ldr + c);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] += __bfloat162float(b[e]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    for (int q = 0; q < outs.n; q++)  // local output, or this owner's rows into every rank's output
      *reinterpret_cast<uint4*>(outs.ptr[q] + (size_t)(row_base + r) * ldo + c) = o;
  }
}

// Distributed RMSNorm, phase 1: the sum of squares of this rank's columns of 32 rows per CTA
// (one warp per 4 rows), stored as 8 16-byte vectors into every rank's partial slot at
// [rank][row0..row0+31]; the last CTA to finish publishes the epoch to every rank.
constexpr int RMS_ROWS = 32;

struct PartList {
  float* ptr[kTpMaxRanks];
  uint64_t* flag[kTpMaxRanks];
};

__global__ void __launch_bounds__(256)
    tp_sumsq_kernel(const __nv_bfloat16* x, int ldx, int rows, int D_local, int rank, int world, int stage_rows,
                    PartList parts, uint64_t epoch, unsigned int* counter) {
  __shared__ __align__(16) float ss[RMS_ROWS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * RMS_ROWS;
  const int nvec = D_local / 8;
#pragma unroll 1
  for (int k = 0; k < RMS_ROWS / 8; k++) {
    const int rr = warp * (RMS_ROWS / 8) + k;
    const int row = row0 + rr;
    float a = 0.f;
    if (row < rows) {
      const __nv_bfloat16* xr = x + (size_t)row * ldx;
      for (int v = lane; v < nvec; v += 32) {
        const uint4 u = *reinterpret_cast<const uint4*>(xr + v * 8);
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float f = __bfloat162float(b[e]);
          a = fmaf(f, f, a);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) ss[rr] = a;
  }
  __syncthreads();
  if (threadIdx.x < world * (RMS_ROWS / 4)) {
    const int q = threadIdx.x / (RMS_ROWS / 4), j = threadIdx.x % (RMS_ROWS / 4);
    const float4 v = reinterpret_cast<const float4*>(ss)[j];
    *reinterpret_cast<float4*>(parts.ptr[q] + (size_t)rank * stage_rows + row0 + j * 4) = v;
  }
  __threadfence_system();  // this thread's peer stores before the CTA's completion count
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int old = atomicAdd(counter, 1u);
    if (old == gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < world; q++) st_release_sys_u64(parts.flag[q], epoch);
    }
  }
}

// Phase 2: once every rank's partials are in (bounded wait), one warp per row: the row's scale
// from the world partials, then y = x * scale * w (+ RoPE on interleaved pairs of each head).
__global__ void __launch_bounds__(256)
    tp_rms_apply_kernel(const __nv_bfloat16* x, int ldx, __nv_bfloat16* y, int ldy, int rows, int D_local,
                        float inv_d, float eps, const void* weight, bool weight_bf16, const float* cosb,
                        const float* sinb, int head_dim, int seq_len, const float* part, int world, int stage_rows,
                        const uint64_t* flags, int flag_stride, uint64_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int q = 0; q < world && ok; q++)
      if (!wait_u64(flags + (size_t)q * flag_stride, epoch)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = D_local / 8;
  const int half = head_dim / 2;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    float a = lane < world ? __ldcg(part + (size_t)lane * stage_rows + row) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    const float sc = rsqrtf(a * inv_d + eps);
    const __nv_bfloat16* xr = x + (size_t)row * ldx;
    __nv_bfloat16* yr = y + (size_t)row * ldy;
    const int pos = seq_len > 0 ? row % seq_len : 0;
    for (int v = lane; v < nvec; v += 32) {
      const int c0 = v * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c0);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] = __bfloat162float(b[e]) * sc;
      if (weight != nullptr) {
        if (weight_bf16) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(weight) + c0));
          const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
          for (int e = 0; e < 8; e++) o[e] *= __bfloat162float(wb[e]);
        } else {
          const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(weight) + c0);
          const float4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
          o[0] *= w0.x, o[1] *= w0.y, o[2] *= w0.z, o[3] *= w0.w;
          o[4] *= w1.x, o[5] *= w1.y, o[6] *= w1.z, o[7] *= w1.w;
        }
      }
      if (cosb != nullptr) {
        const size_t t = (size_t)pos * half + (c0 % head_dim) / 2;
        const float4 cs = __ldg(reinterpret_cast<const float4*>(cosb + t));
        const float4 sn = __ldg(reinterpret_cast<const float4*>(sinb + t));
        const float cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float re = o[2 * q], im = o[2 * q + 1];
          o[2 * q] = re * cv[q] - im * sv[q];
          o[2 * q + 1] = re * sv[q] + im * cv[q];
        }
      }
      uint4 w;
      w.x = pack_bf16x2(o[0], o[1]);
      w.y = pack_bf16x2(o[2], o[3]);
      w.z = pack_bf16x2(o[4], o[5]);
      w.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(yr + c0) = w;
    }
  }
}

struct AckList {
  uint64_t* ptr[kTpMaxRanks];
  int n;
  uint64_t epoch;
};

// Runs after tp_reduce_kernel in stream order: every staged row has been read, so each sender
// may reuse its slot in this rank's staging area.
__global__ void tp_ack_kernel(AckList a) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int i = 0; i < a.n; i++)
      if (a.ptr[i] != nullptr) st_release_sys_u64(a.ptr[i], a.epoch);
  }
}

// ---------------------------------------------------------------------------------------------
// Experimental CTA-pair variant (TpGemmProblem::pair; tested on emulated ranks): 256 x 256 tiles over
// a cluster of 2 CTAs with tcgen05.mma.cta_group::2. Each CTA loads its own 128 rows of A (and,
// all-gather, waits for exactly those rows to land) and its own 128 rows of W; both loads count on
// the leader's barrier (no multicast: every CTA fetches its half itself). The leader's MMA thread
// issues M=256 x N=256 MMAs over both CTAs' shared memory, each CTA's TMEM receives its 128 rows x
// 256 columns, and each CTA's epilogue stores them (all-gather GEMM: output rows; reduce-scatter:
// 128-byte row segments into the owners' staging, as in the 1-SM kernel). Per k-block and CTA this
// reads 32 KB of shared memory for twice the math of the 1-SM 128 x 256 tile.
struct PairCfg {
  static constexpr int BN = 256;
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = BM * BK * 2;          // this CTA's 128 A rows
  static constexpr int B_BYTES = (BN / 2) * BK * 2;    // this CTA's 128 W rows
  static constexpr int TMEM_COLS = 2 * BN;              // two accumulators
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int SMEM = 1024 + RING + 2 * TP_PIECE + 512;
};
constexpr int GROUP_M2 = 4;  // 256-row tiles per weight-tile group

__device__ __forceinline__ void pair_coords(int tile, const TpArgs& p, int& mt2, int& nt) {
  const int num_m2 = (p.num_m_tiles + 1) / 2;
  const int per_group = GROUP_M2 * p.num_n_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int first = g * GROUP_M2;
  const int gsz = min(GROUP_M2, num_m2 - first);
  mt2 = (first + r % gsz + p.m_rot) % num_m2;
  nt = r / gsz;
}

template <bool AG>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    tp_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ TpArgs p) {
  using C = PairCfg;
  constexpr int STAGES = C::STAGES;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* stage = smem + C::RING;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage + 2 * TP_PIECE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* stage_full = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stage_full + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
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
      mbar_init(&tempty[b], 8);  // 4 epilogue warps x 2 CTAs arrive on the leader's copy
      mbar_init(&stage_full[b], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive / load completion
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 6) {
    if constexpr (AG) {
      if (lane == 0) gather_rows(p, stage, stage_full);
    }
  } else if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t pend = 0, pend_ph = 0;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        int mt2, nt;
        pair_coords(tile, p, mt2, nt);
        const int arow = mt2 * 256 + (int)crank * BM;
        const int brow = nt * BN + (int)crank * (BN / 2);
        if constexpr (AG) {
          // this CTA's rows [arow, arow + 128) (none past M): wait for their blocks to land
          const int r0 = arow, r1 = min(arow + BM, p.M);
          for (int q = r0 / p.rows; r0 < r1 && q <= (r1 - 1) / p.rows && ok; q++) {
            if (q == p.rank) continue;
            const long long qb = (long long)q * p.rows;
            const int lo = (int)(max((long long)r0, qb) - qb), hi = (int)(min((long long)r1, qb + p.rows) - qb);
            for (int b = lo / BM; b <= (hi - 1) / BM && ok; b++) {
              const long long bytes = (long long)(min((b + 1) * BM, p.rows) - b * BM) * p.row_bytes;
              ok = wait_done(p.done_blk + q * p.nblk + b, (unsigned int)bytes);
            }
          }
          if (!ok) break;
        }
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * (C::A_BYTES + C::B_BYTES));
          tma_load_2d_pair(sA + s * C::A_BYTES, &tmA, &full[s], kb * BK, arow);
          tma_load_2d_pair(sB + s * C::B_BYTES, &tmB, &full[s], kb * BK, brow);
          pend |= 1u << s;
          pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok && leader) {  // every issued load lands before the CTA leaves
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
          const uint64_t da = umma_desc_kmajor_sw128(smem_u32(sA + s * C::A_BYTES));
          const uint64_t db = umma_desc_kmajor_sw128(smem_u32(sB + s * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; k++) umma_bf16_ss_pair(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
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
    const int n_out = p.epi == TP_EPI_SWIGLU ? p.N / 2 : p.N;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      int mt2, nt;
      pair_coords(tile, p, mt2, nt);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph))) break;
      tc_fence_after();
      const int row0 = mt2 * 256 + (int)crank * BM + q * 32;  // this warp's first row
      if constexpr (!AG) {
        uint8_t* ws = stage + q * 4096;
#pragma unroll 1
        for (int c2 = 0; c2 < BN / 64; c2++) {
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + (c2 * 2 + hh) * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int v = 0; v < 4; v++) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
              w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
              w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
              w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
              const int seg = hh * 4 + v;
              *reinterpret_cast<uint4*>(ws + lane * 128 + ((seg ^ (lane & 7)) * 16)) = w;
            }
          }
          __syncwarp();
          const int col0 = nt * BN + c2 * 64;
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const int rr = k * 4 + (lane >> 3), seg = lane & 7;
            const int grow = row0 + rr;
            const int col = col0 + seg * 8;
            if (grow < p.M && col < p.N) {
              const uint4 w = *reinterpret_cast<const uint4*>(ws + rr * 128 + ((seg ^ (rr & 7)) * 16));
              const int owner = grow / p.rows;
              *reinterpret_cast<uint4*>(p.stage[owner] + ((size_t)p.rank * p.rows + (grow - owner * p.rows)) * p.N +
                                        col) = w;
            }
          }
          __syncwarp();
        }
      } else {
        const int row = row0 + lane;
        __nv_bfloat16* rowp = row < p.M ? p.C + (size_t)row * p.ldc : nullptr;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + c * 32, r);
          tmem_ld_wait();
          const int col0 = nt * BN + c * 32;
          if (rowp != nullptr && col0 < p.N) {
            float v[32];
#pragma unroll
            for (int e = 0; e < 32; e++) v[e] = __uint_as_float(r[e]);
            epi_row32(p, v, col0, rowp + (p.epi == TP_EPI_SWIGLU ? col0 / 2 : col0), n_out);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty0 + acc * 8);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1;
    }
    if constexpr (!AG) __threadfence_system();  // this thread's peer stores before the completion count
  }

  tc_fence_before();
  cluster_sync();  // no remote arrive or MMA may target a CTA that has left
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  if constexpr (!AG) {
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned int old = atomicAdd(p.cta_done, 1u);
      if (old == gridDim.x - 1) {  // last CTA: every partial row of every CTA is stored
        __threadfence_system();
        for (int r = 0; r < p.world; r++) st_release_sys_u64(p.peer_flags[r], p.epoch);
      }
    }
  }
}

template <bool AG>
cudaError_t launch_pair(const TpArgs& a, const CUtensorMap& tA, const CUtensorMap& tB, int num_sms, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(tp_gemm_pair_kernel<AG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PairCfg::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = ((a.num_m_tiles + 1) / 2) * a.num_n_tiles;
  const int clusters = tiles < num_sms / 2 ? tiles : num_sms / 2;
  tp_gemm_pair_kernel<AG><<<2 * clusters, NTHREADS, PairCfg::SMEM, s>>>(tA, tB, a);
  return cudaGetLastError();
}

template <int BN, bool AG>
cudaError_t launch(const TpArgs& a, const CUtensorMap& tA, const CUtensorMap& tB, int num_sms, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(tp_gemm_kernel<BN, AG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg<BN>::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int grid = a.num_tiles < num_sms ? a.num_tiles : num_sms;
  tp_gemm_kernel<BN, AG><<<grid, NTHREADS, Cfg<BN>::SMEM, s>>>(tA, tB, a);
  return cudaGetLastError();
}

}  // namespace

static cudaError_t fill_common(const TpGemmProblem& g, TpArgs& a, int bn, bool even_rows) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaErrorInvalidValue;
  if (g.K % 8 || g.N % 32 || g.world < 1 || g.world > kTpMaxRanks || g.rank < 0 || g.rank >= g.world)
    return cudaErrorInvalidValue;
  // all-gather: every rank owns exactly M / world rows; reduce-scatter: rank p owns rows
  // [p*R, min((p+1)*R, M)) with R = ceil(M / world) (the last owners may hold fewer)
  if (even_rows && g.M % g.world) return cudaErrorInvalidValue;
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.num_m_tiles = (g.M + BM - 1) / BM;
  a.num_n_tiles = (g.N + bn - 1) / bn;
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  a.epi = g.epi;
  a.bias = g.bias;
  a.rank = g.rank;
  a.world = g.world;
  a.rows = (g.M + g.world - 1) / g.world;
  a.epoch = g.epoch;
  a.flags = g.flags;
  a.flag_stride = g.flag_stride;
  for (int r = 0; r < g.world; r++) a.peer_acks[r] = g.peer_acks[r];
  return cudaSuccess;
}

cudaError_t tp_allgather_gemm(const TpGemmProblem& g, cudaStream_t stream) {
  TpArgs a{};
  const int bn = g.pair || g.N >= 256 ? 256 : 128;
  cudaError_t e = fill_common(g, a, bn, true);
  if (e != cudaSuccess) return e;
  if (g.counters == nullptr || g.C == nullptr || g.flags == nullptr) return cudaErrorInvalidValue;
  if (g.epi == TP_EPI_SWIGLU && g.N % 64) return cudaErrorInvalidValue;
  const uint8_t* local = static_cast<const uint8_t*>(g.peer_a[g.rank]);
  a.row_bytes = (long long)g.K * 2;
  for (int r = 0; r < g.world; r++) {
    if (g.peer_a[r] == nullptr || (r != g.rank && g.peer_acks[r] == nullptr)) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(g.peer_a[r]) & 15) return cudaErrorMisalignedAddress;
    a.peer_a[r] = static_cast<const uint8_t*>(g.peer_a[r]);
  }
  if ((a.row_bytes * a.rows) % 16) return cudaErrorInvalidValue;
  a.local_a = const_cast<uint8_t*>(local);
  a.C = g.C;
  a.ldc = g.ldc;
  a.claim = g.counters;
  a.done = g.counters + g.world;
  a.done_blk = g.counters + 2 * g.world;
  a.nblk = (a.rows + BM - 1) / BM;
  if (a.row_bytes * BM > 0xffffffffll) return cudaErrorInvalidValue;  // block byte counts are u32
  a.pieces = (int)((a.row_bytes * a.rows + TP_PIECE - 1) / TP_PIECE);
  a.m_rot = g.pair ? (g.rank * a.rows) / 256 : (g.rank * a.rows) / BM;
  e = cudaMemsetAsync(g.counters, 0, sizeof(unsigned int) * (size_t)tp_ag_counter_words(g.M, g.world), stream);
  if (e != cudaSuccess) return e;
  CUtensorMap tA, tB;
  if (!make_tmap_2d_bf16(&tA, local, g.K, g.M, g.K, BK, BM)) return cudaErrorInvalidValue;
  if (!make_tmap_2d_bf16(&tB, g.W, g.K, g.N, g.ldw, BK, g.pair ? bn / 2 : bn)) return cudaErrorInvalidValue;
  const int sms = g.num_sms > 0 ? g.num_sms : 148;
  if (g.pair) return launch_pair<true>(a, tA, tB, sms, stream);
  return bn == 256 ? launch<256, true>(a, tA, tB, sms, stream) : launch<128, true>(a, tA, tB, sms, stream);
}

cudaError_t tp_gemm_reducescatter(const TpGemmProblem& g, cudaStream_t stream) {
  TpArgs a{};
  const int bn = g.pair || g.N >= 256 ? 256 : 128;
  cudaError_t e = fill_common(g, a, bn, false);
  if (e != cudaSuccess) return e;
  if (g.counters == nullptr || g.epi != TP_EPI_NONE) return cudaErrorInvalidValue;  // partial sums: no epilogue op
  for (int r = 0; r < g.world; r++) {
    if (g.stage[r] == nullptr || g.peer_flags[r] == nullptr) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(g.stage[r]) & 15) return cudaErrorMisalignedAddress;
    a.stage[r] = static_cast<__nv_bfloat16*>(g.stage[r]);
    a.peer_flags[r] = g.peer_flags[r];
  }
  a.cta_done = g.counters;
  a.m_rot = (((g.rank + 1) % g.world) * a.rows) / (g.pair ? 256 : BM);
  e = cudaMemsetAsync(g.counters, 0, sizeof(unsigned int), stream);
  if (e != cudaSuccess) return e;
  CUtensorMap tA, tB;
  if (!make_tmap_2d_bf16(&tA, g.A, g.K, g.M, g.lda, BK, BM)) return cudaErrorInvalidValue;
  if (!make_tmap_2d_bf16(&tB, g.W, g.K, g.N, g.ldw, BK, g.pair ? bn / 2 : bn)) return cudaErrorInvalidValue;
  const int sms = g.num_sms > 0 ? g.num_sms : 148;
  if (g.pair) return launch_pair<false>(a, tA, tB, sms, stream);
  return bn == 256 ? launch<256, false>(a, tA, tB, sms, stream) : launch<128, false>(a, tA, tB, sms, stream);
}

cudaError_t tp_reduce(const TpReduceProblem& r, cudaStream_t stream) {
  if (r.world < 1 || r.world > kTpMaxRanks || r.N % 8 || r.rows < 0 || r.stage == nullptr || r.flags == nullptr)
    return cudaErrorInvalidValue;
  OutList outs{};
  long long row_base = 0;
  if (r.out_peers_n > 0) {  // all-reduce: broadcast this owner's reduced rows to every rank
    if (r.out_peers_n != r.world) return cudaErrorInvalidValue;
    outs.n = r.world;
    for (int q = 0; q < r.world; q++) {
      if (r.out_peers[q] == nullptr) return cudaErrorInvalidValue;
      outs.ptr[q] = static_cast<__nv_bfloat16*>(r.out_peers[q]);
    }
    row_base = r.row_base;
  } else {
    if (r.out == nullptr) return cudaErrorInvalidValue;
    outs.n = 1;
    outs.ptr[0] = static_cast<__nv_bfloat16*>(r.out);
  }
  const int stage_rows = r.stage_rows > 0 ? r.stage_rows : r.rows;
  const long long work = (long long)r.rows * (r.N / 8);
  int grid = (int)((work + 255) / 256);
  if (grid > 4 * 148) grid = 4 * 148;
  if (grid < 1) grid = 1;
  if (r.gate != nullptr && r.gate_rows <= 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(r.bias) & 15) != 0) return cudaErrorMisalignedAddress;
  ReduceEpi ep{r.bias, r.gate, r.gate_stride, r.gate_rows, r.grow0};
  tp_reduce_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(r.stage), r.world, r.rows, stage_rows,
                                             r.N, static_cast<const __nv_bfloat16*>(r.residual), r.ldr, outs,
                                             row_base, r.ldo, r.flags, r.flag_stride, r.epoch, ep);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  AckList a{};
  a.n = r.world;
  a.epoch = r.epoch;
  for (int q = 0; q < r.world; q++) a.ptr[q] = q == r.rank ? nullptr : r.peer_acks[q];
  tp_ack_kernel<<<1, 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t tp_rmsnorm(const TpRmsProblem& r, cudaStream_t stream) {
  if (r.world < 1 || r.world > kTpMaxRanks || r.rank < 0 || r.rank >= r.world || r.rows < 0) return cudaErrorInvalidValue;
  if (r.D_local <= 0 || r.D_local % 8 || r.D_full < r.D_local || r.x == nullptr || r.y == nullptr) return cudaErrorInvalidValue;
  // phase 1 stores whole 32-row groups: the slot must cover them
  if (r.ldx % 8 || r.ldy % 8 || r.stage_rows % RMS_ROWS || r.stage_rows < r.rows || r.stage_rows < RMS_ROWS)
    return cudaErrorInvalidValue;
  if (r.part_local == nullptr || r.flags == nullptr || r.counter == nullptr) return cudaErrorInvalidValue;
  auto mis = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (mis(r.x) || mis(r.y) || mis(r.weight) || mis(r.cos) || mis(r.sin)) return cudaErrorMisalignedAddress;
  if (r.cos != nullptr && (r.sin == nullptr || r.head_dim % 8 || r.D_local % r.head_dim || r.seq_len <= 0))
    return cudaErrorInvalidValue;
  PartList parts{};
  for (int q = 0; q < r.world; q++) {
    if (r.part_peers[q] == nullptr || r.peer_flags[q] == nullptr || mis(r.part_peers[q])) return cudaErrorInvalidValue;
    parts.ptr[q] = r.part_peers[q];
    parts.flag[q] = r.peer_flags[q];
  }
  cudaError_t e = cudaSuccess;
  if (r.phases & 1) {
    e = cudaMemsetAsync(r.counter, 0, sizeof(unsigned int), stream);
    if (e != cudaSuccess) return e;
    const int blocks = r.rows > 0 ? (r.rows + RMS_ROWS - 1) / RMS_ROWS : 1;
    tp_sumsq_kernel<<<blocks, 256, 0, stream>>>(r.x, r.ldx, r.rows, r.D_local, r.rank, r.world, r.stage_rows, parts,
                                                r.epoch, r.counter);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (!(r.phases & 2)) return cudaSuccess;
  int grid = (r.rows + 7) / 8;
  if (grid > 8 * 148) grid = 8 * 148;
  if (grid < 1) grid = 1;
  tp_rms_apply_kernel<<<grid, 256, 0, stream>>>(r.x, r.ldx, r.y, r.ldy, r.rows, r.D_local, 1.f / (float)r.D_full, r.eps,
                                                r.weight, r.weight_bf16, r.cos, r.sin, r.head_dim, r.seq_len,
                                                r.part_local, r.world, r.stage_rows, r.flags, r.flag_stride, r.epoch);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  AckList a{};
  a.n = r.world;
  a.epoch = r.epoch;
  for (int q = 0; q < r.world; q++) a.ptr[q] = q == r.rank ? nullptr : r.peer_acks[q];
  tp_ack_kernel<<<1, 32, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace ft
