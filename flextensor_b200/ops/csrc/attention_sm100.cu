// Flash attention forward on 5th-generation tensor cores (sm_100a), head_dim 128, bf16.
//
// One CTA per (batch, query head, 256 queries) = two 128-query tiles A and B
// that ping-pong on the tensor core: while one tile's softmax warpgroup turns
// S into P, the MMA warp runs the other tile's GEMMs. 320 threads:
//   warps 0-3   softmax + epilogue of tile A (warp w owns TMEM lanes 32(w%4)..+31 = its query rows)
//   warps 4-7   softmax + epilogue of tile B
//   warp 8      TMEM owner + MMA issuer (one elected lane)
//   warp 9      TMA producer: Q_A, Q_B once; K_j and V_j (128 keys) into two 2-stage rings
//               (3-D tensor maps: keys past the sequence end read as zeros, never the next batch)
// TMEM (512 columns): S_A | S_B | O_A | O_B, 128 fp32 columns each. P_X (bf16, two per
// 32-bit column) is written by tcgen05.st over the first 64 columns of S_X and consumed by
// the TS-form MMA (A operand from TMEM), so P never touches shared memory.
// MMA issue order per KV block j:  PV_A(j) S_A(j+1) PV_B(j) S_B(j+1); S_X(j+1) reuses the
// columns PV_X(j) reads as P, which tcgen05.mma's in-order execution makes safe.
// Softmax per row (one thread = one row): one TMEM round trip brings the whole S row into
// registers; row max (4 independent chains), P = exp2(s*scale*log2e - m) packed in place and the
// row sum (4 partial sums) all happen in registers; O is rescaled in TMEM only
// when some row's max grew past 2^8 (stale-max trick; the final 1/l normalisation is exact).
// Every branch around a warp-collective tcgen05.ld/st is warp-uniform (votes).
// All waits are bounded; a timeout records the device error word and the CTA unwinds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "ft_attn.h"
#include "ft_ops.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(attn_device_error)

namespace {

constexpr int TILE = 128;                 // queries per tile, keys per block
constexpr int HD = 128;                   // head dim
constexpr int CHUNK = 128 * 64 * 2;       // one [128 rows x 64 cols] bf16 swizzled box (16 KB)
constexpr int KV_STAGES = 2;
constexpr float RESCALE_THRESHOLD = 8.0f;
constexpr int NTHREADS = 320;            // plain attention: 10 warps
constexpr int NTHREADS_CP = 352;         // context-parallel: + warp 10, the K/V gather warp
constexpr int CP_PIECE = 12288;          // bytes per gather step (peer -> smem -> local HBM)

struct AttnArgs {
  int B, Sq, Sk, Hq, Hk;
  __nv_bfloat16* o;
  long long o_row, o_batch;
  float scale_log2;
  int causal;
  int n_qblocks;  // 256-query blocks per (b, h)
  int diag;
  unsigned long long* trace;  // debug: clock64 timeline of CTA 0 (null in production)
};

struct SmemBase {
  uint8_t q[2][2 * CHUNK];                // tile, d-half
  uint8_t k[KV_STAGES][2 * CHUNK];
  uint8_t v[KV_STAGES][2 * CHUNK];
  uint64_t q_full;
  uint64_t k_full[KV_STAGES], k_empty[KV_STAGES], v_full[KV_STAGES], v_empty[KV_STAGES];
  uint64_t s_full[2], p_half[2], p_full[2], o_done[2];
  uint64_t drain;
  uint32_t tmem_base;
};
struct SmemCP : SmemBase {
  alignas(128) uint8_t stage[2][CP_PIECE];  // gather staging (peer -> here -> local HBM)
  uint64_t stage_full[2];
  int run_a[kCpMaxRanks], run_len[kCpMaxRanks];  // KV block order: runs [a, a+len) for distance 0..W-1
};
template <bool CP>
using SmemT = typename std::conditional<CP, SmemCP, SmemBase>::type;

// Context-parallel extension: this rank's queries attend over the K/V of all ranks. Each rank
// writes its K/V rows into its own copy of the full-sequence buffer [B, 2, S, Hk, 128] (K block,
// then V block) and publishes an epoch flag; inside this kernel, warp 10 of every CTA pulls peers'
// rows into the local buffer (claiming 12 KB pieces from a per-peer ticket counter, so any
// resident CTA can finish a chunk and no CTA waits on a CTA that is not running), and the TMA
// producer waits for a peer's chunk to be complete before loading its keys. KV blocks are
// processed own-shard first, then peers in the order they are gathered.
struct CpArgs {
  int rank, world, shard_rows;
  long long row_bytes, part_bytes, batch_bytes, shard_bytes;  // token row / K or V part / batch / one rank's rows
  const uint8_t* peer_kv[kCpMaxRanks];             // each rank's full-sequence K|V buffer (own at [rank])
  uint8_t* local_kv;
  const uint64_t* flags;                           // flags[q * flag_stride]: epoch rank q published
  int flag_stride;
  uint64_t* peer_acks[kCpMaxRanks];                // where to tell rank p we finished reading its rows
  uint64_t epoch;
  unsigned int* claim;                             // [world], zero at launch
  unsigned int* done;                              // [world], zero at launch
  int pieces_per_part, pieces_per_batch, batches;
};

__device__ __forceinline__ unsigned long long f2pack_early(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp2 on the FMA pipe, used for 1/8 of the probabilities (EMU, measured) so the 16/clk MUFU pipe is
// not the softmax bottleneck. Cody-Waite range reduction x = r + f with r = rint(x) (the
// 1.5*2^23 magic-add rounding), 2^f on f in [-1/2, 1/2] by a cubic fitted for this kernel by
// weighted least squares on relative error (max rel. error 7.5e-5, far below bf16's 3.9e-3),
// and 2^r by adding r to the exponent field. x <= -126 returns 0.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -126.f);
  const float t = xc + 12582912.f;
  const float r = t - 12582912.f;
  const float f = xc - r;
  const float p = fmaf(fmaf(fmaf(0.05517098f, f, 0.24260971f), f, 0.69326097f), f, 0.99992818f);
  const int ri = __float_as_int(t) - 0x4B400000;
  const float y = __int_as_float(__float_as_int(p) + (ri << 23));
  return x <= -126.f ? 0.f : y;
}

// exp2 of a PAIR on the FMA pipe with packed fp32x2 arithmetic (same reduction and cubic as
// exp2_fma): the magic add leaves r in the low mantissa bits of t, so (bits(t) << 23) is r in the
// exponent field (the magic constant's own bits shift out of the 32-bit word), and 2^r * p is one
// integer add per element.
__device__ __forceinline__ unsigned long long exp2_fma2(float x0, float x1) {
  const unsigned long long xc = f2pack_early(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  unsigned long long t, r, f, p;
  const unsigned long long magic = f2pack_early(12582912.f, 12582912.f);
  const unsigned long long nmagic = f2pack_early(-12582912.f, -12582912.f);
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(xc), "l"(magic));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(t), "l"(nmagic));
  const unsigned long long neg1 = f2pack_early(-1.f, -1.f);
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(f) : "l"(r), "l"(neg1), "l"(xc));
  const unsigned long long c3 = f2pack_early(0.05517098f, 0.05517098f), c2 = f2pack_early(0.24260971f, 0.24260971f);
  const unsigned long long c1 = f2pack_early(0.69326097f, 0.69326097f), c0 = f2pack_early(0.99992818f, 0.99992818f);
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(c3), "l"(f), "l"(c2));
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(p) : "l"(f), "l"(c1));
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(p) : "l"(f), "l"(c0));
  const uint32_t t0 = (uint32_t)t, t1 = (uint32_t)(t >> 32);
  const uint32_t y0 = (uint32_t)p + (t0 << 23), y1 = (uint32_t)(p >> 32) + (t1 << 23);
  const uint32_t z0 = x0 <= -126.f ? 0u : y0, z1 = x1 <= -126.f ? 0u : y1;
  return ((unsigned long long)z1 << 32) | z0;
}

// Registers written by an asynchronous tcgen05.ld are only valid after tcgen05.wait::ld; this
// empty asm "rewrites" them after the wait so no use is scheduled above it.
__device__ __forceinline__ void reg_fence32(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i++) asm volatile("" : "+r"(r[i]));
}

// Blackwell packed fp32 pairs and 3-input max (halve the softmax's FFMA / FADD / FMNMX count)
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}

// stores words 0..15 of a 32-word register array (no reinterpret of the array: keeps it in registers)
__device__ __forceinline__ void tmem_st_32x32b_x16_lo(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}

__device__ __forceinline__ bool spin_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(smem_u32(bar), parity)) {
    if ((unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES / 4) return false;
  }
  return true;
}

// debug timeline: slot layout [event][j] with 64 blocks max per event kind
__device__ __forceinline__ void trace_at(const AttnArgs& a, int ev, int j) {
  if (a.trace != nullptr && blockIdx.x == 0 && j < 64) a.trace[ev * 64 + j] = clock64();
}

__device__ __forceinline__ bool key_ok(int kp, int qpos, int Sk, int causal) {
  return kp < Sk && (!causal || kp <= qpos);
}

__device__ bool cp_wait_flag(const uint64_t* f, uint64_t epoch) {
  const long long t0 = clock64();
  while (ld_acquire_sys_u64(f) < epoch) {
    if ((unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES) {
      record_error(kErrPeerTimeout);
      return false;
    }
    if (error_raised()) return false;
    __nanosleep(128);
  }
  return true;
}

__device__ bool cp_wait_done(const unsigned int* d, unsigned int target) {
  const long long t0 = clock64();
  while (ld_acquire_gpu_u32(d) < target) {
    if ((unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES) {
      record_error(kErrWaitTimeout);
      return false;
    }
    if (error_raised()) return false;
    __nanosleep(64);
  }
  fence_proxy_async_global();  // the rows were written by bulk (async-proxy) stores of other CTAs
  return true;
}

// KV blocks in gather order: a block is processed once every rank whose rows it holds is
// local; blocks needing only this rank's rows come first. A block belongs to the run of the
// rank (among those whose rows it holds) that is gathered last, so run d is rank
// (rank + d)'s block range, trimmed by its first / last block when that block also holds rows
// of a rank gathered later. O(world) work, done by one thread at CTA start.
__device__ int cp_block_owner(const CpArgs& c, int kb, int Sk) {
  const int lo = kb * TILE / c.shard_rows, hi = min(kb * TILE + TILE - 1, Sk - 1) / c.shard_rows;
  int best = lo, bd = -1;
  for (int q = lo; q <= hi; q++) {
    const int d = (q - c.rank + c.world) % c.world;
    if (d > bd) {
      bd = d;
      best = q;
    }
  }
  return best;
}

__device__ void cp_build_runs(SmemCP& sm, const CpArgs& c, int Sk) {
  for (int d = 0; d < c.world; d++) {
    const int p = (c.rank + d) % c.world;
    int a = p * c.shard_rows / TILE, b = ((p + 1) * c.shard_rows - 1) / TILE;
    if (a <= b && cp_block_owner(c, a, Sk) != p) a++;
    if (a <= b && cp_block_owner(c, b, Sk) != p) b--;
    sm.run_a[d] = a;
    sm.run_len[d] = b >= a ? b - a + 1 : 0;
  }
}

// Next KV block in run order (call once per block, in order).
struct KvCursor {
  int d = 0, i = 0;
  __device__ __forceinline__ int next(const SmemCP& sm) {
    while (i >= sm.run_len[d]) {
      d++;
      i = 0;
    }
    return sm.run_a[d] + i++;
  }
};

// Warp 10 (one lane): claim 12 KB pieces of peers' rows and move them peer -> smem -> local
// HBM with bulk copies, two pieces in flight; the CTA that completes a peer's chunk tells the
// peer it may overwrite those rows.
__device__ void cp_gather(SmemCP& sm, const CpArgs& c) {
  const unsigned int npieces = (unsigned int)(c.pieces_per_batch * c.batches);
  uint32_t ph[2] = {0, 0};
  int issued = 0, pend_p = -1;
  bool ok = true;
  auto finish = [&](int p) {  // the store of a piece of chunk p has been performed
    fence_proxy_async_global();
    const unsigned int old = atom_add_release_gpu_u32(c.done + p, 1u);
    if (old + 1 == npieces) {
      __threadfence_system();
      st_release_sys_u64(c.peer_acks[p], c.epoch);
    }
  };
  for (int d = 1; d < c.world && ok; d++) {
    const int p = (c.rank + d) % c.world;
    bool flagged = false;
    for (;;) {
      const unsigned int idx = atomicAdd(c.claim + p, 1u);
      if (idx >= npieces) break;
      if (!flagged) {
        if (!cp_wait_flag(c.flags + (size_t)p * c.flag_stride, c.epoch)) {
          ok = false;
          break;
        }
        flagged = true;
      }
      const int b = idx / c.pieces_per_batch;
      const int rem = idx % c.pieces_per_batch;
      const int part = rem / c.pieces_per_part;  // 0: K rows, 1: V rows
      const long long off = (long long)(rem % c.pieces_per_part) * CP_PIECE;
      const uint32_t n = (uint32_t)min((long long)CP_PIECE, c.shard_bytes - off);
      const long long at =
          (long long)b * c.batch_bytes + (long long)part * c.part_bytes + (long long)p * c.shard_bytes + off;
      const int st = issued & 1;
      mbar_arrive_expect_tx(&sm.stage_full[st], n);
      bulk_load_g2s(sm.stage[st], c.peer_kv[p] + at, n, &sm.stage_full[st]);
      if (!mbar_wait(&sm.stage_full[st], ph[st])) {
        spin_drain(&sm.stage_full[st], ph[st]);  // never leave the CTA with a load in flight
        ok = false;
        break;
      }
      ph[st] ^= 1;
      bulk_store_s2g(c.local_kv + at, sm.stage[st], n);
      bulk_commit();
      issued++;
      if (pend_p >= 0) {
        bulk_wait<1>();  // the previous piece's store is performed
        finish(pend_p);
      }
      pend_p = p;
    }
  }
  bulk_wait<0>();
  if (ok && pend_p >= 0) finish(pend_p);
}

// EMU: how many of every 8 exp2 pairs run on the FMA pipe (exp2_fma) instead of MUFU.
template <int EMU>
__device__ __forceinline__ bool emu_pair(int i) {
  const int k = i & 7;
  if constexpr (EMU == 2) return k == 2 || k == 6;
  if constexpr (EMU == 4) return (k & 1) == 1;
  if constexpr (EMU == 1) return k == 5;
  if constexpr (EMU == 0) return false;
  if constexpr (EMU == 3) return k == 2 || k == 5 || k == 7;
  return k == 5;  // default: 1 pair in 8 (measured best across the self-attention shapes)
}

template <bool CP, int EMU = 1>
__global__ void __launch_bounds__(CP ? NTHREADS_CP : NTHREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnArgs a, const __grid_constant__ CpArgs cp) {
  extern __shared__ uint8_t smem_raw[];
  SmemT<CP>& sm = *reinterpret_cast<SmemT<CP>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int qb = blockIdx.x % a.n_qblocks;
  const int h = (blockIdx.x / a.n_qblocks) % a.Hq;
  const int b = blockIdx.x / (a.n_qblocks * a.Hq);
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qb * 2 * TILE;
  int n_kv = (a.Sk + TILE - 1) / TILE;
  if (a.causal) n_kv = min(n_kv, (q0 + 2 * TILE + TILE - 1) / TILE);
  const bool has_b = q0 + TILE < a.Sq;  // second tile has at least one real query

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < KV_STAGES; s++) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < 2; t++) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_half[t], 4);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.o_done[t], 1);
    }
    mbar_init(&sm.drain, 1);
    if constexpr (CP) {
      mbar_init(&sm.stage_full[0], 1);
      mbar_init(&sm.stage_full[1], 1);
      cp_build_runs(sm, cp, a.Sk);
    }
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (CP && warp == 10) {
    // ------------------------------------------------------------------ K/V gather (CP only)
    if constexpr (CP) {
      if (lane == 0) cp_gather(sm, cp);
    }
  } else if (warp == 9) {
    // The producer's ring waits sleep (suspend hint) instead of probing: its loads run two
    // stages ahead, so a late wake-up costs nothing, and the issue slots of its scheduler go to
    // the softmax warps there (measured: softmax warp 1 publishes ~70 cycles earlier).
    auto wait_tma = [](uint64_t* bar, uint32_t ph) { return mbar_wait_t<kWaitSleep>(bar, ph); };
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&sm.q_full, 4 * CHUNK);
      for (int t = 0; t < 2; t++)
        for (int c = 0; c < 2; c++)
          tma_load_3d(sm.q[t] + c * CHUNK, &tmQ, &sm.q_full, h * HD + c * 64, q0 + t * TILE, b);
      bool ok = true;
      uint32_t kpend = 0, kph = 0, vpend = 0, vph = 0;
      uint32_t ready = 0;  // CP: peers whose rows are complete in the local buffer
      [[maybe_unused]] KvCursor cur;
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        int kb = j;
        if constexpr (CP) {
          kb = cur.next(sm);
          const unsigned int npieces = (unsigned int)(cp.pieces_per_batch * cp.batches);
          const int lo = kb * TILE / cp.shard_rows, hi = min(kb * TILE + TILE - 1, a.Sk - 1) / cp.shard_rows;
          for (int q = lo; q <= hi && ok; q++) {
            if (q == cp.rank || (ready >> q & 1u)) continue;
            ok = cp_wait_done(cp.done + q, npieces);
            ready |= 1u << q;
          }
          if (!ok) break;
        }
        if (!wait_tma(&sm.k_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.k_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++)
          tma_load_3d(sm.k[s] + c * CHUNK, &tmK, &sm.k_full[s], hk * HD + c * 64, kb * TILE, b);
        kpend |= 1u << s;
        kph = (kph & ~(1u << s)) | (ph << s);
        if (!wait_tma(&sm.v_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.v_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++)
          tma_load_3d(sm.v[s] + c * CHUNK, &tmV, &sm.v_full[s], hk * HD + c * 64, kb * TILE, b);
        vpend |= 1u << s;
        vph = (vph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {  // unwinding: every issued load must land before the CTA exits
        spin_drain(&sm.q_full, 0);
        for (int s = 0; s < KV_STAGES; s++) {
          if (kpend >> s & 1) spin_drain(&sm.k_full[s], (kph >> s) & 1);
          if (vpend >> s & 1) spin_drain(&sm.v_full[s], (vph >> s) & 1);
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(TILE, TILE);
      constexpr uint32_t idO = umma_idesc_bf16_f32(TILE, HD, false, true);  // V is MN-major
      bool ok = mbar_wait(&sm.q_full, 0);
      // Descriptors are built once per operand base; a K step adds its byte offset / 16 to the
      // start-address field (shared addresses stay below 2^18, so the 14-bit field never carries).
      // Descriptors are built once per operand base; a K step adds its byte offset / 16 to the
      // start-address field (shared addresses stay below 2^18, so the 14-bit field never
      // carries). Measured: p_full -> S(j+1) issued 156 cycles instead of 181.
      auto issue_S = [&](int t, int s) {
        const uint64_t dq = umma_desc_kmajor_sw128(smem_u32(sm.q[t]));
        const uint64_t dk = umma_desc_kmajor_sw128(smem_u32(sm.k[s]));
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const uint32_t off = ((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4;
          umma_bf16_ss(tbase + t * 128, dq + off, dk + off, idS, kk > 0);
        }
        umma_commit(&sm.s_full[t]);
      };
      // O += P V over keys [16*k0, 16*k1); P (bf16 pairs) sits in the first 64 columns of S
      auto issue_PV_part = [&](int t, int s, int j, int k0, int k1) {
        const uint64_t dv = umma_desc_mnmajor_sw128(smem_u32(sm.v[s]), CHUNK);
#pragma unroll
        for (int kk = k0; kk < k1; kk++)
          umma_bf16_ts(tbase + 256 + t * 128, tbase + t * 128 + kk * 8, dv + ((kk * 16 * 128) >> 4), idO,
                       (j | kk) != 0);
      };
      // P arrives in two halves: the first four PV steps start while the softmax is still
      // producing keys 64..127
      auto issue_PV = [&](int t, int s, int j) -> bool {
        if (!mbar_wait(&sm.p_half[t], j & 1)) return false;
        tc_fence_after();
        issue_PV_part(t, s, j, 0, TILE / 32);
        if (!mbar_wait(&sm.p_full[t], j & 1)) return false;
        if (t == 0) trace_at(a, 18, j);
        tc_fence_after();
        issue_PV_part(t, s, j, TILE / 32, TILE / 16);
        umma_commit(&sm.o_done[t]);
        return true;
      };
      if (ok && n_kv > 0) {
        ok = mbar_wait(&sm.k_full[0], 0);
        if (ok) {
          tc_fence_after();
          issue_S(0, 0);
          if (has_b) issue_S(1, 0);
          umma_commit(&sm.k_empty[0]);
        }
      }
      for (int j = 0; ok && j < n_kv; j++) {
        const int s = j % KV_STAGES, s1 = (j + 1) % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1, ph1 = ((j + 1) / KV_STAGES) & 1;
        const bool more = j + 1 < n_kv;
        if (!mbar_wait(&sm.v_full[s], ph)) {
          ok = false;
          break;
        }
        trace_at(a, 0, j);
        if (!issue_PV(0, s, j)) {
          ok = false;
          break;
        }
        if (more) {
          if (!mbar_wait(&sm.k_full[s1], ph1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          trace_at(a, 1, j);
          issue_S(0, s1);
        }
        if (has_b) {
          trace_at(a, 2, j);
          if (!issue_PV(1, s, j)) {
            ok = false;
            break;
          }
          if (more) issue_S(1, s1);
        }
        umma_commit(&sm.v_empty[s]);
        if (more) umma_commit(&sm.k_empty[s1]);
      }
      if (!ok) {
        umma_commit(&sm.drain);
        spin_drain(&sm.drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int t = warp >> 2;           // tile
    const int quad = warp & 3;         // TMEM lane quadrant
    const int r = quad * 32 + lane;    // row in tile
    const int qpos = q0 + t * TILE + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tbase + t * 128 + lane_off;
    const uint32_t tO = tbase + 256 + t * 128 + lane_off;
    const bool active = (t == 0) || has_b;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    [[maybe_unused]] KvCursor cur;
    for (int j = 0; active && j < n_kv; j++) {
      int kbase = j * TILE;
      if constexpr (CP) kbase = cur.next(sm) * TILE;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (r == 0) trace_at(a, 4 + 4 * t, j);
      if (a.diag == 2) {  // timing diagnostic: no softmax work at all
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[t]);
        continue;
      }
      const bool masked = (kbase + TILE > a.Sk) || (a.causal && kbase + TILE > q0 + t * TILE);
      // Single pass over the S row: all 128 columns in flight in one TMEM round trip,
      // 8-way tree max, exp2 in registers, P packed in place (pair i of chunk c -> word i),
      // four 16-column TMEM stores. Registers: 128 for the row + a few scalars.
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld_32x32b_x32(tS + c * 32, v[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; c++) reg_fence32(v[c]);
      if (r == 0) trace_at(a, 5 + 4 * t, j);
      if (masked) {
        // keys [kbase, kbase + lim) are visible to this row
        const int lim = min(a.Sk, a.causal ? qpos + 1 : a.Sk) - kbase;
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int e = 0; e < 32; e++)
            if (c * 32 + e >= lim) v[c][e] = 0xff800000u;
      }
      float mx;
      {
        float m0 = __uint_as_float(v[0][0]), m1 = __uint_as_float(v[1][0]);
        float m2 = __uint_as_float(v[2][0]), m3 = __uint_as_float(v[3][0]);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          m0 = max3(m0, __uint_as_float(v[0][e]), __uint_as_float(v[0][e + 1]));
          m1 = max3(m1, __uint_as_float(v[1][e]), __uint_as_float(v[1][e + 1]));
          m2 = max3(m2, __uint_as_float(v[2][e]), __uint_as_float(v[2][e + 1]));
          m3 = max3(m3, __uint_as_float(v[3][e]), __uint_as_float(v[3][e + 1]));
        }
        mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      }
      mx *= a.scale_log2;
      // Rescale decision is warp-uniform (tcgen05.ld/st below are warp-collective): if any row's
      // max grew past the threshold (or is still -inf), every row of the warp moves to its exact
      // new max. O itself is rescaled after P is formed so the S row registers are dead by then.
      const bool need = (mx > m + RESCALE_THRESHOLD) || (m == -INFINITY);
      const bool rescale = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (rescale) {
        const float m_new = fmaxf(m, mx);
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      const float msub = (m == -INFINITY) ? 0.f : m;
      if (r == 0) trace_at(a, 12 + 2 * t, j);
      unsigned long long rsc[4] = {0ull, 0ull, 0ull, 0ull};  // packed (even, odd) partial row sums
      const unsigned long long scale2 = f2pack(a.scale_log2, a.scale_log2);
      const unsigned long long negm2 = f2pack(-msub, -msub);
#pragma unroll
      for (int c = 0; c < 4; c++) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const unsigned long long x2 =
              fma2(f2pack(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])), scale2, negm2);
          float x0, x1;
          f2unpack(x2, x0, x1);
          float p0, p1;
          if (emu_pair<EMU>(i)) {  // EMU pairs in 8 on the FMA pipe
            const unsigned long long e2 = exp2_fma2(x0, x1);
            p0 = __uint_as_float((uint32_t)e2);
            p1 = __uint_as_float((uint32_t)(e2 >> 32));
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          rsc[i & 3] = add2(rsc[i & 3], f2pack(p0, p1));
          v[c][i] = pack_bf16x2(p0, p1);  // word i is no longer needed as input (2i >= i)
        }
        tmem_st_32x32b_x16_lo(tS + c * 16, v[c]);
        if (c == 1) {
          // O must be rescaled before ANY of this block's PV steps run, i.e. before p_half.
          // Chunks 0-1 are stored, so their registers are free for the O round trip here.
          if (rescale && j > 0) {
            // O_X is quiescent once PV_X(j-1) completed (its commit precedes S_X(j)'s)
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.o_done[t], (j - 1) & 1))) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int oc = 0; oc < 4; oc++) {
              uint32_t o[32];
              tmem_ld_32x32b_x32(tO + oc * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st_32x32b_x32(tO + oc * 32, o);
            }
          }
          // keys 0..63 done: let the MMA warp start on them
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_half[t]);
          if (r == 0) trace_at(a, 13 + 2 * t, j);
        }
      }
      float rs;
      {
        float a0, a1, b0, b1, c0, c1, d0, d1;
        f2unpack(add2(rsc[0], rsc[1]), a0, a1);
        f2unpack(add2(rsc[2], rsc[3]), b0, b1);
        rs = (a0 + a1) + (b0 + b1);
        (void)c0, (void)c1, (void)d0, (void)d1;
      }
      if (r == 0) trace_at(a, 6 + 4 * t, j);
      if (!ok) break;
      l += rs;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[t]);
      if (r == 0) trace_at(a, 7 + 4 * t, j);
      if (t == 0 && quad > 0 && lane == 0) trace_at(a, quad == 3 ? 3 : 15 + quad, j);  // 3, 16, 17
    }
    // epilogue: O / l -> bf16
    if (active && ok && n_kv > 0 && __all_sync(0xffffffffu, mbar_wait(&sm.o_done[t], (n_kv - 1) & 1))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + c * 32, v);
        tmem_ld_wait();
        if (qpos < a.Sq) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[u * 8 + 0]) * inv, __uint_as_float(v[u * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[u * 8 + 2]) * inv, __uint_as_float(v[u * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[u * 8 + 4]) * inv, __uint_as_float(v[u * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[u * 8 + 6]) * inv, __uint_as_float(v[u * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + u * 8) = w;
          }
        }
      }
    } else if (active && n_kv == 0 && qpos < a.Sq) {
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD;
      for (int d = 0; d < HD; d++) out[d] = __float2bfloat16(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Experimental variant (timing comparisons, ``_diag_mode`` 200 + EMU): ONE 128-query tile per CTA
// with S double-buffered in TMEM, so the QK^T of block j+1 and j+2 no longer waits on the softmax
// of block j. TMEM: S0 (columns 0-127), S1 (128-255), O (256-383). MMA issue order:
//   S(0) S(1) | PV(0) S(2) | PV(1) S(3) | ...     S(j+2) reuses the columns PV(j) reads as P.
// The softmax warps run block after block without waiting on the tensor core (the S they need was
// issued one block earlier). P barriers are per S buffer, so the softmax running one block ahead
// never completes a phase the MMA warp has not seen. 192 threads: warps 0-3 softmax/epilogue (rows),
// warp 4 TMEM owner + MMA issuer, warp 5 TMA producer. K/V traffic from L2 is twice the 2-tile
// kernel's (each CTA reads the whole K/V of its head for 128 queries).
constexpr int KV1 = 3;  // K/V ring depth of the one-tile kernel (224 KB of shared memory)
struct SmemOne {
  uint8_t q[2 * CHUNK];
  uint8_t k[KV1][2 * CHUNK];
  uint8_t v[KV1][2 * CHUNK];
  uint64_t q_full;
  uint64_t k_full[KV1], k_empty[KV1], v_full[KV1], v_empty[KV1];
  uint64_t s_full[2], p_half[2], p_full[2], o_done;
  uint64_t o_final;  // committed once, after the last PV: o_done can lag two phases at the end
  uint64_t drain;
  uint32_t tmem_base;
};
constexpr int NTHREADS1 = 192;

template <int EMU>
__global__ void __launch_bounds__(NTHREADS1, 1)
    attn1_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  SmemOne& sm = *reinterpret_cast<SmemOne*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = blockIdx.x % a.n_qblocks;
  const int h = (blockIdx.x / a.n_qblocks) % a.Hq;
  const int b = blockIdx.x / (a.n_qblocks * a.Hq);
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qb * TILE;
  int n_kv = (a.Sk + TILE - 1) / TILE;
  if (a.causal) n_kv = min(n_kv, (q0 + TILE + TILE - 1) / TILE);

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < KV1; s++) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int u = 0; u < 2; u++) {
      mbar_init(&sm.s_full[u], 1);
      mbar_init(&sm.p_half[u], 4);
      mbar_init(&sm.p_full[u], 4);
    }
    mbar_init(&sm.o_done, 1);
    mbar_init(&sm.o_final, 1);
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (warp == 5) {
    // ------------------------------------------------------------------ TMA producer
    auto wait_tma = [](uint64_t* bar, uint32_t ph) { return mbar_wait_t<kWaitSleep>(bar, ph); };
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&sm.q_full, 2 * CHUNK);
      for (int c = 0; c < 2; c++) tma_load_3d(sm.q + c * CHUNK, &tmQ, &sm.q_full, h * HD + c * 64, q0, b);
      bool ok = true;
      uint32_t kpend = 0, kph = 0, vpend = 0, vph = 0;
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % KV1;
        const uint32_t ph = (j / KV1) & 1;
        if (!wait_tma(&sm.k_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.k_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++) tma_load_3d(sm.k[s] + c * CHUNK, &tmK, &sm.k_full[s], hk * HD + c * 64, j * TILE, b);
        kpend |= 1u << s;
        kph = (kph & ~(1u << s)) | (ph << s);
        if (!wait_tma(&sm.v_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.v_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++) tma_load_3d(sm.v[s] + c * CHUNK, &tmV, &sm.v_full[s], hk * HD + c * 64, j * TILE, b);
        vpend |= 1u << s;
        vph = (vph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {  // unwinding: every issued load must land before the CTA exits
        spin_drain(&sm.q_full, 0);
        for (int s = 0; s < KV1; s++) {
          if (kpend >> s & 1) spin_drain(&sm.k_full[s], (kph >> s) & 1);
          if (vpend >> s & 1) spin_drain(&sm.v_full[s], (vph >> s) & 1);
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(TILE, TILE);
      constexpr uint32_t idO = umma_idesc_bf16_f32(TILE, HD, false, true);  // V is MN-major
      bool ok = mbar_wait(&sm.q_full, 0);
      const uint64_t dq = umma_desc_kmajor_sw128(smem_u32(sm.q));
      auto issue_S = [&](int j) {  // S(j) into buffer j % 2 from K stage j % KV1
        const int s = j % KV1;
        const uint64_t dk = umma_desc_kmajor_sw128(smem_u32(sm.k[s]));
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const uint32_t off = ((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4;
          umma_bf16_ss(tbase + (j & 1) * 128, dq + off, dk + off, idS, kk > 0);
        }
        umma_commit(&sm.s_full[j & 1]);
        umma_commit(&sm.k_empty[s]);
      };
      auto issue_PV_part = [&](int j, int k0, int k1) {
        const uint64_t dv = umma_desc_mnmajor_sw128(smem_u32(sm.v[j % KV1]), CHUNK);
#pragma unroll
        for (int kk = k0; kk < k1; kk++)
          umma_bf16_ts(tbase + 256, tbase + (j & 1) * 128 + kk * 8, dv + ((kk * 16 * 128) >> 4), idO, (j | kk) != 0);
      };
      for (int j = 0; ok && j < 2 && j < n_kv; j++) {
        ok = mbar_wait(&sm.k_full[j % KV1], (j / KV1) & 1);
        if (!ok) break;
        tc_fence_after();
        issue_S(j);
      }
      for (int j = 0; ok && j < n_kv; j++) {
        const int s = j % KV1;
        const uint32_t pph = (j >> 1) & 1;  // phase of this S buffer's P barriers
        if (!mbar_wait(&sm.v_full[s], (j / KV1) & 1) || !mbar_wait(&sm.p_half[j & 1], pph)) {
          ok = false;
          break;
        }
        trace_at(a, 0, j);
        tc_fence_after();
        issue_PV_part(j, 0, TILE / 32);
        if (!mbar_wait(&sm.p_full[j & 1], pph)) {
          ok = false;
          break;
        }
        trace_at(a, 18, j);
        tc_fence_after();
        issue_PV_part(j, TILE / 32, TILE / 16);
        umma_commit(&sm.o_done);
        umma_commit(&sm.v_empty[s]);
        if (j == n_kv - 1) umma_commit(&sm.o_final);
        if (j + 2 < n_kv) {
          if (!mbar_wait(&sm.k_full[(j + 2) % KV1], ((j + 2) / KV1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_S(j + 2);
          trace_at(a, 1, j);
        }
      }
      if (!ok) {
        umma_commit(&sm.drain);
        spin_drain(&sm.drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int quad = warp;           // TMEM lane quadrant = rows 32*quad .. +31
    const int r = quad * 32 + lane;
    const int qpos = q0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tO = tbase + 256 + lane_off;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; j++) {
      const int kbase = j * TILE;
      const uint32_t tS = tbase + (j & 1) * 128 + lane_off;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[j & 1], (j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (r == 0) trace_at(a, 4, j);
      const bool masked = (kbase + TILE > a.Sk) || (a.causal && kbase + TILE > q0);
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld_32x32b_x32(tS + c * 32, v[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; c++) reg_fence32(v[c]);
      if (r == 0) trace_at(a, 5, j);
      if (masked) {
        const int lim = min(a.Sk, a.causal ? qpos + 1 : a.Sk) - kbase;
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int e = 0; e < 32; e++)
            if (c * 32 + e >= lim) v[c][e] = 0xff800000u;
      }
      float mx;
      {
        float m0 = __uint_as_float(v[0][0]), m1 = __uint_as_float(v[1][0]);
        float m2 = __uint_as_float(v[2][0]), m3 = __uint_as_float(v[3][0]);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          m0 = max3(m0, __uint_as_float(v[0][e]), __uint_as_float(v[0][e + 1]));
          m1 = max3(m1, __uint_as_float(v[1][e]), __uint_as_float(v[1][e + 1]));
          m2 = max3(m2, __uint_as_float(v[2][e]), __uint_as_float(v[2][e + 1]));
          m3 = max3(m3, __uint_as_float(v[3][e]), __uint_as_float(v[3][e + 1]));
        }
        mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      }
      mx *= a.scale_log2;
      const bool need = (mx > m + RESCALE_THRESHOLD) || (m == -INFINITY);
      const bool rescale = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (rescale) {
        const float m_new = fmaxf(m, mx);
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      const float msub = (m == -INFINITY) ? 0.f : m;
      if (r == 0) trace_at(a, 12, j);
      unsigned long long rsc[4] = {0ull, 0ull, 0ull, 0ull};
      const unsigned long long scale2 = f2pack(a.scale_log2, a.scale_log2);
      const unsigned long long negm2 = f2pack(-msub, -msub);
#pragma unroll
      for (int c = 0; c < 4; c++) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const unsigned long long x2 =
              fma2(f2pack(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])), scale2, negm2);
          float x0, x1;
          f2unpack(x2, x0, x1);
          float p0, p1;
          if (emu_pair<EMU>(i)) {
            const unsigned long long e2 = exp2_fma2(x0, x1);
            p0 = __uint_as_float((uint32_t)e2);
            p1 = __uint_as_float((uint32_t)(e2 >> 32));
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          rsc[i & 3] = add2(rsc[i & 3], f2pack(p0, p1));
          v[c][i] = pack_bf16x2(p0, p1);
        }
        tmem_st_32x32b_x16_lo(tS + c * 16, v[c]);
        if (c == 1) {
          if (rescale && j > 0) {
            // O is quiescent once PV(j-1) completed; PV(j) waits on this block's p_half
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.o_done, (j - 1) & 1))) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int oc = 0; oc < 4; oc++) {
              uint32_t o[32];
              tmem_ld_32x32b_x32(tO + oc * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st_32x32b_x32(tO + oc * 32, o);
            }
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_half[j & 1]);
          if (r == 0) trace_at(a, 13, j);
        }
      }
      if (!ok) break;
      float rs;
      {
        float a0, a1, b0, b1;
        f2unpack(add2(rsc[0], rsc[1]), a0, a1);
        f2unpack(add2(rsc[2], rsc[3]), b0, b1);
        rs = (a0 + a1) + (b0 + b1);
      }
      if (r == 0) trace_at(a, 6, j);
      l += rs;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[j & 1]);
      if (r == 0) trace_at(a, 7, j);
    }
    if (ok && n_kv > 0 && __all_sync(0xffffffffu, mbar_wait(&sm.o_final, 0))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + c * 32, v);
        tmem_ld_wait();
        if (qpos < a.Sq) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[u * 8 + 0]) * inv, __uint_as_float(v[u * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[u * 8 + 2]) * inv, __uint_as_float(v[u * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[u * 8 + 4]) * inv, __uint_as_float(v[u * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[u * 8 + 6]) * inv, __uint_as_float(v[u * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + u * 8) = w;
          }
        }
      }
    } else if (n_kv == 0 && qpos < a.Sq) {
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD;
      for (int d = 0; d < HD; d++) out[d] = __float2bfloat16(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Split-row variant (``_diag_mode`` 300 + EMU): the default kernel's two ping-ponging 128-query
// tiles, with every query row's softmax shared by TWO warps, one per 64-key half of the S row.
// 18 warps (576 threads):
//   warps 0-7   tile A: warps 0-3 keys 0-63, warps 4-7 keys 64-127 (warp w: TMEM lanes 32(w%4)..+31)
//   warps 8-15  tile B, same split
//   warp 16     TMEM owner + MMA issuer;  warp 17  TMA producer
// Each softmax warp's chain per KV block is half the default one (64 instead of 128 values per
// thread), and four softmax warps per scheduler keep the MUFU and FMA pipes busier, which
// shortens the softmax -> PV -> QK^T chain that sets the default kernel's period.
// The two halves of a row agree on its running max by exchanging their partial maxima through
// shared memory (double-buffered by block parity, a 64-thread named barrier per warp pair), so
// they take identical rescale decisions. The exchange is an mbarrier per warp pair (64 arrivals,
// bounded waits), never a hardware named barrier, so a warp that unwinds on an error cannot leave
// its partner blocked. P of keys 0-63 is packed into S columns 0-31 and P of
// keys 64-127 into columns 64-95 (each half overwrites only S columns it has already read).
// Barriers per tile: p_lo (8 arrivals: half-0 warps once their P is stored, half-1 warps once
// their share of any O rescale is done) gates PV over keys 0-63; p_hi (4 arrivals, half-1 warps'
// P) gates PV over keys 64-127. O rescales (rare: stale-max threshold 2^8) are split by column
// halves and finish before p_lo, i.e. before any PV of the block.
constexpr int NTHREADS2X = 576;
struct Smem2x : SmemBase {
  float xmax[2][2][2][TILE];  // [block parity][tile][half][row]: partial row maxima
  float lsum[2][2][TILE];     // [tile][half][row]: partial row sums for the epilogue
  uint64_t p_lo[2], p_hi[2];
  uint64_t xbar[2][4];        // [tile][quad]: the two warps that share rows 32*quad..+31
};

// Both warps of a pair arrive (all lanes, after their shared-memory writes) and wait, bounded,
// for the phase of this exchange.
__device__ __forceinline__ bool pair_exchange(uint64_t* bar, uint32_t parity) {
  mbar_arrive(bar);
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

template <int EMU>
__global__ void __launch_bounds__(NTHREADS2X, 1)
    attn2x_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem2x& sm = *reinterpret_cast<Smem2x*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int qb = blockIdx.x % a.n_qblocks;
  const int h = (blockIdx.x / a.n_qblocks) % a.Hq;
  const int b = blockIdx.x / (a.n_qblocks * a.Hq);
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qb * 2 * TILE;
  int n_kv = (a.Sk + TILE - 1) / TILE;
  if (a.causal) n_kv = min(n_kv, (q0 + 2 * TILE + TILE - 1) / TILE);
  const bool has_b = q0 + TILE < a.Sq;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < KV_STAGES; s++) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < 2; t++) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_lo[t], 8);
      mbar_init(&sm.p_hi[t], 4);
      mbar_init(&sm.o_done[t], 1);
      for (int q = 0; q < 4; q++) mbar_init(&sm.xbar[t][q], 64);
    }
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 16) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (warp == 17) {
    // ------------------------------------------------------------------ TMA producer
    auto wait_tma = [](uint64_t* bar, uint32_t ph) { return mbar_wait_t<kWaitSleep>(bar, ph); };
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&sm.q_full, 4 * CHUNK);
      for (int t = 0; t < 2; t++)
        for (int c = 0; c < 2; c++)
          tma_load_3d(sm.q[t] + c * CHUNK, &tmQ, &sm.q_full, h * HD + c * 64, q0 + t * TILE, b);
      bool ok = true;
      uint32_t kpend = 0, kph = 0, vpend = 0, vph = 0;
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        if (!wait_tma(&sm.k_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.k_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++) tma_load_3d(sm.k[s] + c * CHUNK, &tmK, &sm.k_full[s], hk * HD + c * 64, j * TILE, b);
        kpend |= 1u << s;
        kph = (kph & ~(1u << s)) | (ph << s);
        if (!wait_tma(&sm.v_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.v_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++) tma_load_3d(sm.v[s] + c * CHUNK, &tmV, &sm.v_full[s], hk * HD + c * 64, j * TILE, b);
        vpend |= 1u << s;
        vph = (vph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {  // unwinding: every issued load must land before the CTA exits
        spin_drain(&sm.q_full, 0);
        for (int s = 0; s < KV_STAGES; s++) {
          if (kpend >> s & 1) spin_drain(&sm.k_full[s], (kph >> s) & 1);
          if (vpend >> s & 1) spin_drain(&sm.v_full[s], (vph >> s) & 1);
        }
      }
    }
  } else if (warp == 16) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(TILE, TILE);
      constexpr uint32_t idO = umma_idesc_bf16_f32(TILE, HD, false, true);  // V is MN-major
      bool ok = mbar_wait(&sm.q_full, 0);
      auto issue_S = [&](int t, int s) {
        const uint64_t dq = umma_desc_kmajor_sw128(smem_u32(sm.q[t]));
        const uint64_t dk = umma_desc_kmajor_sw128(smem_u32(sm.k[s]));
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const uint32_t off = ((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4;
          umma_bf16_ss(tbase + t * 128, dq + off, dk + off, idS, kk > 0);
        }
        umma_commit(&sm.s_full[t]);
      };
      // O += P V over keys [16*k0, 16*k1): P of keys 0-63 in S columns 0-31, of keys 64-127 in 64-95
      auto issue_PV_part = [&](int t, int s, int j, int k0, int k1) {
        const uint64_t dv = umma_desc_mnmajor_sw128(smem_u32(sm.v[s]), CHUNK);
#pragma unroll
        for (int kk = k0; kk < k1; kk++)
          umma_bf16_ts(tbase + 256 + t * 128, tbase + t * 128 + kk * 8 + (kk >= 4 ? 32 : 0),
                       dv + ((kk * 16 * 128) >> 4), idO, (j | kk) != 0);
      };
      auto issue_PV = [&](int t, int s, int j) -> bool {
        if (!mbar_wait(&sm.p_lo[t], j & 1)) return false;
        tc_fence_after();
        issue_PV_part(t, s, j, 0, TILE / 32);
        if (!mbar_wait(&sm.p_hi[t], j & 1)) return false;
        tc_fence_after();
        issue_PV_part(t, s, j, TILE / 32, TILE / 16);
        umma_commit(&sm.o_done[t]);
        return true;
      };
      if (ok && n_kv > 0) {
        ok = mbar_wait(&sm.k_full[0], 0);
        if (ok) {
          tc_fence_after();
          issue_S(0, 0);
          if (has_b) issue_S(1, 0);
          umma_commit(&sm.k_empty[0]);
        }
      }
      for (int j = 0; ok && j < n_kv; j++) {
        const int s = j % KV_STAGES, s1 = (j + 1) % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1, ph1 = ((j + 1) / KV_STAGES) & 1;
        const bool more = j + 1 < n_kv;
        if (!mbar_wait(&sm.v_full[s], ph)) {
          ok = false;
          break;
        }
        if (!issue_PV(0, s, j)) {
          ok = false;
          break;
        }
        if (more) {
          if (!mbar_wait(&sm.k_full[s1], ph1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_S(0, s1);
        }
        if (has_b) {
          if (!issue_PV(1, s, j)) {
            ok = false;
            break;
          }
          if (more) issue_S(1, s1);
        }
        umma_commit(&sm.v_empty[s]);
        if (more) umma_commit(&sm.k_empty[s1]);
      }
      if (!ok) {
        umma_commit(&sm.drain);
        spin_drain(&sm.drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int t = warp >> 3;            // tile
    const int half = (warp >> 2) & 1;   // key half of the S row (and column half of O)
    const int quad = warp & 3;          // TMEM lane quadrant
    const int r = quad * 32 + lane;     // row in tile
    const int qpos = q0 + t * TILE + r;
    uint64_t* xbar = &sm.xbar[t][quad];  // exchange barrier shared with the other half's warp
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tbase + t * 128 + lane_off;
    const uint32_t tO = tbase + 256 + t * 128 + lane_off;
    const bool active = (t == 0) || has_b;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; active && j < n_kv; j++) {
      const int kbase = j * TILE + half * 64;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool masked = (kbase + 64 > a.Sk) || (a.causal && kbase + 64 > q0 + t * TILE);
      uint32_t v[2][32];
#pragma unroll
      for (int c = 0; c < 2; c++) tmem_ld_32x32b_x32(tS + half * 64 + c * 32, v[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 2; c++) reg_fence32(v[c]);
      if (masked) {
        const int lim = min(a.Sk, a.causal ? qpos + 1 : a.Sk) - kbase;  // keys [kbase, kbase+lim) visible
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
          for (int e = 0; e < 32; e++)
            if (c * 32 + e >= lim) v[c][e] = 0xff800000u;
      }
      float mx;
      {
        float m0 = __uint_as_float(v[0][0]), m1 = __uint_as_float(v[0][1]);
        float m2 = __uint_as_float(v[1][0]), m3 = __uint_as_float(v[1][1]);
#pragma unroll
        for (int e = 2; e < 32; e += 4) {
          m0 = max3(m0, __uint_as_float(v[0][e]), __uint_as_float(v[0][e + 1]));
          m1 = max3(m1, __uint_as_float(v[0][e + 2]), __uint_as_float(v[0][e + 3]));
          m2 = max3(m2, __uint_as_float(v[1][e]), __uint_as_float(v[1][e + 1]));
          m3 = max3(m3, __uint_as_float(v[1][e + 2]), __uint_as_float(v[1][e + 3]));
        }
        mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      }
      // both halves of the row see the same full-row max
      sm.xmax[j & 1][t][half][r] = mx;
      if (!pair_exchange(xbar, j & 1)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, sm.xmax[j & 1][t][half ^ 1][r]) * a.scale_log2;
      const bool need = (mx > m + RESCALE_THRESHOLD) || (m == -INFINITY);
      const bool rescale = __any_sync(0xffffffffu, need);  // same rows in both warps: same decision
      float alpha = 1.f;
      if (rescale) {
        const float m_new = fmaxf(m, mx);
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      const bool o_fix = rescale && j > 0;  // O holds earlier blocks' sums: rescale it before PV(j)
      if (half == 1 && !o_fix) {  // nothing of O to fix here: PV over keys 0-63 may start
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_lo[t]);
      }
      const float msub = (m == -INFINITY) ? 0.f : m;
      unsigned long long rsc[4] = {0ull, 0ull, 0ull, 0ull};
      const unsigned long long scale2 = f2pack(a.scale_log2, a.scale_log2);
      const unsigned long long negm2 = f2pack(-msub, -msub);
#pragma unroll
      for (int c = 0; c < 2; c++) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const unsigned long long x2 =
              fma2(f2pack(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])), scale2, negm2);
          float x0, x1;
          f2unpack(x2, x0, x1);
          float p0, p1;
          if (emu_pair<EMU>(i)) {
            const unsigned long long e2 = exp2_fma2(x0, x1);
            p0 = __uint_as_float((uint32_t)e2);
            p1 = __uint_as_float((uint32_t)(e2 >> 32));
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          rsc[i & 3] = add2(rsc[i & 3], f2pack(p0, p1));
          v[c][i] = pack_bf16x2(p0, p1);
        }
        tmem_st_32x32b_x16_lo(tS + half * 64 + c * 16, v[c]);
      }
      {
        float a0, a1, b0, b1;
        f2unpack(add2(rsc[0], rsc[1]), a0, a1);
        f2unpack(add2(rsc[2], rsc[3]), b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
      if (o_fix) {
        // this half's 64 columns of O, once PV(j-1) completed (its commit precedes S(j)'s); the
        // S registers are dead by now, so the O round trip adds no register pressure
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.o_done[t], (j - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int oc = 0; oc < 2; oc++) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + half * 64 + oc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + half * 64 + oc * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (half == 0 || o_fix) mbar_arrive(&sm.p_lo[t]);
        if (half == 1) mbar_arrive(&sm.p_hi[t]);
      }
    }
    // epilogue: the row sum is the two halves' sums; each half writes its 64 output columns
    if (active && ok) {
      sm.lsum[t][half][r] = l;
      ok = pair_exchange(xbar, n_kv & 1);
      l += sm.lsum[t][half ^ 1][r];
    }
    if (active && ok && n_kv > 0 && __all_sync(0xffffffffu, mbar_wait(&sm.o_done[t], (n_kv - 1) & 1))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD + half * 64;
#pragma unroll
      for (int c = 0; c < 2; c++) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + half * 64 + c * 32, v);
        tmem_ld_wait();
        if (qpos < a.Sq) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[u * 8 + 0]) * inv, __uint_as_float(v[u * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[u * 8 + 2]) * inv, __uint_as_float(v[u * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[u * 8 + 4]) * inv, __uint_as_float(v[u * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[u * 8 + 6]) * inv, __uint_as_float(v[u * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + u * 8) = w;
          }
        }
      }
    } else if (active && n_kv == 0 && qpos < a.Sq) {
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD + half * 64;
      for (int d = 0; d < 64; d++) out[d] = __float2bfloat16(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 16) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// P-through-shared-memory variant (``_diag_mode`` 400 + EMU). The default kernel keeps P in TMEM
// over the S columns, so QK^T of block j+1 can only be issued after P.V of block j has consumed
// P: per tile the period is softmax + handoff + P.V + QK^T. Here each softmax warp releases S
// as soon as the row is in registers (s_free), and writes P as a 128-byte-swizzled K-major tile
// into shared memory; the MMA warp issues S(j+1) on s_free and P.V(j) on p_full, whichever is
// ready first (it polls both tiles' barriers), so QK^T of the next block overlaps the softmax
// of the current one. Shared memory: Q (2 tiles) + K and V (2 stages each) + ONE P tile shared
// by tiles A and B in turn (224 KB): a tile's softmax writes P once the other tile's P.V that
// last read the buffer completed (p_free_a / p_free_b, one phase per block each).
struct SmemP : SmemBase {
  alignas(1024) uint8_t p[2 * CHUNK];  // [128 rows x 128 keys] bf16, two 64-key swizzled chunks
  uint64_t s_free[2], p_free[2];       // p_free[t]: P.V of tile t finished reading the P buffer
};

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int EMU>
__global__ void __launch_bounds__(NTHREADS, 1)
    attnP_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  SmemP& sm = *reinterpret_cast<SmemP*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int qb = blockIdx.x % a.n_qblocks;
  const int h = (blockIdx.x / a.n_qblocks) % a.Hq;
  const int b = blockIdx.x / (a.n_qblocks * a.Hq);
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qb * 2 * TILE;
  int n_kv = (a.Sk + TILE - 1) / TILE;
  if (a.causal) n_kv = min(n_kv, (q0 + 2 * TILE + TILE - 1) / TILE);
  const bool has_b = q0 + TILE < a.Sq;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < KV_STAGES; s++) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < 2; t++) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.s_free[t], 4);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.o_done[t], 1);
      mbar_init(&sm.p_free[t], 1);
    }
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (warp == 9) {
    // ------------------------------------------------------------------ TMA producer
    auto wait_tma = [](uint64_t* bar, uint32_t ph) { return mbar_wait_t<kWaitSleep>(bar, ph); };
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&sm.q_full, 4 * CHUNK);
      for (int t = 0; t < 2; t++)
        for (int c = 0; c < 2; c++)
          tma_load_3d(sm.q[t] + c * CHUNK, &tmQ, &sm.q_full, h * HD + c * 64, q0 + t * TILE, b);
      bool ok = true;
      uint32_t kpend = 0, kph = 0, vpend = 0, vph = 0;
      for (int j = 0; j < n_kv && ok; j++) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        if (!wait_tma(&sm.k_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.k_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++) tma_load_3d(sm.k[s] + c * CHUNK, &tmK, &sm.k_full[s], hk * HD + c * 64, j * TILE, b);
        kpend |= 1u << s;
        kph = (kph & ~(1u << s)) | (ph << s);
        if (!wait_tma(&sm.v_empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.v_full[s], 2 * CHUNK);
        for (int c = 0; c < 2; c++) tma_load_3d(sm.v[s] + c * CHUNK, &tmV, &sm.v_full[s], hk * HD + c * 64, j * TILE, b);
        vpend |= 1u << s;
        vph = (vph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {
        spin_drain(&sm.q_full, 0);
        for (int s = 0; s < KV_STAGES; s++) {
          if (kpend >> s & 1) spin_drain(&sm.k_full[s], (kph >> s) & 1);
          if (vpend >> s & 1) spin_drain(&sm.v_full[s], (vph >> s) & 1);
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------ MMA issuer (event driven)
    if (elect_one()) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(TILE, TILE);
      constexpr uint32_t idO = umma_idesc_bf16_f32(TILE, HD, false, true);  // P K-major, V MN-major
      bool ok = mbar_wait(&sm.q_full, 0);
      const int nt = has_b ? 2 : 1;
      auto issue_S = [&](int t, int j) {
        const int s = j % KV_STAGES;
        const uint64_t dq = umma_desc_kmajor_sw128(smem_u32(sm.q[t]));
        const uint64_t dk = umma_desc_kmajor_sw128(smem_u32(sm.k[s]));
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          const uint32_t off = ((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4;
          umma_bf16_ss(tbase + t * 128, dq + off, dk + off, idS, kk > 0);
        }
        umma_commit(&sm.s_full[t]);
      };
      auto issue_PV = [&](int t, int j) {
        const int s = j % KV_STAGES;
        const uint64_t dp = umma_desc_kmajor_sw128(smem_u32(sm.p));
        const uint64_t dv = umma_desc_mnmajor_sw128(smem_u32(sm.v[s]), CHUNK);
#pragma unroll
        for (int kk = 0; kk < TILE / 16; kk++) {
          const uint32_t off = ((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4;
          umma_bf16_ss(tbase + 256 + t * 128, dp + off, dv + ((kk * 16 * 128) >> 4), idO, (j | kk) != 0);
        }
        umma_commit(&sm.o_done[t]);
        umma_commit(&sm.p_free[t]);
      };
      // per tile: next block whose S to issue (needs s_free of the block before), next P.V
      int sj[2] = {0, 0}, pj[2] = {0, 0};
      int s_cnt[KV_STAGES] = {0, 0}, v_cnt[KV_STAGES] = {0, 0};  // issues per stage of the current use
      const long long t0 = clock64();
      while (ok && (pj[0] < n_kv || (nt == 2 && pj[1] < n_kv))) {
        bool progress = false;
        for (int t = 0; t < nt; t++) {
          // S(sj): block 0 needs nothing but K; later blocks need the softmax to have read S(sj-1)
          if (sj[t] < n_kv) {
            const int j = sj[t];
            const bool free_ok = j == 0 || mbar_test_wait(smem_u32(&sm.s_free[t]), (j - 1) & 1);
            if (free_ok && mbar_test_wait(smem_u32(&sm.k_full[j % KV_STAGES]), (j / KV_STAGES) & 1)) {
              tc_fence_after();
              issue_S(t, j);
              sj[t]++;
              progress = true;
              if (++s_cnt[j % KV_STAGES] == nt) {
                umma_commit(&sm.k_empty[j % KV_STAGES]);
                s_cnt[j % KV_STAGES] = 0;
              }
            }
          }
          // P.V(pj): P in shared memory and V landed
          if (pj[t] < n_kv && pj[t] < sj[t]) {
            const int j = pj[t];
            if (mbar_test_wait(smem_u32(&sm.p_full[t]), j & 1) &&
                mbar_test_wait(smem_u32(&sm.v_full[j % KV_STAGES]), (j / KV_STAGES) & 1)) {
              tc_fence_after();
              issue_PV(t, j);
              pj[t]++;
              progress = true;
              if (++v_cnt[j % KV_STAGES] == nt) {
                umma_commit(&sm.v_empty[j % KV_STAGES]);
                v_cnt[j % KV_STAGES] = 0;
              }
            }
          }
        }
        if (!progress && (unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES * 4) {
          record_error(kErrWaitTimeout);
          ok = false;
        }
        if (!progress && error_raised()) ok = false;
      }
      if (!ok) {
        umma_commit(&sm.drain);
        spin_drain(&sm.drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qpos = q0 + t * TILE + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tbase + t * 128 + lane_off;
    const uint32_t tO = tbase + 256 + t * 128 + lane_off;
    const bool active = (t == 0) || has_b;
    uint8_t* prow = sm.p + r * 128;  // this thread's row in both 64-key chunks
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; active && j < n_kv; j++) {
      const int kbase = j * TILE;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool masked = (kbase + TILE > a.Sk) || (a.causal && kbase + TILE > q0 + t * TILE);
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld_32x32b_x32(tS + c * 32, v[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; c++) reg_fence32(v[c]);
      // S is in registers: the MMA warp may overwrite it with the next block's S right away
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free[t]);
      if (masked) {
        const int lim = min(a.Sk, a.causal ? qpos + 1 : a.Sk) - kbase;
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int e = 0; e < 32; e++)
            if (c * 32 + e >= lim) v[c][e] = 0xff800000u;
      }
      float mx;
      {
        float m0 = __uint_as_float(v[0][0]), m1 = __uint_as_float(v[1][0]);
        float m2 = __uint_as_float(v[2][0]), m3 = __uint_as_float(v[3][0]);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          m0 = max3(m0, __uint_as_float(v[0][e]), __uint_as_float(v[0][e + 1]));
          m1 = max3(m1, __uint_as_float(v[1][e]), __uint_as_float(v[1][e + 1]));
          m2 = max3(m2, __uint_as_float(v[2][e]), __uint_as_float(v[2][e + 1]));
          m3 = max3(m3, __uint_as_float(v[3][e]), __uint_as_float(v[3][e + 1]));
        }
        mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      }
      mx *= a.scale_log2;
      const bool need = (mx > m + RESCALE_THRESHOLD) || (m == -INFINITY);
      const bool rescale = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (rescale) {
        const float m_new = fmaxf(m, mx);
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      const float msub = (m == -INFINITY) ? 0.f : m;
      unsigned long long rsc[4] = {0ull, 0ull, 0ull, 0ull};
      const unsigned long long scale2 = f2pack(a.scale_log2, a.scale_log2);
      const unsigned long long negm2 = f2pack(-msub, -msub);
#pragma unroll
      for (int c = 0; c < 4; c++) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const unsigned long long x2 =
              fma2(f2pack(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])), scale2, negm2);
          float x0, x1;
          f2unpack(x2, x0, x1);
          float p0, p1;
          if (emu_pair<EMU>(i)) {
            const unsigned long long e2 = exp2_fma2(x0, x1);
            p0 = __uint_as_float((uint32_t)e2);
            p1 = __uint_as_float((uint32_t)(e2 >> 32));
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          rsc[i & 3] = add2(rsc[i & 3], f2pack(p0, p1));
          v[c][i] = pack_bf16x2(p0, p1);
        }
      }
      {
        float a0, a1, b0, b1;
        f2unpack(add2(rsc[0], rsc[1]), a0, a1);
        f2unpack(add2(rsc[2], rsc[3]), b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
      if (rescale && j > 0) {
        // O_t is quiescent once P.V(j-1) of this tile completed
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.o_done[t], (j - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int oc = 0; oc < 4; oc++) {
          uint32_t o[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
              "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
              : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3]), "=r"(o[4]), "=r"(o[5]), "=r"(o[6]), "=r"(o[7]),
                "=r"(o[8]), "=r"(o[9]), "=r"(o[10]), "=r"(o[11]), "=r"(o[12]), "=r"(o[13]), "=r"(o[14]),
                "=r"(o[15])
              : "r"(tO + oc * 32));
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x16(tO + oc * 32, o);
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
              "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
              : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3]), "=r"(o[4]), "=r"(o[5]), "=r"(o[6]), "=r"(o[7]),
                "=r"(o[8]), "=r"(o[9]), "=r"(o[10]), "=r"(o[11]), "=r"(o[12]), "=r"(o[13]), "=r"(o[14]),
                "=r"(o[15])
              : "r"(tO + oc * 32 + 16));
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x16(tO + oc * 32 + 16, o);
        }
        tmem_st_wait();
      }
      // the shared P buffer: the other tile's P.V of the previous turn must have read it
      // (tile A at block j waits for tile B's block j-1, tile B for tile A's block j)
      if (has_b) {
        const int other = t ^ 1;
        const int need_blk = t == 0 ? j - 1 : j;
        if (need_blk >= 0 && !__all_sync(0xffffffffu, mbar_wait(&sm.p_free[other], need_blk & 1))) {
          ok = false;
          break;
        }
      } else if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&sm.p_free[0], (j - 1) & 1))) {
        ok = false;
        break;
      }
      // P row: keys 8c..8c+7 -> 16-byte chunk c, 128-byte swizzle within each 64-key chunk
#pragma unroll
      for (int c = 0; c < 16; c++) {
        const uint4 w = make_uint4(v[c >> 2][(c & 3) * 4 + 0], v[c >> 2][(c & 3) * 4 + 1],
                                   v[c >> 2][(c & 3) * 4 + 2], v[c >> 2][(c & 3) * 4 + 3]);
        *reinterpret_cast<uint4*>(prow + (c >> 3) * CHUNK + (((c & 7) ^ (r & 7)) << 4)) = w;
      }
      fence_async_smem();  // generic-proxy stores -> visible to the tensor core's reads
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[t]);
    }
    if (active && ok && n_kv > 0 && __all_sync(0xffffffffu, mbar_wait(&sm.o_done[t], (n_kv - 1) & 1))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + c * 32, v);
        tmem_ld_wait();
        if (qpos < a.Sq) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[u * 8 + 0]) * inv, __uint_as_float(v[u * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[u * 8 + 2]) * inv, __uint_as_float(v[u * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[u * 8 + 4]) * inv, __uint_as_float(v[u * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[u * 8 + 6]) * inv, __uint_as_float(v[u * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(out + c * 32 + u * 8) = w;
          }
        }
      }
    } else if (active && n_kv == 0 && qpos < a.Sq) {
      __nv_bfloat16* out = a.o + (long long)b * a.o_batch + (long long)qpos * a.o_row + h * HD;
      for (int d = 0; d < HD; d++) out[d] = __float2bfloat16(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

bool make_tmap_3d(CUtensorMap* map, const void* base, int H, int S, int B, long long row_stride,
                  long long batch_stride) {
  // dims (inner->outer): head*dim columns, sequence rows, batch; box 64 x 128 x 1, 128-byte swizzle
  return make_tmap_3d_bf16(map, base, (uint64_t)H * HD, (uint64_t)S, (uint64_t)B, (uint64_t)row_stride,
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
  a.n_qblocks = (p.Sq + 2 * TILE - 1) / (2 * TILE);
  a.diag = p.diag_mode;
  a.trace = reinterpret_cast<unsigned long long*>(p.trace);
  if (p.diag_mode >= 200 && p.diag_mode <= 201) {  // experimental one-tile kernel (see attn1_fwd_kernel)
    a.n_qblocks = (p.Sq + TILE - 1) / TILE;
    a.diag = 0;
    const int smem1 = (int)sizeof(SmemOne) + 1024;
    const long long grid1 = (long long)a.n_qblocks * p.Hq * p.B;
    if (grid1 > 0x7fffffff) return cudaErrorInvalidValue;
    auto go1 = [&](auto kern) -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1);
      if (e != cudaSuccess) return e;
      kern<<<(int)grid1, NTHREADS1, smem1, stream>>>(tq, tk, tv, a);
      return cudaGetLastError();
    };
    return p.diag_mode == 200 ? go1(attn1_fwd_kernel<0>) : go1(attn1_fwd_kernel<1>);
  }
  if (p.diag_mode >= 400 && p.diag_mode <= 402) {  // P through shared memory (see attnP_fwd_kernel)
    a.diag = 0;
    const int smemP = (int)sizeof(SmemP) + 1024;
    const long long gridP = (long long)a.n_qblocks * p.Hq * p.B;
    if (gridP > 0x7fffffff) return cudaErrorInvalidValue;
    auto goP = [&](auto kern) -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smemP);
      if (e != cudaSuccess) return e;
      kern<<<(int)gridP, NTHREADS, smemP, stream>>>(tq, tk, tv, a);
      return cudaGetLastError();
    };
    return p.diag_mode == 400 ? goP(attnP_fwd_kernel<0>)
                              : (p.diag_mode == 401 ? goP(attnP_fwd_kernel<1>) : goP(attnP_fwd_kernel<2>));
  }
  if (p.diag_mode >= 300 && p.diag_mode <= 302) {  // split-row variant (see attn2x_fwd_kernel)
    a.diag = 0;
    const int smem2 = (int)sizeof(Smem2x) + 1024;
    const long long grid2 = (long long)a.n_qblocks * p.Hq * p.B;
    if (grid2 > 0x7fffffff) return cudaErrorInvalidValue;
    auto go2 = [&](auto kern) -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2);
      if (e != cudaSuccess) return e;
      kern<<<(int)grid2, NTHREADS2X, smem2, stream>>>(tq, tk, tv, a);
      return cudaGetLastError();
    };
    return p.diag_mode == 300 ? go2(attn2x_fwd_kernel<0>)
                              : (p.diag_mode == 301 ? go2(attn2x_fwd_kernel<1>) : go2(attn2x_fwd_kernel<2>));
  }
  const int smem = (int)sizeof(SmemBase) + 1024;
  const long long grid = (long long)a.n_qblocks * p.Hq * p.B;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  CpArgs none{};
  // diag_mode 100..104 (timing experiments only): run with that many exp2 pairs in 8 on the FMA pipe
  const int emu = (p.diag_mode >= 100 && p.diag_mode <= 104) ? p.diag_mode - 100 : 1;
  if (emu != 1) a.diag = 0;
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<(int)grid, NTHREADS, smem, stream>>>(tq, tk, tv, a, none);
    return cudaGetLastError();
  };
  switch (emu) {
    case 0:
      return go(attn_fwd_kernel<false, 0>);
    case 2:
      return go(attn_fwd_kernel<false, 2>);
    case 3:
      return go(attn_fwd_kernel<false, 3>);
    case 4:
      return go(attn_fwd_kernel<false, 4>);
    default: {
      static bool attr = false;
      if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr = true;
      }
      attn_fwd_kernel<false, 1><<<(int)grid, NTHREADS, smem, stream>>>(tq, tk, tv, a, none);
      return cudaGetLastError();
    }
  }
}

cudaError_t attention_cp_fwd(const AttnProblem& p, const AttnCpProblem& c, cudaStream_t stream) {
  if (p.B == 0 || p.Sq == 0) return cudaSuccess;
  if (p.Hq % p.Hk || p.causal) return cudaErrorInvalidValue;
  if (c.world < 1 || c.world > kCpMaxRanks || c.rank < 0 || c.rank >= c.world || c.shard_rows <= 0 ||
      (long long)c.world * c.shard_rows != p.Sk ||
      c.flags == nullptr || c.counters == nullptr)
    return cudaErrorInvalidValue;
  for (int r = 0; r < c.world; r++)
    if (c.peer_kv[r] == nullptr || (r != c.rank && c.peer_acks[r] == nullptr)) return cudaErrorInvalidValue;
  // K|V interleaved per token: row = [K (Hk*128) | V (Hk*128)] bf16, rows contiguous, batches contiguous
  const long long row_el = (long long)p.Hk * HD;  // [B, 2, Sk, Hk, 128]: K block, then V block
  const uint8_t* base = static_cast<const uint8_t*>(c.peer_kv[c.rank]);
  if (reinterpret_cast<uintptr_t>(base) & 255) return cudaErrorMisalignedAddress;
  CUtensorMap tq, tk, tv;
  if (!make_tmap_3d(&tq, p.q, p.Hq, p.Sq, p.B, p.q_row, p.q_batch)) return cudaErrorInvalidValue;
  if (!make_tmap_3d(&tk, base, p.Hk, p.Sk, p.B, row_el, 2 * row_el * p.Sk)) return cudaErrorInvalidValue;
  if (!make_tmap_3d(&tv, base + row_el * p.Sk * 2, p.Hk, p.Sk, p.B, row_el, 2 * row_el * p.Sk))
    return cudaErrorInvalidValue;
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
  a.causal = 0;
  a.n_qblocks = (p.Sq + 2 * TILE - 1) / (2 * TILE);
  a.diag = p.diag_mode;
  a.trace = reinterpret_cast<unsigned long long*>(p.trace);
  CpArgs k{};
  k.rank = c.rank;
  k.world = c.world;
  k.shard_rows = c.shard_rows;
  k.row_bytes = row_el * 2;
  k.part_bytes = k.row_bytes * p.Sk;
  k.batch_bytes = 2 * k.part_bytes;
  k.shard_bytes = k.row_bytes * c.shard_rows;
  for (int r = 0; r < c.world; r++) {
    k.peer_kv[r] = static_cast<const uint8_t*>(c.peer_kv[r]);
    k.peer_acks[r] = c.peer_acks[r];
  }
  k.local_kv = static_cast<uint8_t*>(c.peer_kv[c.rank]);
  k.flags = c.flags;
  k.flag_stride = c.flag_stride;
  k.epoch = c.epoch;
  k.claim = c.counters;
  k.done = c.counters + c.world;
  k.pieces_per_part = (int)((k.shard_bytes + CP_PIECE - 1) / CP_PIECE);
  k.pieces_per_batch = 2 * k.pieces_per_part;
  k.batches = p.B;
  cudaError_t e = cudaMemsetAsync(c.counters, 0, 2 * sizeof(unsigned int) * c.world, stream);
  if (e != cudaSuccess) return e;
  const int smem = (int)sizeof(SmemCP) + 1024;
  static bool attr = false;
  if (!attr) {
    e = cudaFuncSetAttribute(attn_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const long long grid = (long long)a.n_qblocks * p.Hq * p.B;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  attn_fwd_kernel<true><<<(int)grid, NTHREADS_CP, smem, stream>>>(tq, tk, tv, a, k);
  return cudaGetLastError();
}

}  // namespace ft
