// Decode attention (one query per sequence over a KV cache), split over the keys
// ("flash-decoding"), GQA, head_dim 128, bf16, for sm_100a.
//
// A decode step reads every cached key and value once and does ~2 FLOPs per byte: the kernel is
// bound by HBM bandwidth. The G <= 16 query heads that share a KV head form the M side of the
// products (padded to 16 rows), far below the 64/128 rows of a tcgen05 tile, so the products use
// warp-level m16n8k16 MMAs with the query fragments held in registers for the whole CTA:
//   * grid = (key split, KV head, sequence); a CTA covers a contiguous run of 64-key tiles of one
//     sequence's cache for one KV head and all G query heads of that group, so each K/V byte is
//     read once per group;
//   * warp 4 (one elected lane) streams 32-key K and V tiles with 4-D tensor maps ([B, L, Hk,
//     128] cache, 128-byte swizzle, no multicast) into mbarrier-guarded stages; every consumer
//     warp owns two stages of its own, so a stage is only ever waited on by one warp, in order
//     (a phase-parity wait can then never see a phase two ahead of the one it means);
//   * warps 0-3 each take every 4th tile: S = Q K^T (K fragments by ldmatrix from the swizzled
//     tile), an online softmax on the accumulator fragments (row max / sum across the four lanes
//     of a row by shuffles, exp2 on MUFU), P re-packed in registers as the A operand, and
//     O += P V (V fragments by ldmatrix.trans); O stays in registers;
//   * the four warps' (O, max, sum) are merged in shared memory; one split writes bf16 output,
//     several write fp32 partials to a caller-provided scratch that decode_combine_kernel merges.
// Keys at or past a sequence's length are masked in S, and their V rows (possibly uninitialised
// cache memory) are zeroed in shared memory so 0 * NaN never reaches O. Every wait is bounded:
// a timeout records the device error word, the producer drains its own loads and the consumers
// fall through their remaining tiles without computing.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ft_ops.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(decode_device_error)

namespace {

constexpr int DHD = 128;              // head dim
constexpr int KT = 32;                // keys per tile
constexpr int NCW = 4;                // consumer warps
constexpr int SPW = 2;                // stages per consumer warp
constexpr int DSTAGES = NCW * SPW;
constexpr int DTHREADS = 32 * (NCW + 1);
constexpr int BOX_BYTES = KT * 128;   // one [32 keys x 64 dims] bf16 box (4 KB)
constexpr int STAGE_BYTES = 4 * BOX_BYTES;  // K (two boxes) + V (two boxes)

struct DecArgs {
  int B, Hq, Hk, L, G;         // L: cache capacity (tokens); G: query heads per KV head
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
  long long q_elems, o_elems;  // extents of q / o (elements) for the bounds checks below
};

// Global stores are bounds-checked against the extents the host passed (one compare each; they
// run once per output element, not in the key loop): an index outside records kErrBadArgs in
// the device error word and the access is skipped.
__device__ __forceinline__ bool in_range(long long i, long long n) {
  if (i >= 0 && i < n) return true;
  record_error(kErrBadArgs);
  return false;
}

struct DecSmem {
  uint8_t stage[DSTAGES][STAGE_BYTES];  // per stage: K box 0 | K box 1 | V box 0 | V box 1
  float wm[NCW][16], wl[NCW][16];       // per warp: row max / sum for the merge
  uint64_t full[DSTAGES], empty[DSTAGES];
};

// byte offset of 16-byte chunk `c` (0..15 over 128 dims) of row `r` in a [32 x 128] tile stored
// as two 128-byte-swizzled [32 x 64] boxes
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return (uint32_t)((c >> 3) * BOX_BYTES + r * 128 + (((c & 7) ^ (r & 7)) << 4));
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

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// D += A(16x16, row) * B(16x8, col), bf16 inputs, fp32 accumulators
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ldq2(const __nv_bfloat16* p, bool ok) {
  return ok ? *reinterpret_cast<const uint32_t*>(p) : 0u;
}

__global__ void __launch_bounds__(DTHREADS, 1)
    decode_split_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, DecArgs a) {
  extern __shared__ uint8_t smem_raw[];
  DecSmem& sm = *reinterpret_cast<DecSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int len = a.seqlens ? min(a.seqlens[b], a.L) : a.kv_len;
  const int t_begin = split * a.tiles_per_split;
  const int t_end = min(t_begin + a.tiles_per_split, (len + KT - 1) / KT);
  const int n_tiles = max(0, t_end - t_begin);

  if (tid == 0) {
    for (int s = 0; s < DSTAGES; s++) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);  // the consumer warp that used the stage
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t pend = 0, pph = 0;
      bool ok = true;
      for (int i = 0; i < n_tiles && ok; i++) {
        const int j = i / NCW;                      // use number of tile i's warp
        const int s = (i % NCW) * SPW + (j % SPW);  // that warp's stage
        const uint32_t ph = (j / SPW) & 1;
        if (!mbar_wait(&sm.empty[s], ph ^ 1)) {
          ok = false;
          break;
        }
        const int key0 = (t_begin + i) * KT;
        mbar_arrive_expect_tx(&sm.full[s], STAGE_BYTES);
        for (int c = 0; c < 2; c++) {
          tma_load_4d(sm.stage[s] + c * BOX_BYTES, &tmK, &sm.full[s], c * 64, hk, key0, b);
          tma_load_4d(sm.stage[s] + (2 + c) * BOX_BYTES, &tmV, &sm.full[s], c * 64, hk, key0, b);
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
    const int r0 = lane >> 2, cq = (lane & 3) * 2;  // accumulator rows r0 / r0+8, columns cq, cq+1
    // Q as A fragments for the 8 k-steps (rows = heads of the group, zero past G)
    uint32_t qa[8][4];
    {
      // rows past G are zero; their addresses are clamped to row 0 so no address past the
      // group (or past the end of q for the last group) is ever formed
      const long long qoff = (long long)b * a.q_b + (long long)hk * a.G * DHD;
      const bool ok0 = r0 < a.G, ok1 = r0 + 8 < a.G;
      const bool in0 = in_range(qoff + (ok0 ? r0 : 0) * DHD + DHD - 1, a.q_elems);
      const bool in1 = in_range(qoff + (ok1 ? r0 + 8 : 0) * DHD + DHD - 1, a.q_elems);
      const __nv_bfloat16* q0p = a.q + qoff + (ok0 ? r0 : 0) * DHD;
      const __nv_bfloat16* q1p = a.q + qoff + (ok1 ? r0 + 8 : 0) * DHD;
#pragma unroll
      for (int kk = 0; kk < 8; kk++) {
        qa[kk][0] = ldq2(q0p + kk * 16 + cq, ok0 && in0);
        qa[kk][1] = ldq2(q1p + kk * 16 + cq, ok1 && in1);
        qa[kk][2] = ldq2(q0p + kk * 16 + 8 + cq, ok0 && in0);
        qa[kk][3] = ldq2(q1p + kk * 16 + 8 + cq, ok1 && in1);
      }
    }
    float o[16][4];
#pragma unroll
    for (int dn = 0; dn < 16; dn++) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows r0, r0+8 (l: this lane's part)
    bool ok = true;
    for (int i = warp; i < n_tiles; i += NCW) {
      const int j = i / NCW;
      const int s = warp * SPW + (j % SPW);
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.full[s], (j / SPW) & 1));
      if (ok) {
        const int key0 = (t_begin + i) * KT;
        const int nvalid = min(KT, len - key0);
        const uint32_t kbase = smem_u32(sm.stage[s]);
        const uint32_t vbase = kbase + 2 * BOX_BYTES;
        if (nvalid < KT) {  // zero the V rows past the length (cache memory there may hold NaN)
          uint8_t* vt = sm.stage[s] + 2 * BOX_BYTES;
          for (int e = lane; e < (KT - nvalid) * 16; e += 32) {
            const int rr = nvalid + e / 16, c = e % 16;
            *reinterpret_cast<uint4*>(vt + tile_off(rr, c)) = make_uint4(0u, 0u, 0u, 0u);
          }
          __syncwarp();
        }
        // ---- S = Q K^T : 4 n-tiles of 8 keys
        float sc[4][4];
#pragma unroll
        for (int jn = 0; jn < 4; jn++) {
          sc[jn][0] = sc[jn][1] = sc[jn][2] = sc[jn][3] = 0.f;
          const int krow = jn * 8 + (lane & 7);
#pragma unroll
          for (int kp = 0; kp < 4; kp++) {  // k-step pairs: chunks 4kp .. 4kp+3
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kbase + tile_off(krow, 4 * kp + (lane >> 3)), b0, b1, b2, b3);
            mma16816(sc[jn], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], b0, b1);
            mma16816(sc[jn], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3], b2, b3);
          }
        }
        // ---- online softmax on the fragments (rows r0: sc[.][0..1], r0+8: sc[.][2..3])
        float tm0 = -INFINITY, tm1 = -INFINITY;
#pragma unroll
        for (int jn = 0; jn < 4; jn++) {
          const int k = jn * 8 + cq;
#pragma unroll
          for (int e = 0; e < 2; e++) {
            const bool v = k + e < nvalid;
            sc[jn][e] = v ? sc[jn][e] * a.scale_log2 : -INFINITY;
            sc[jn][2 + e] = v ? sc[jn][2 + e] * a.scale_log2 : -INFINITY;
            tm0 = fmaxf(tm0, sc[jn][e]);
            tm1 = fmaxf(tm1, sc[jn][2 + e]);
          }
        }
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 1));
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 2));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 1));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 2));
        const float n0 = fmaxf(m0, tm0), n1 = fmaxf(m1, tm1);
        const float s0 = n0 == -INFINITY ? 0.f : n0, s1 = n1 == -INFINITY ? 0.f : n1;
        const float al0 = m0 == -INFINITY ? 0.f : ex2f(m0 - s0), al1 = m1 == -INFINITY ? 0.f : ex2f(m1 - s1);
        m0 = n0;
        m1 = n1;
        l0 *= al0;
        l1 *= al1;
#pragma unroll
        for (int dn = 0; dn < 16; dn++) {
          o[dn][0] *= al0;
          o[dn][1] *= al0;
          o[dn][2] *= al1;
          o[dn][3] *= al1;
        }
        uint32_t pa[2][4];  // P as A fragments, one per 16-key k-step
#pragma unroll
        for (int jn = 0; jn < 4; jn++) {
          const float p0 = ex2f(sc[jn][0] - s0), p1 = ex2f(sc[jn][1] - s0);
          const float p2 = ex2f(sc[jn][2] - s1), p3 = ex2f(sc[jn][3] - s1);
          l0 += p0 + p1;
          l1 += p2 + p3;
          pa[jn >> 1][(jn & 1) * 2 + 0] = pack_bf16x2(p0, p1);
          pa[jn >> 1][(jn & 1) * 2 + 1] = pack_bf16x2(p2, p3);
        }
        // ---- O += P V : 16 n-tiles of 8 dims, 2 k-steps of 16 keys
#pragma unroll
        for (int kp = 0; kp < 2; kp++) {
          const int vrow = kp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
          for (int dp = 0; dp < 8; dp++) {  // dim n-tile pairs 2dp, 2dp+1
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vbase + tile_off(vrow, 2 * dp + (lane >> 4)), b0, b1, b2, b3);
            mma16816(o[2 * dp], pa[kp][0], pa[kp][1], pa[kp][2], pa[kp][3], b0, b1);
            mma16816(o[2 * dp + 1], pa[kp][0], pa[kp][1], pa[kp][2], pa[kp][3], b2, b3);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);
    }
    // ---- merge the four warps: row sums over the lanes of a row, then (O, m, l) across warps
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if ((lane & 3) == 0) {
      sm.wm[warp][r0] = m0;
      sm.wm[warp][r0 + 8] = m1;
      sm.wl[warp][r0] = l0;
      sm.wl[warp][r0 + 8] = l1;
    }
    // consumers only (the producer may still be draining): named barrier over the 4 warps
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NCW) : "memory");
    float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCW; w++) {
      M0 = fmaxf(M0, sm.wm[w][r0]);
      M1 = fmaxf(M1, sm.wm[w][r0 + 8]);
    }
    const float f0 = M0 == -INFINITY || m0 == -INFINITY ? 0.f : ex2f(m0 - M0);
    const float f1 = M1 == -INFINITY || m1 == -INFINITY ? 0.f : ex2f(m1 - M1);
    float L0 = 0.f, L1 = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; w++) {
      const float mw0 = sm.wm[w][r0], mw1 = sm.wm[w][r0 + 8];
      L0 += mw0 == -INFINITY ? 0.f : ex2f(mw0 - M0) * sm.wl[w][r0];
      L1 += mw1 == -INFINITY ? 0.f : ex2f(mw1 - M1) * sm.wl[w][r0 + 8];
    }
    // every warp's weighted O into its own slice red[warp][row][dim] (fp32, 8 KB per warp, in the
    // idle K/V stages: every load of this CTA landed and was consumed), rows >= G skipped; then
    // each output element is the sum of the four slices
    float* red = reinterpret_cast<float*>(sm.stage[0]);
    float* mine = red + warp * 16 * DHD;
    const bool w0 = r0 < a.G, w1 = r0 + 8 < a.G;
#pragma unroll
    for (int dn = 0; dn < 16; dn++) {
      const int d = dn * 8 + cq;
      if (w0) *reinterpret_cast<float2*>(&mine[r0 * DHD + d]) = make_float2(o[dn][0] * f0, o[dn][1] * f0);
      if (w1) *reinterpret_cast<float2*>(&mine[(r0 + 8) * DHD + d]) = make_float2(o[dn][2] * f1, o[dn][3] * f1);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NCW) : "memory");
    if (warp == 0 && (lane & 3) == 0) {  // the merged row statistics (every warp read wm/wl above)
      sm.wm[0][r0] = M0;
      sm.wm[0][r0 + 8] = M1;
      sm.wl[0][r0] = L0;
      sm.wl[0][r0 + 8] = L1;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NCW) : "memory");
    for (int e = tid; e < a.G * DHD; e += 32 * NCW) {
      const int g = e / DHD, d = e % DHD;
      const int hq = hk * a.G + g;
      float val = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; w++) val += red[(w * 16 + g) * DHD + d];
      if (a.n_split == 1) {
        const float L = sm.wl[0][g];
        const long long oi = (long long)b * a.o_b + (long long)hq * DHD + d;
        if (in_range(oi, a.o_elems)) a.o[oi] = __float2bfloat16(ok && L > 0.f ? val / L : 0.f);
      } else {
        const long long row = ((long long)split * a.B + b) * a.Hq + hq;
        const long long rows = (long long)a.n_split * a.B * a.Hq;
        if (!in_range(row, rows)) continue;
        a.part_o[row * DHD + d] = ok ? val : 0.f;
        if (d == 0) {
          a.part_ml[row * 2] = ok ? sm.wm[0][g] : -INFINITY;
          a.part_ml[row * 2 + 1] = ok ? sm.wl[0][g] : 0.f;
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
  const long long oi = (long long)b * a.o_b + (long long)hq * DHD + d;
  if (in_range(oi, a.o_elems)) a.o[oi] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

bool make_tmap_cache(CUtensorMap* map, const void* base, int Hk, int L, int B, long long tok_stride,
                     long long batch_stride) {
  return make_tmap_4d_bf16(map, base, DHD, (uint64_t)Hk, (uint64_t)L, (uint64_t)B, DHD, (uint64_t)tok_stride,
                           (uint64_t)batch_stride, 64, 1, KT, 1);
}

}  // namespace

int decode_splits(int B, int Hk, int max_len, int num_sms) {
  const int tiles = (max(max_len, 1) + KT - 1) / KT;
  const int base = max(1, B * Hk);
  // about one wave of CTAs: each split adds a partial row to write and a merge pass, which cost
  // more than a partly empty wave (B200, Llama-70B decode shape 32 x 2304, 8 KV heads: 1 split
  // 54.3 us, 2 splits 66.6 us, 4 splits 76.8 us); splits pay off when B * Hk is below the SM count
  int n = (max(num_sms, 1) + base - 1) / base;
  n = max(1, min(n, tiles / (4 * NCW)));              // at least four tiles per consumer warp
  return n;
}

size_t decode_scratch_floats(int B, int Hq, int n_split) {
  return n_split > 1 ? (size_t)n_split * B * Hq * (DHD + 2) : 0;
}

cudaError_t decode_attention(const DecodeProblem& p, cudaStream_t stream) {
  if (p.B == 0) return cudaSuccess;
  if (p.Hk <= 0 || p.Hq % p.Hk || p.L <= 0) return cudaErrorInvalidValue;
  const int G = p.Hq / p.Hk;
  if (G > 16) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(p.k) & 15) || (reinterpret_cast<uintptr_t>(p.v) & 15) ||
      (reinterpret_cast<uintptr_t>(p.q) & 3) || (p.q_b & 1))
    return cudaErrorMisalignedAddress;
  CUtensorMap tk, tv;
  if (!make_tmap_cache(&tk, p.k, p.Hk, p.L, p.B, p.k_tok, p.k_batch)) return cudaErrorInvalidValue;
  if (!make_tmap_cache(&tv, p.v, p.Hk, p.L, p.B, p.v_tok, p.v_batch)) return cudaErrorInvalidValue;
  DecArgs a;
  a.B = p.B;
  a.Hq = p.Hq;
  a.Hk = p.Hk;
  a.L = p.L;
  a.G = G;
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
  a.q_elems = p.q_elems;
  a.o_elems = p.o_elems;
  if (a.q_elems <= 0 || a.o_elems <= 0) return cudaErrorInvalidValue;
  a.part_o = p.scratch;
  a.part_ml = p.scratch ? p.scratch + (size_t)a.n_split * p.B * p.Hq * DHD : nullptr;
  if (a.n_split > 1 && p.scratch == nullptr) return cudaErrorInvalidValue;
  if (p.B > 65535 || p.Hk > 65535) return cudaErrorInvalidValue;
  const int smem = (int)sizeof(DecSmem) + 1024;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  decode_split_kernel<<<dim3(a.n_split, p.Hk, p.B), DTHREADS, smem, stream>>>(tk, tv, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.n_split == 1) return e;
  decode_combine_kernel<<<p.B * p.Hq, DHD, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace ft
