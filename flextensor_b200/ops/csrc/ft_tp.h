// Tensor-parallel fused collective GEMMs (tp_sm100.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ft {

constexpr int kTpMaxRanks = 8;

enum TpEpilogue : int {
  TP_EPI_NONE = 0,
  TP_EPI_BIAS = 1,
  TP_EPI_SWIGLU = 2,  // weight rows interleaved (gate_j, up_j): C[:, j] = silu(g_j) * u_j, N/2 outputs
  TP_EPI_BIAS_GELU = 3,  // tanh GELU of (acc + bias)
};

struct TpGemmProblem {
  int M = 0, N = 0, K = 0;     // M = all rows (world * rows per rank)
  int rank = 0, world = 1;
  const __nv_bfloat16* A = nullptr;  // reduce-scatter: local [M, K] input (lda)
  int lda = 0;
  const __nv_bfloat16* W = nullptr;  // [N, K] weight shard (ldw)
  int ldw = 0;
  const __nv_bfloat16* bias = nullptr;
  int epi = TP_EPI_NONE;
  // all-gather -> GEMM
  const void* peer_a[kTpMaxRanks] = {};  // each rank's full [M, K] A buffer (own rows written + published)
  __nv_bfloat16* C = nullptr;            // local output [M, N or N/2] (ldc)
  int ldc = 0;
  const uint64_t* flags = nullptr;       // local flags[q * flag_stride] = epoch rank q published
  int flag_stride = 1;
  uint64_t* peer_acks[kTpMaxRanks] = {}; // word telling rank p we finished reading its rows
  // GEMM -> reduce-scatter
  void* stage[kTpMaxRanks] = {};         // rank p's staging [world][M/world][N] for this slot
  uint64_t* peer_flags[kTpMaxRanks] = {};// word telling rank p our partial rows are complete
  uint64_t epoch = 0;
  unsigned int* counters = nullptr;      // scratch: tp_ag_counter_words (all-gather) / 1 (reduce-scatter), zeroed here
  int num_sms = 0;
  int pair = 0;  // experimental: 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2)
};

struct TpReduceProblem {
  int rank = 0, world = 1, rows = 0, N = 0;
  const void* stage = nullptr;           // local [world][rows][N]
  const void* residual = nullptr;        // optional [rows, N] (ldr)
  int ldr = 0;
  void* out = nullptr;                   // [rows, N] (ldo); may alias residual
  int ldo = 0;
  const uint64_t* flags = nullptr;       // local flags[q * flag_stride]
  int flag_stride = 1;
  uint64_t epoch = 0;
  uint64_t* peer_acks[kTpMaxRanks] = {}; // word telling rank q its slot in our staging is free
  int stage_rows = 0;                    // row stride of the staging slots (0: = rows)
  // all-reduce: write the reduced rows to every rank's output at row_base (instead of `out`);
  // the acknowledgements that follow then also mean "my rows are in your output"
  void* out_peers[kTpMaxRanks] = {};
  int out_peers_n = 0;
  long long row_base = 0;
  // out = residual + gate * (sum + bias): bias bf16 [N]; gate fp32 rows of gate_stride, one per
  // group of gate_rows consecutive global rows (global row = grow0 + local row)
  const __nv_bfloat16* bias = nullptr;
  const float* gate = nullptr;
  long long gate_stride = 0;
  int gate_rows = 0;
  long long grow0 = 0;
};

// RMSNorm over a hidden dimension split across tensor-parallel ranks (each rank holds D_local
// consecutive columns, whole heads): y = x * rsqrt(sum over all ranks of x^2 / D_full + eps) * w
// [then RoPE per head]. The per-row partial sums of squares travel over peer stores.
struct TpRmsProblem {
  int rank = 0, world = 1, rows = 0, D_local = 0, D_full = 0;
  const __nv_bfloat16* x = nullptr;
  int ldx = 0;
  __nv_bfloat16* y = nullptr;           // may alias x
  int ldy = 0;
  const void* weight = nullptr;         // [D_local] shard (fp32 or bf16), optional
  bool weight_bf16 = false;
  float eps = 1e-6f;
  const float* cos = nullptr;           // optional RoPE tables [seq_len, head_dim/2]
  const float* sin = nullptr;
  int head_dim = 0, seq_len = 0;
  float* part_peers[kTpMaxRanks] = {};  // rank q's partial-sum slot: [world][stage_rows] fp32
  const float* part_local = nullptr;    // this rank's slot
  int stage_rows = 0;                   // multiple of 32, >= rows
  uint64_t* peer_flags[kTpMaxRanks] = {};  // word on rank q: "our partials of this epoch are in"
  const uint64_t* flags = nullptr;      // local flags[q * flag_stride] = epoch rank q published
  int flag_stride = 1;
  uint64_t* peer_acks[kTpMaxRanks] = {};   // word on rank q: "its partials in our slot are read"
  uint64_t epoch = 0;
  unsigned int* counter = nullptr;      // scratch, zeroed here
  int phases = 3;                       // bit 0: sums of squares + publish; bit 1: wait, scale, acknowledge
};

// Scratch words the all-gather GEMM needs: per-peer claim and done tickets, plus per-peer byte
// counts of every 128-row block (none with a single rank).
inline int tp_ag_counter_words(int M, int world) {
  return world > 1 ? world * (2 + (M / world + 127) / 128) : 2 * world;
}

cudaError_t tp_allgather_gemm(const TpGemmProblem& g, cudaStream_t stream);
cudaError_t tp_gemm_reducescatter(const TpGemmProblem& g, cudaStream_t stream);
cudaError_t tp_reduce(const TpReduceProblem& r, cudaStream_t stream);
cudaError_t tp_rmsnorm(const TpRmsProblem& r, cudaStream_t stream);
int tp_device_error(bool reset);

}  // namespace ft
