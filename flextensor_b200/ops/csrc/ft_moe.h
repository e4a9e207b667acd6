// Expert-parallel MoE GEMMs with dispatch / combine fused in (moe_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ft {

constexpr int kMoeMaxRanks = 8;
constexpr int kMoeMaxLocalExperts = 8;

// Every rank is a token source and owns `local_experts` experts (global id rank*E_l + j).
// A source packs the rows it routes to expert e contiguously in its send buffer, in expert
// order, and publishes table = {cnt[E], off[E]} (int32) plus an epoch flag.
struct MoeProblem {
  int rank = 0, world = 1, local_experts = 1;
  int d = 0;          // model dim (gate/up K, down N)
  int f = 0;          // expert FFN width (down K; gate/up N = 2f, interleaved gate/up rows)
  int max_rows = 0;   // capacity of the expert-side row buffers (padded rows)
  // expert side
  const void* peer_send[kMoeMaxRanks] = {};     // each source's send buffer [rows, d]
  const int* peer_table[kMoeMaxRanks] = {};     // each source's {cnt[E], off[E]}
  const uint64_t* flags = nullptr;              // local: flags[q * flag_stride] = epoch source q published
  int flag_stride = 1;
  uint64_t* send_acks[kMoeMaxRanks] = {};       // word telling source p we finished pulling its rows
  void* a_local = nullptr;                      // [max_rows, d] gathered rows (expert groups padded to 128)
  void* h_local = nullptr;                      // [max_rows, f] SwiGLU activations
  const void* w_gate_up[kMoeMaxLocalExperts] = {};  // [2f, d] per local expert
  const void* w_down[kMoeMaxLocalExperts] = {};     // [d, f] per local expert
  void* peer_comb[kMoeMaxRanks] = {};           // each source's combine buffer [rows, d] (same rows as send)
  uint64_t* comb_flags[kMoeMaxRanks] = {};      // word telling source p our outputs for it are complete
  uint64_t epoch = 0;
  unsigned int* counters = nullptr;             // scratch: 2 * world + 1 entries, zeroed by the launchers
  int num_sms = 0;
};

// Gate/up GEMM pulling the routed rows (dispatch) + SwiGLU epilogue.
cudaError_t moe_dispatch_gemm(const MoeProblem& p, cudaStream_t stream);
// Down GEMM storing each output row into its source's combine buffer (combine) + flags.
cudaError_t moe_combine_gemm(const MoeProblem& p, cudaStream_t stream);

// Source side: out[t] = residual[t] + sum_k weight[t,k] * comb[pos[t,k]] after every expert
// rank flagged; then acknowledge (so experts may be refilled).
struct MoeCombineProblem {
  int tokens = 0, topk = 2, d = 0, world = 1, rank = 0;
  const void* comb = nullptr;        // [rows, d]
  const int* pos = nullptr;          // [tokens, topk] row of each (token, k) in comb
  const float* weight = nullptr;     // [tokens, topk]
  const void* residual = nullptr;    // [tokens, d] or null
  void* out = nullptr;               // [tokens, d] (may alias residual)
  const uint64_t* flags = nullptr;   // local comb flags[q * flag_stride] from expert rank q
  int flag_stride = 1;
  uint64_t epoch = 0;
};
cudaError_t moe_combine_reduce(const MoeCombineProblem& p, cudaStream_t stream);
int moe_device_error(bool reset);

}  // namespace ft
