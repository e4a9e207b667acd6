// Attention forward problem description (attention_sm100.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ft {

struct AttnProblem {
  int B = 0, Sq = 0, Sk = 0, Hq = 0, Hk = 0;  // [B, S, H, 128] tensors, heads packed
  const __nv_bfloat16* q = nullptr;
  const __nv_bfloat16* k = nullptr;
  const __nv_bfloat16* v = nullptr;
  __nv_bfloat16* o = nullptr;
  long long q_row = 0, k_row = 0, v_row = 0, o_row = 0;        // element stride between tokens
  long long q_batch = 0, k_batch = 0, v_batch = 0, o_batch = 0;  // element stride between batches
  float scale = 1.f;
  bool causal = false;
  int diag_mode = 0;
  void* trace = nullptr;  // debug only: uint64[12*64] clock64 timeline of CTA 0  // timing diagnostics only: 1 = no exp2, 2 = no softmax work (results invalid)
  int num_sms = 0;
};

cudaError_t attention_fwd(const AttnProblem& p, cudaStream_t stream);

// Context-parallel attention with the K/V all-gather fused in (see attention_sm100.cu).
constexpr int kCpMaxRanks = 8;
struct AttnCpProblem {
  int rank = 0, world = 1, shard_rows = 0;   // Sk == world * shard_rows
  void* peer_kv[kCpMaxRanks] = {};           // each rank's [B, 2, Sk, Hk, 128] bf16 buffer (K block, V block)
  const uint64_t* flags = nullptr;           // local: flags[q * flag_stride] = epoch rank q published
  int flag_stride = 1;
  uint64_t* peer_acks[kCpMaxRanks] = {};     // per peer p: the word that tells p we finished reading it
  uint64_t epoch = 0;
  unsigned int* counters = nullptr;          // 2 * world uint32 scratch, zeroed by the launcher
};
cudaError_t attention_cp_fwd(const AttnProblem& p, const AttnCpProblem& cp, cudaStream_t stream);

}  // namespace ft
