// Attention forward problem description (attention_sm100.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

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

}  // namespace ft
