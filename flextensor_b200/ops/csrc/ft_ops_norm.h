// Argument blocks of the row-wise normalisation kernels (norm.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ft {

struct LnArgs {
  const __nv_bfloat16* x = nullptr;
  int ldx = 0;
  __nv_bfloat16* y = nullptr;
  int ldy = 0;
  int D = 0;
  float eps = 1e-6f;
  const void* weight = nullptr;  // optional affine (fp32 or bf16, see affine_bf16)
  const void* bias = nullptr;
  bool affine_bf16 = false;
  const float* scale = nullptr;  // optional modulation, fp32 [rows/mod_rows, mod_stride]
  const float* shift = nullptr;
  int mod_rows = 0;              // rows sharing one modulation vector (0 = all rows)
  int mod_stride = 0;
};

struct RmsArgs {
  const __nv_bfloat16* x = nullptr;
  int ldx = 0;
  __nv_bfloat16* y = nullptr;
  int ldy = 0;
  int D = 0;
  float eps = 1e-6f;
  const void* weight = nullptr;
  bool weight_bf16 = false;
  const float* cos = nullptr;  // optional RoPE tables [seq_len, head_dim/2]
  const float* sin = nullptr;
  int head_dim = 0;
  int seq_len = 0;
  bool no_norm = false;  // rotary embedding only (no RMS scaling, no weight)
};

cudaError_t ln_modulate(const LnArgs& a, int rows, cudaStream_t st);
cudaError_t rmsnorm(const RmsArgs& a, int rows, cudaStream_t st);

}  // namespace ft
