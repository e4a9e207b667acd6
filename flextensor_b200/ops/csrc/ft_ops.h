// Host-side declarations of the flextensor_b200 native kernels and runtime.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ft {

enum Epilogue : int {
  EPI_NONE = 0,          // C = A.W^T
  EPI_BIAS = 1,          // C = A.W^T + b
  EPI_BIAS_GELU = 2,     // C = gelu_tanh(A.W^T + b)
  EPI_BIAS_GATE_RES = 3, // C = R + g * (A.W^T + b)        (g fp32 per column, per gate_rows rows)
  EPI_BIAS_RES = 4,      // C = R + (A.W^T + b)
};

struct GemmProblem {
  int M = 0, N = 0, K = 0;
  const __nv_bfloat16* A = nullptr;
  int lda = 0;
  const __nv_bfloat16* W = nullptr;
  int ldw = 0;
  __nv_bfloat16* C = nullptr;
  int ldc = 0;
  const __nv_bfloat16* bias = nullptr;
  const __nv_bfloat16* residual = nullptr;
  int ldr = 0;
  const float* gate = nullptr;
  int gate_rows = 0;
  int epi = EPI_NONE;
  int num_sms = 0;
  int force_bn = 0;   // 64/128/256: 1-SM tile width; 512: force the 2-SM 256x256 kernel
  bool pair_ok = false;  // allow the 2-SM kernel when the shape suits it
};

cudaError_t gemm_bf16(const GemmProblem& g, cudaStream_t stream);

// 2-D bf16 tensor map: inner extent `inner` (contiguous), `outer` rows with row
// stride `ld` elements; box = box_inner x box_outer; 128-byte swizzle when
// box_inner*2 == 128, zero fill out of bounds.
bool make_tmap_2d_bf16(CUtensorMap* map, const void* base, int inner, int outer, int ld, int box_inner,
                       int box_outer);
bool make_tmap_2d_bf16_swz(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                           int box_inner, int box_outer, int swizzle_bytes);

// 3-D bf16 tensor map (inner, rows, batches) with element strides; 128-byte swizzle box.
bool make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t batches,
                       uint64_t row_stride_elems, uint64_t batch_stride_elems, int box_inner, int box_rows);

// 4-D bf16 tensor map (d0 contiguous; d1..d3 with element strides s1..s3); box b0 x b1 x b2 x b3,
// 128-byte swizzle when b0*2 == 128, zero fill out of bounds.
bool make_tmap_4d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3,
                       uint64_t s1, uint64_t s2, uint64_t s3, int b0, int b1, int b2, int b3);

// Decode attention (decode_sm100.cu): q [B, Hq, 128] (one query per sequence) over a KV cache
// [B, L, Hk, 128] (token / batch strides in elements), keys [0, len_b) of sequence b.
struct DecodeProblem {
  int B = 0, Hq = 0, Hk = 0, L = 0;
  const __nv_bfloat16* q = nullptr;
  long long q_b = 0;
  const __nv_bfloat16* k = nullptr;
  const __nv_bfloat16* v = nullptr;
  long long k_tok = 0, k_batch = 0, v_tok = 0, v_batch = 0;
  __nv_bfloat16* o = nullptr;
  long long o_b = 0;
  const int* seqlens = nullptr;  // device [B]; null: every sequence has kv_len keys
  int kv_len = 0;
  int max_len = 0;               // upper bound of the lengths (host side)
  float scale = 1.f;
  int n_split = 1;
  float* scratch = nullptr;      // decode_scratch_floats(B, Hq, n_split) fp32 when n_split > 1
  long long q_elems = 0, o_elems = 0;  // extents of the q / o allocations (elements from q / o)
};
int decode_splits(int B, int Hk, int max_len, int num_sms);
size_t decode_scratch_floats(int B, int Hq, int n_split);
cudaError_t decode_attention(const DecodeProblem& p, cudaStream_t stream);
int decode_device_error(bool reset);

int gemm_device_error(bool reset);
int norm_device_error(bool reset);
int attn_device_error(bool reset);

}  // namespace ft
