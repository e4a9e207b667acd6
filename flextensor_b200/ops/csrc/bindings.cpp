// Python bindings of the native kernels and runtime (module ft_b200_C).
//
// Every op validates device, dtype, shape and stride before launching and
// launches on the caller's current CUDA stream; a failed launch raises.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "ft_attn.h"
#include "ft_ops.h"
#include "ft_ops_norm.h"
#include "ft_runtime.h"
#include "ft_tp.h"
#include "ft_moe.h"

namespace {

using at::Tensor;

void check_cuda_bf16(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit inner stride");
}

void check_ok(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

int num_sms_for(int dev) {
  static int cache[64] = {0};
  if (dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cache[dev] = n;
  return n;
}

void gemm(const Tensor& A, const Tensor& W, Tensor& C, const c10::optional<Tensor>& bias,
          const c10::optional<Tensor>& residual, const c10::optional<Tensor>& gate, int64_t gate_rows, int64_t epi,
          int64_t force_bn) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(W, "W");
  check_cuda_bf16(C, "C");
  TORCH_CHECK(A.size(1) == W.size(1), "K mismatch: A ", A.sizes(), " W ", W.sizes());
  TORCH_CHECK(C.size(0) == A.size(0) && C.size(1) == W.size(0), "C shape ", C.sizes(), " != [M, N]");
  TORCH_CHECK(A.get_device() == W.get_device() && A.get_device() == C.get_device(), "tensors on different devices");
  c10::cuda::CUDAGuard g(A.device());
  ft::GemmProblem p;
  p.M = A.size(0);
  p.N = W.size(0);
  p.K = A.size(1);
  p.A = reinterpret_cast<const __nv_bfloat16*>(A.data_ptr());
  p.lda = A.stride(0);
  p.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  p.ldw = W.stride(0);
  p.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
  p.ldc = C.stride(0);
  p.epi = (int)epi;
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->is_cuda() && bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() &&
                    bias->numel() == p.N, "bias must be contiguous bf16 [N]");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (residual && residual->defined()) {
    check_cuda_bf16(*residual, "residual");
    TORCH_CHECK(residual->size(0) == p.M && residual->size(1) == p.N, "residual must be [M, N]");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  if (gate && gate->defined()) {
    TORCH_CHECK(gate->is_cuda() && gate->scalar_type() == at::kFloat && gate->is_contiguous(),
                "gate must be contiguous fp32");
    TORCH_CHECK(gate->numel() % p.N == 0, "gate numel must be a multiple of N");
    if (gate_rows > 0) TORCH_CHECK((p.M + gate_rows - 1) / gate_rows * p.N <= gate->numel(), "gate too small");
    p.gate = gate->data_ptr<float>();
    p.gate_rows = (int)gate_rows;
  }
  p.num_sms = num_sms_for(A.get_device());
  p.force_bn = (int)force_bn;
  static const bool pair_env = [] {
    const char* e = std::getenv("FT_GEMM_2SM");
    return e == nullptr || e[0] != '0';  // 2-SM kernel by default; FT_GEMM_2SM=0 disables it
  }();
  p.pair_ok = pair_env;
  check_ok(ft::gemm_bf16(p, at::cuda::getCurrentCUDAStream()), "gemm_bf16");
}

const void* opt_ptr(const c10::optional<Tensor>& t) { return (t && t->defined()) ? t->data_ptr() : nullptr; }

void ln_modulate(const Tensor& x, Tensor& y, const c10::optional<Tensor>& weight, const c10::optional<Tensor>& bias,
                 const c10::optional<Tensor>& scale, const c10::optional<Tensor>& shift, int64_t mod_rows,
                 double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(y, "y");
  TORCH_CHECK(x.sizes() == y.sizes(), "x/y shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  ft::LnArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.ldy = y.stride(0);
  a.D = x.size(1);
  a.eps = (float)eps;
  if (weight && weight->defined()) {
    TORCH_CHECK(weight->numel() == a.D && weight->is_contiguous(), "weight must be [D]");
    a.weight = weight->data_ptr();
    a.affine_bf16 = weight->scalar_type() == at::kBFloat16;
    if (bias && bias->defined()) {
      TORCH_CHECK(bias->scalar_type() == weight->scalar_type() && bias->numel() == a.D, "bias must match weight");
      a.bias = bias->data_ptr();
    }
  }
  for (const c10::optional<Tensor>* t : {&scale, &shift}) {
    if (*t && (*t)->defined()) {
      TORCH_CHECK((*t)->scalar_type() == at::kFloat && (*t)->stride(-1) == 1, "scale/shift must be fp32 rows");
      TORCH_CHECK((*t)->size(-1) == a.D, "scale/shift last dim must be D");
    }
  }
  if (scale && scale->defined()) {
    a.scale = scale->data_ptr<float>();
    a.mod_stride = scale->dim() > 1 ? scale->stride(-2) : 0;
  }
  if (shift && shift->defined()) {
    a.shift = shift->data_ptr<float>();
    if (shift->dim() > 1) TORCH_CHECK(shift->stride(-2) == a.mod_stride || !a.scale, "scale/shift row strides differ");
    if (!a.scale) a.mod_stride = shift->dim() > 1 ? shift->stride(-2) : 0;
  }
  a.mod_rows = (int)mod_rows;
  check_ok(ft::ln_modulate(a, x.size(0), at::cuda::getCurrentCUDAStream()), "ln_modulate");
}

void rmsnorm(const Tensor& x, Tensor& y, const c10::optional<Tensor>& weight, const c10::optional<Tensor>& cos,
             const c10::optional<Tensor>& sin, int64_t head_dim, int64_t seq_len, double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(y, "y");
  TORCH_CHECK(x.sizes() == y.sizes(), "x/y shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  ft::RmsArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.ldy = y.stride(0);
  a.D = x.size(1);
  a.eps = (float)eps;
  a.no_norm = eps < 0;  // rope only
  if (weight && weight->defined()) {
    TORCH_CHECK(weight->numel() == a.D && weight->is_contiguous(), "weight must be [D]");
    a.weight = weight->data_ptr();
    a.weight_bf16 = weight->scalar_type() == at::kBFloat16;
  }
  if (cos && cos->defined()) {
    TORCH_CHECK(sin && sin->defined(), "sin table required with cos");
    TORCH_CHECK(cos->scalar_type() == at::kFloat && sin->scalar_type() == at::kFloat && cos->is_contiguous() &&
                    sin->is_contiguous(), "rope tables must be contiguous fp32");
    TORCH_CHECK(cos->numel() == seq_len * head_dim / 2 && sin->numel() == cos->numel(),
                "rope tables must be [seq_len, head_dim/2]");
    a.cos = cos->data_ptr<float>();
    a.sin = sin->data_ptr<float>();
    a.head_dim = (int)head_dim;
    a.seq_len = (int)seq_len;
  }
  check_ok(ft::rmsnorm(a, x.size(0), at::cuda::getCurrentCUDAStream()), "rmsnorm");
}

void attention(const Tensor& q, const Tensor& k, const Tensor& v, Tensor& o, double scale, bool causal,
               int64_t diag_mode, const c10::optional<Tensor>& trace) {
  for (const Tensor* p : {&q, &k, &v, const_cast<const Tensor*>(&o)}) {
    TORCH_CHECK(p->is_cuda() && p->scalar_type() == at::kBFloat16 && p->dim() == 4,
                "attention tensors must be 4-D bf16 CUDA [B, S, H, D]");
    TORCH_CHECK(p->stride(3) == 1, "head dim must be contiguous");
  }
  TORCH_CHECK(q.size(3) == 128 && k.size(3) == 128 && v.size(3) == 128, "head_dim 128 only");
  TORCH_CHECK(k.sizes() == v.sizes(), "k/v shape mismatch");
  TORCH_CHECK(q.size(0) == k.size(0) && q.sizes() == o.sizes(), "q/k/o batch or shape mismatch");
  TORCH_CHECK(q.size(2) % k.size(2) == 0, "query heads must be a multiple of kv heads");
  c10::cuda::CUDAGuard g(q.device());
  ft::AttnProblem p;
  p.B = q.size(0);
  p.Sq = q.size(1);
  p.Sk = k.size(1);
  p.Hq = q.size(2);
  p.Hk = k.size(2);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.q_row = q.stride(1);
  p.k_row = k.stride(1);
  p.v_row = v.stride(1);
  p.o_row = o.stride(1);
  p.q_batch = q.stride(0);
  p.k_batch = k.stride(0);
  p.v_batch = v.stride(0);
  p.o_batch = o.stride(0);
  TORCH_CHECK(q.stride(2) == 128 && k.stride(2) == 128 && v.stride(2) == 128 && o.stride(2) == 128,
              "heads must be packed (stride 128 between heads)");
  p.scale = (float)scale;
  p.causal = causal;
  p.diag_mode = (int)diag_mode;
  if (trace && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->numel() >= 20 * 64,
                "trace must be a CUDA int64 tensor with >= 1280 entries");
    p.trace = trace->data_ptr();
  }
  p.num_sms = num_sms_for(q.get_device());
  check_ok(ft::attention_fwd(p, at::cuda::getCurrentCUDAStream()), "attention_fwd");
}

// Context-parallel attention: q [B, Sq, Hq, 128] local queries, o like q; kv_local is this
// rank's [B, 2, Sk, Hk, 128] K/V buffer (own rows written and published before the call).
// q [B, Hq, 128] (or [B, 1, Hq, 128]), caches [B, L, Hk, 128] with packed heads; keys [0, len_b).
void decode_attention(const Tensor& q, const Tensor& kc, const Tensor& vc, Tensor& o,
                      const c10::optional<Tensor>& seqlens, int64_t kv_len, int64_t max_len, double scale,
                      int64_t n_split) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && o.scalar_type() == at::kBFloat16,
              "decode attention: bf16 CUDA q / out");
  TORCH_CHECK(kc.is_cuda() && vc.is_cuda() && kc.scalar_type() == at::kBFloat16 && vc.scalar_type() == at::kBFloat16 &&
                  kc.dim() == 4 && vc.dim() == 4 && kc.sizes() == vc.sizes(),
              "decode attention: k/v caches must be bf16 CUDA [B, L, Hk, 128] of one shape");
  const int64_t B = kc.size(0), L = kc.size(1), Hk = kc.size(2);
  TORCH_CHECK(kc.size(3) == 128 && kc.stride(3) == 1 && kc.stride(2) == 128 && vc.stride(3) == 1 && vc.stride(2) == 128,
              "caches: head_dim 128, contiguous, heads packed");
  const Tensor q3 = q.dim() == 4 ? q.squeeze(1) : q;
  const Tensor o3 = o.dim() == 4 ? o.squeeze(1) : o;
  TORCH_CHECK(q3.dim() == 3 && q3.size(0) == B && q3.size(2) == 128 && q3.stride(2) == 1 && q3.stride(1) == 128,
              "q must be [B, Hq, 128] with packed heads");
  TORCH_CHECK(o3.sizes() == q3.sizes() && o3.stride(2) == 1 && o3.stride(1) == 128, "out must match q");
  const int64_t Hq = q3.size(1);
  TORCH_CHECK(Hq % Hk == 0, "query heads must be a multiple of kv heads");
  TORCH_CHECK(max_len >= 0 && max_len <= L && kv_len >= 0 && kv_len <= L, "lengths must lie in [0, L]");
  c10::cuda::CUDAGuard g(q.device());
  ft::DecodeProblem p;
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hk = (int)Hk;
  p.L = (int)L;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q3.data_ptr());
  p.q_b = q3.stride(0);
  p.k = reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr());
  p.k_tok = kc.stride(1);
  p.k_batch = kc.stride(0);
  p.v_tok = vc.stride(1);
  p.v_batch = vc.stride(0);
  p.o = reinterpret_cast<__nv_bfloat16*>(o3.data_ptr());
  p.o_b = o3.stride(0);
  // reachable extents from the data pointers: the last sequence's last head row
  p.q_elems = (B - 1) * q3.stride(0) + Hq * 128;
  p.o_elems = (B - 1) * o3.stride(0) + Hq * 128;
  if (seqlens && seqlens->defined()) {
    TORCH_CHECK(seqlens->is_cuda() && seqlens->scalar_type() == at::kInt && seqlens->numel() == B &&
                    seqlens->is_contiguous(),
                "seqlens: int32 CUDA tensor with one length per sequence");
    p.seqlens = seqlens->data_ptr<int>();
  }
  p.kv_len = (int)kv_len;
  p.max_len = (int)(p.seqlens ? max_len : kv_len);
  p.scale = (float)scale;
  p.n_split = n_split > 0 ? (int)n_split : ft::decode_splits(p.B, p.Hk, p.max_len, num_sms_for(q.get_device()));
  Tensor scratch;
  if (p.n_split > 1) {
    scratch = at::empty({(int64_t)ft::decode_scratch_floats(p.B, p.Hq, p.n_split)},
                        q.options().dtype(at::kFloat));
    p.scratch = scratch.data_ptr<float>();
  }
  const cudaError_t e = ft::decode_attention(p, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == cudaSuccess, "decode_attention: ", cudaGetErrorString(e));
}

void attention_cp(const Tensor& q, const Tensor& kv_local, Tensor& o, double scale, std::vector<uint64_t> peer_kv,
                  uint64_t flags, int64_t flag_stride, std::vector<uint64_t> peer_acks, int64_t rank,
                  int64_t shard_rows, uint64_t epoch, Tensor& counters) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 4 && q.size(3) == 128 &&
                  q.stride(3) == 1 && q.stride(2) == 128, "q: [B, S, H, 128] bf16 CUDA, heads packed");
  TORCH_CHECK(o.sizes() == q.sizes() && o.stride(2) == 128 && o.stride(3) == 1, "o must match q");
  TORCH_CHECK(kv_local.is_cuda() && kv_local.scalar_type() == at::kBFloat16 && kv_local.dim() == 5 &&
                  kv_local.size(1) == 2 && kv_local.size(4) == 128 && kv_local.is_contiguous(),
              "kv_local: contiguous [B, 2, Sk, Hk, 128] bf16");
  const int world = (int)peer_kv.size();
  TORCH_CHECK(world >= 1 && world <= ft::kCpMaxRanks && (int)peer_acks.size() == world, "one kv/ack pointer per rank");
  TORCH_CHECK(peer_kv[rank] == reinterpret_cast<uint64_t>(kv_local.data_ptr()), "peer_kv[rank] must be kv_local");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= 2 * world,
              "counters: int32 CUDA tensor with 2*world entries");
  c10::cuda::CUDAGuard g(q.device());
  ft::AttnProblem p;
  p.B = q.size(0);
  p.Sq = q.size(1);
  p.Sk = kv_local.size(2);
  p.Hq = q.size(2);
  p.Hk = kv_local.size(3);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.q_row = q.stride(1);
  p.o_row = o.stride(1);
  p.q_batch = q.stride(0);
  p.o_batch = o.stride(0);
  p.scale = (float)scale;
  ft::AttnCpProblem c;
  c.rank = (int)rank;
  c.world = world;
  c.shard_rows = (int)shard_rows;
  for (int r = 0; r < world; r++) {
    c.peer_kv[r] = reinterpret_cast<void*>(peer_kv[r]);
    c.peer_acks[r] = reinterpret_cast<uint64_t*>(peer_acks[r]);
  }
  c.flags = reinterpret_cast<const uint64_t*>(flags);
  c.flag_stride = (int)flag_stride;
  c.epoch = epoch;
  c.counters = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  check_ok(ft::attention_cp_fwd(p, c, at::cuda::getCurrentCUDAStream()), "attention_cp_fwd");
}

// Epoch flags over peer memory (the CP and TP layers' signalling): publish stores `epoch` into
// flags[p][rank*n_slots + slot] of every rank p; wait_acks waits (bounded, on the device) until
// every peer's acks[rank][p*n_slots + slot] of this rank reached `epoch`.
static ft::PeerTable flag_table(const std::vector<uint64_t>& flags, const std::vector<uint64_t>& acks, int rank,
                                int n_slots) {
  const int world = (int)flags.size();
  TORCH_CHECK(world >= 1 && world <= ft::kMaxRanks && acks.size() == flags.size(), "one flag/ack array per rank");
  ft::PeerTable t;
  for (int p = 0; p < world; p++) {
    t.heap[p] = nullptr;
    t.flags[p] = reinterpret_cast<uint64_t*>(flags[p]);
    t.acks[p] = reinterpret_cast<uint64_t*>(acks[p]);
  }
  t.rank = rank;
  t.world = world;
  t.n_slots = n_slots;
  return t;
}

void p2p_publish_raw(std::vector<uint64_t> flags, std::vector<uint64_t> acks, int rank, int n_slots, int slot,
                     uint64_t epoch) {
  auto t = flag_table(flags, acks, rank, n_slots);
  check_ok(ft::p2p_publish(t, slot, epoch, at::cuda::getCurrentCUDAStream()), "p2p_publish");
}

void p2p_wait_acks_raw(std::vector<uint64_t> flags, std::vector<uint64_t> acks, int rank, int n_slots, int slot,
                       uint64_t epoch) {
  auto t = flag_table(flags, acks, rank, n_slots);
  check_ok(ft::p2p_wait_acks(t, slot, epoch, at::cuda::getCurrentCUDAStream()), "p2p_wait_acks");
}

// Tensor-parallel fused GEMMs. a_full: this rank's [M, K] buffer (own rows written + published);
// w: [N, K] shard; out: [M, N] (or [M, N/2] with SwiGLU). Pointers of peers come as integers.
void tp_ag_gemm(const Tensor& a_full, const Tensor& w, Tensor& out, const c10::optional<Tensor>& bias, int64_t epi,
                std::vector<uint64_t> peer_a, uint64_t flags, int64_t flag_stride, std::vector<uint64_t> peer_acks,
                int64_t rank, uint64_t epoch, Tensor& counters, bool pair) {
  TORCH_CHECK(a_full.is_cuda() && a_full.scalar_type() == at::kBFloat16 && a_full.dim() == 2 && a_full.is_contiguous(),
              "a_full: contiguous [M, K] bf16");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.stride(1) == 1, "w: [N, K] bf16");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.stride(1) == 1, "out: 2-D bf16");
  const int world = (int)peer_a.size();
  TORCH_CHECK(world >= 1 && world <= ft::kTpMaxRanks && (int)peer_acks.size() == world, "one pointer per rank");
  TORCH_CHECK(peer_a[rank] == reinterpret_cast<uint64_t>(a_full.data_ptr()), "peer_a[rank] must be a_full");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt &&
                  counters.numel() >= ft::tp_ag_counter_words((int)a_full.size(0), world),
              "counters: tp_ag_counter_words(M, world) int32 words");
  c10::cuda::CUDAGuard g(a_full.device());
  ft::TpGemmProblem p;
  p.M = a_full.size(0);
  p.K = a_full.size(1);
  p.N = w.size(0);
  p.rank = (int)rank;
  p.world = world;
  p.W = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.ldw = w.stride(0);
  if (bias && bias->defined()) p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  p.epi = (int)epi;
  TORCH_CHECK(out.size(0) == p.M && out.size(1) == (p.epi == ft::TP_EPI_SWIGLU ? p.N / 2 : p.N), "out shape");
  for (int r = 0; r < world; r++) {
    p.peer_a[r] = reinterpret_cast<const void*>(peer_a[r]);
    p.peer_acks[r] = reinterpret_cast<uint64_t*>(peer_acks[r]);
  }
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.flags = reinterpret_cast<const uint64_t*>(flags);
  p.flag_stride = (int)flag_stride;
  p.epoch = epoch;
  p.counters = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  p.num_sms = num_sms_for(a_full.get_device());
  p.pair = pair ? 1 : 0;
  check_ok(ft::tp_allgather_gemm(p, at::cuda::getCurrentCUDAStream()), "tp_allgather_gemm");
}

void tp_gemm_rs(const Tensor& a, const Tensor& w, std::vector<uint64_t> stage, std::vector<uint64_t> peer_flags,
                int64_t rank, uint64_t epoch, Tensor& counters, bool pair) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.dim() == 2 && a.stride(1) == 1, "a: [M, K] bf16");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.stride(1) == 1, "w: [N, K] bf16");
  const int world = (int)stage.size();
  TORCH_CHECK(world >= 1 && world <= ft::kTpMaxRanks && (int)peer_flags.size() == world, "one pointer per rank");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= 1, "counters");
  c10::cuda::CUDAGuard g(a.device());
  ft::TpGemmProblem p;
  p.M = a.size(0);
  p.K = a.size(1);
  p.N = w.size(0);
  p.rank = (int)rank;
  p.world = world;
  p.A = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
  p.lda = a.stride(0);
  p.W = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.ldw = w.stride(0);
  for (int r = 0; r < world; r++) {
    p.stage[r] = reinterpret_cast<void*>(stage[r]);
    p.peer_flags[r] = reinterpret_cast<uint64_t*>(peer_flags[r]);
  }
  p.epoch = epoch;
  p.counters = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  p.num_sms = num_sms_for(a.get_device());
  p.pair = pair ? 1 : 0;
  check_ok(ft::tp_gemm_reducescatter(p, at::cuda::getCurrentCUDAStream()), "tp_gemm_reducescatter");
}

void tp_reduce(const Tensor& stage, int64_t world, int64_t rows, Tensor& out, const c10::optional<Tensor>& residual,
               uint64_t flags, int64_t flag_stride, uint64_t epoch, std::vector<uint64_t> peer_acks, int64_t rank,
               std::vector<uint64_t> out_peers, int64_t row_base, int64_t stage_rows, const c10::optional<Tensor>& bias,
               const c10::optional<Tensor>& gate, int64_t gate_rows, int64_t grow0) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.stride(1) == 1, "out");
  c10::cuda::CUDAGuard g(out.device());
  ft::TpReduceProblem r;
  r.rank = (int)rank;
  r.world = (int)world;
  r.rows = (int)rows;
  r.N = out.size(1);
  r.stage = stage.data_ptr();
  if (residual && residual->defined()) {
    TORCH_CHECK(residual->stride(1) == 1 && residual->sizes() == out.sizes(), "residual like out");
    r.residual = residual->data_ptr();
    r.ldr = residual->stride(0);
  }
  r.out = out.data_ptr();
  r.ldo = out.stride(0);
  r.flags = reinterpret_cast<const uint64_t*>(flags);
  r.flag_stride = (int)flag_stride;
  r.epoch = epoch;
  TORCH_CHECK((int)peer_acks.size() == r.world, "one ack pointer per rank");
  for (int q = 0; q < r.world; q++) r.peer_acks[q] = reinterpret_cast<uint64_t*>(peer_acks[q]);
  r.stage_rows = (int)stage_rows;
  if (!out_peers.empty()) {
    TORCH_CHECK((int)out_peers.size() == r.world, "one output pointer per rank");
    for (int q = 0; q < r.world; q++) r.out_peers[q] = reinterpret_cast<void*>(out_peers[q]);
    r.out_peers_n = r.world;
    r.row_base = row_base;
  }
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == r.N, "bias: [N] bf16");
    r.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (gate && gate->defined()) {
    TORCH_CHECK(gate->scalar_type() == at::kFloat && gate->stride(-1) == 1 && gate->size(-1) == r.N,
                "gate: fp32 rows of N");
    TORCH_CHECK(gate_rows > 0, "gate_rows: rows per gate vector");
    r.gate = gate->data_ptr<float>();
    r.gate_stride = gate->dim() > 1 ? gate->stride(0) : 0;
    r.gate_rows = (int)gate_rows;
    r.grow0 = grow0;
  }
  check_ok(ft::tp_reduce(r, at::cuda::getCurrentCUDAStream()), "tp_reduce");
}

// Distributed RMSNorm over a column-sharded hidden dimension (optionally with RoPE). part_peers:
// every rank's fp32 partial slot [world][stage_rows] for this call; flags/acks as in tp_reduce.
void tp_rmsnorm(const Tensor& x, Tensor& y, const c10::optional<Tensor>& weight, const c10::optional<Tensor>& cos,
                const c10::optional<Tensor>& sin, int64_t head_dim, int64_t seq_len, double eps, int64_t d_full,
                std::vector<uint64_t> part_peers, int64_t stage_rows, std::vector<uint64_t> peer_flags, uint64_t flags,
                int64_t flag_stride, std::vector<uint64_t> peer_acks, int64_t rank, uint64_t epoch, Tensor& counter,
                int64_t phases) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x: [rows, D] bf16");
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.sizes() == x.sizes() && y.stride(1) == 1, "y like x");
  const int world = (int)part_peers.size();
  TORCH_CHECK(world >= 1 && world <= ft::kTpMaxRanks && (int)peer_flags.size() == world &&
                  (int)peer_acks.size() == world && rank >= 0 && rank < world, "one pointer per rank");
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt && counter.numel() >= 1, "counter");
  c10::cuda::CUDAGuard g(x.device());
  ft::TpRmsProblem r;
  r.rank = (int)rank;
  r.world = world;
  r.rows = x.size(0);
  r.D_local = x.size(1);
  r.D_full = (int)d_full;
  r.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  r.ldx = x.stride(0);
  r.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  r.ldy = y.stride(0);
  if (weight && weight->defined()) {
    TORCH_CHECK(weight->numel() == r.D_local && weight->is_contiguous(), "weight: [D_local]");
    TORCH_CHECK(weight->scalar_type() == at::kFloat || weight->scalar_type() == at::kBFloat16, "weight dtype");
    r.weight = weight->data_ptr();
    r.weight_bf16 = weight->scalar_type() == at::kBFloat16;
  }
  if (cos && cos->defined()) {
    TORCH_CHECK(sin && sin->defined() && cos->scalar_type() == at::kFloat && sin->scalar_type() == at::kFloat &&
                    cos->is_contiguous() && sin->is_contiguous() && cos->numel() == seq_len * head_dim / 2 &&
                    sin->numel() == cos->numel(), "rope tables: contiguous fp32 [seq_len, head_dim/2]");
    r.cos = cos->data_ptr<float>();
    r.sin = sin->data_ptr<float>();
    r.head_dim = (int)head_dim;
    r.seq_len = (int)seq_len;
  }
  r.eps = (float)eps;
  for (int q = 0; q < world; q++) {
    r.part_peers[q] = reinterpret_cast<float*>(part_peers[q]);
    r.peer_flags[q] = reinterpret_cast<uint64_t*>(peer_flags[q]);
    r.peer_acks[q] = reinterpret_cast<uint64_t*>(peer_acks[q]);
  }
  r.part_local = r.part_peers[rank];
  r.stage_rows = (int)stage_rows;
  r.flags = reinterpret_cast<const uint64_t*>(flags);
  r.flag_stride = (int)flag_stride;
  r.epoch = epoch;
  r.counter = reinterpret_cast<unsigned int*>(counter.data_ptr<int>());
  r.phases = (int)phases;
  check_ok(ft::tp_rmsnorm(r, at::cuda::getCurrentCUDAStream()), "tp_rmsnorm");
}

// Expert-parallel MoE expert GEMMs (dispatch = gate/up with the row pull, else down with the
// combine stores). Peer addresses arrive as integers; weights as one tensor per local expert.
void moe_gemm(bool dispatch, int64_t rank, int64_t local_experts, int64_t d, int64_t f, int64_t max_rows,
              std::vector<uint64_t> peer_send, std::vector<uint64_t> peer_table, uint64_t flags, int64_t flag_stride,
              std::vector<uint64_t> send_acks, Tensor& a_local, Tensor& h_local, std::vector<Tensor> weights,
              std::vector<uint64_t> peer_comb, std::vector<uint64_t> comb_flags, uint64_t epoch, Tensor& counters) {
  const int world = (int)peer_table.size();
  TORCH_CHECK(world >= 1 && world <= ft::kMoeMaxRanks, "1..8 ranks");
  TORCH_CHECK((int)weights.size() == local_experts, "one weight per local expert");
  TORCH_CHECK(a_local.is_cuda() && a_local.is_contiguous() && h_local.is_cuda() && h_local.is_contiguous(), "buffers");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= 2 * world + 1, "counters");
  c10::cuda::CUDAGuard g(a_local.device());
  ft::MoeProblem p;
  p.rank = (int)rank;
  p.world = world;
  p.local_experts = (int)local_experts;
  p.d = (int)d;
  p.f = (int)f;
  p.max_rows = (int)max_rows;
  for (int r = 0; r < world; r++) {
    p.peer_table[r] = reinterpret_cast<const int*>(peer_table[r]);
    if (dispatch) {
      p.peer_send[r] = reinterpret_cast<const void*>(peer_send.at(r));
      p.send_acks[r] = reinterpret_cast<uint64_t*>(send_acks.at(r));
    } else {
      p.peer_comb[r] = reinterpret_cast<void*>(peer_comb.at(r));
      p.comb_flags[r] = reinterpret_cast<uint64_t*>(comb_flags.at(r));
    }
  }
  for (int j = 0; j < (int)local_experts; j++) {
    const Tensor& w = weights[j];
    TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.is_contiguous(), "expert weights: contiguous bf16");
    if (dispatch) {
      TORCH_CHECK(w.size(0) == 2 * f && w.size(1) == d, "gate/up weight must be [2f, d]");
      p.w_gate_up[j] = w.data_ptr();
    } else {
      TORCH_CHECK(w.size(0) == d && w.size(1) == f, "down weight must be [d, f]");
      p.w_down[j] = w.data_ptr();
    }
  }
  p.flags = reinterpret_cast<const uint64_t*>(flags);
  p.flag_stride = (int)flag_stride;
  p.a_local = a_local.data_ptr();
  p.h_local = h_local.data_ptr();
  p.epoch = epoch;
  p.counters = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  p.num_sms = num_sms_for(a_local.get_device());
  auto st = at::cuda::getCurrentCUDAStream();
  check_ok(dispatch ? ft::moe_dispatch_gemm(p, st) : ft::moe_combine_gemm(p, st), "moe_gemm");
}

void moe_reduce(const Tensor& comb, const Tensor& pos, const Tensor& weight, const c10::optional<Tensor>& residual,
                Tensor& out, uint64_t flags, int64_t flag_stride, int64_t world, int64_t rank, uint64_t epoch) {
  TORCH_CHECK(pos.scalar_type() == at::kInt && weight.scalar_type() == at::kFloat && pos.is_contiguous() &&
                  weight.is_contiguous() && pos.sizes() == weight.sizes(), "pos int32 / weight fp32 [tokens, topk]");
  TORCH_CHECK(out.is_contiguous() && comb.is_contiguous(), "contiguous comb/out");
  c10::cuda::CUDAGuard g(out.device());
  ft::MoeCombineProblem p;
  p.tokens = pos.size(0);
  p.topk = pos.size(1);
  p.d = out.size(1);
  p.world = (int)world;
  p.rank = (int)rank;
  p.comb = comb.data_ptr();
  p.pos = pos.data_ptr<int>();
  p.weight = weight.data_ptr<float>();
  if (residual && residual->defined()) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == out.sizes(), "residual like out");
    p.residual = residual->data_ptr();
  }
  p.out = out.data_ptr();
  p.flags = reinterpret_cast<const uint64_t*>(flags);
  p.flag_stride = (int)flag_stride;
  p.epoch = epoch;
  check_ok(ft::moe_combine_reduce(p, at::cuda::getCurrentCUDAStream()), "moe_combine_reduce");
}

// Direct call of the striped gather with a caller-owned counter buffer (tests and tools).
void p2p_gather_raw(std::vector<uint64_t> heaps, std::vector<uint64_t> flags, std::vector<uint64_t> acks, int rank,
                    int n_slots, int slot, uint64_t epoch, uint64_t slot_offset, uint64_t stripe_bytes,
                    uint64_t total_bytes, const Tensor& counters, int ctas) {
  const int world = (int)heaps.size();
  TORCH_CHECK(world >= 1 && world <= ft::kMaxRanks && flags.size() == heaps.size() && acks.size() == heaps.size(),
              "one heap/flag/ack pointer per rank, at most ", ft::kMaxRanks);
  TORCH_CHECK(rank >= 0 && rank < world, "rank ", rank, " outside [0, ", world, ")");
  TORCH_CHECK(n_slots >= 1 && slot >= 0 && slot < n_slots, "slot ", slot, " outside [0, ", n_slots, ")");
  TORCH_CHECK(ctas >= 1, "ctas must be >= 1");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= n_slots,
              "counters: int32 CUDA tensor with one entry per slot");
  ft::PeerTable t;
  for (int p = 0; p < world; p++) {
    t.heap[p] = reinterpret_cast<uint8_t*>(heaps[p]);
    t.flags[p] = reinterpret_cast<uint64_t*>(flags[p]);
    t.acks[p] = reinterpret_cast<uint64_t*>(acks[p]);
  }
  t.rank = rank;
  t.world = world;
  t.n_slots = n_slots;
  c10::cuda::CUDAGuard g(counters.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const cudaError_t e = ft::p2p_gather(t, slot, epoch, slot_offset, stripe_bytes, total_bytes,
                                       reinterpret_cast<unsigned int*>(counters.data_ptr<int>()), ctas, s);
  TORCH_CHECK(e == cudaSuccess, "p2p_gather: ", cudaGetErrorString(e));
}

int device_error(bool reset) {
  int e = ft::gemm_device_error(reset);
  int n = ft::norm_device_error(reset);
  int a = ft::attn_device_error(reset);
  int p = ft::p2p_device_error(reset);
  int t = ft::tp_device_error(reset);
  int m = ft::moe_device_error(reset);
  int d = ft::decode_device_error(reset);
  return e ? e : (n ? n : (a ? a : (p ? p : (t ? t : (m ? m : d)))));
}

struct PyEngine {
  std::unique_ptr<ft::TransferEngine> e;
  int device;
  PyEngine(int dev, int n_slots, int n_keys, bool timing) : device(dev) {
    c10::cuda::CUDAGuard g(dev);
    e = std::make_unique<ft::TransferEngine>(dev, n_slots, n_keys, timing);
  }
  cudaStream_t cs() { return at::cuda::getCurrentCUDAStream(device).stream(); }
  void begin() { e->begin(cs()); }
  void submit(int slot, const Tensor& dst, const Tensor& src, int key) {
    TORCH_CHECK(dst.is_cuda() && src.device().is_cpu(), "submit copies host -> device");
    const size_t n = src.numel() * src.element_size();
    TORCH_CHECK(dst.numel() * dst.element_size() >= n, "destination slot too small");
    c10::cuda::CUDAGuard g(device);
    e->submit(slot, dst.data_ptr(), src.data_ptr(), n, key);
  }
  void wait_ready(int key) { e->wait_ready(key, cs()); }
  void finish_use(int slot) { e->finish_use(slot, cs()); }
  void join() { e->join(cs()); }
  void enable_striping(std::vector<uintptr_t> heaps, std::vector<uintptr_t> flags, std::vector<uintptr_t> acks,
                       int rank, int n_slots, std::vector<uint64_t> slot_offsets, uintptr_t counters, int ctas,
                       int gather_mode) {
    const int world = (int)heaps.size();
    TORCH_CHECK(world >= 1 && world <= ft::kMaxRanks, "world size must be in [1, 8]");
    TORCH_CHECK((int)flags.size() == world && (int)acks.size() == world, "per-rank pointer lists differ in length");
    ft::PeerTable t;
    for (int i = 0; i < world; i++) {
      t.heap[i] = reinterpret_cast<uint8_t*>(heaps[i]);
      t.flags[i] = reinterpret_cast<uint64_t*>(flags[i]);
      t.acks[i] = reinterpret_cast<uint64_t*>(acks[i]);
    }
    t.rank = rank;
    t.world = world;
    t.n_slots = n_slots;
    TORCH_CHECK(rank >= 0 && rank < world, "rank outside [0, world)");
    TORCH_CHECK(n_slots >= 1 && (int)slot_offsets.size() == n_slots, "one heap offset per slot");
    TORCH_CHECK(ctas >= 1, "ctas must be >= 1");
    e->enable_striping(t, slot_offsets, reinterpret_cast<unsigned int*>(counters), ctas, gather_mode);
  }
  // total_bytes < 0: src is the whole packed block. Otherwise src holds only this rank's
  // stripe of a packed block of total_bytes bytes.
  void submit_striped(int slot, const Tensor& src, int key, int64_t total_bytes) {
    TORCH_CHECK(src.device().is_cpu() && src.is_contiguous(), "striped submit copies a contiguous host block");
    c10::cuda::CUDAGuard g(device);
    const size_t held = src.numel() * src.element_size();
    if (total_bytes < 0) {
      e->submit_striped(slot, src.data_ptr(), held, key, false);
    } else {
      TORCH_CHECK(held >= e->stripe_bytes((size_t)total_bytes), "stripe buffer holds ", held, " bytes, needs ",
                  e->stripe_bytes((size_t)total_bytes));
      e->submit_striped(slot, src.data_ptr(), (size_t)total_bytes, key, true);
    }
  }
  size_t stripe_bytes(size_t total) const { return e->stripe_bytes(total); }
  void drain_striped() {
    c10::cuda::CUDAGuard g(device);
    e->drain_striped();
  }
  void synchronize() { e->synchronize(); }
  std::vector<std::tuple<int, float, float, float>> take_phase_samples() {
    std::vector<std::tuple<int, float, float, float>> out;
    for (auto& s : e->take_phase_samples()) out.emplace_back(s.key, s.acks_ms, s.h2d_ms, s.gather_ms);
    return out;
  }
  std::vector<std::tuple<int, size_t, float, float>> take_samples() {
    std::vector<std::tuple<int, size_t, float, float>> out;
    for (auto& s : e->take_samples()) out.emplace_back(s.key, s.bytes, s.transfer_ms, s.wait_ms);
    return out;
  }
};

}  // namespace

// Exact-size pinned host bytes: one portable cudaHostAlloc, released with cudaFreeHost when the
// last tensor (or view) over it goes away. torch's caching host allocator rounds each request up
// to a power of two, which for a 36 GB packed arena pins 64 GB of host memory.
at::Tensor pinned_empty(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "pinned_empty: nbytes must be positive, got ", nbytes);
  void* p = nullptr;
  const cudaError_t e = cudaHostAlloc(&p, static_cast<size_t>(nbytes), cudaHostAllocPortable);
  TORCH_CHECK(e == cudaSuccess, "cudaHostAlloc(", nbytes, " bytes) failed: ", cudaGetErrorString(e));
  return torch::from_blob(
      p, {nbytes}, [](void* q) { cudaFreeHost(q); }, at::TensorOptions().dtype(at::kByte).device(at::kCPU));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "flextensor_b200 native kernels (sm_100a) and runtime";
  m.def("gemm", &gemm, "tcgen05 GEMM C = epi(A W^T)", py::arg("A"), py::arg("W"), py::arg("C"),
        py::arg("bias") = py::none(), py::arg("residual") = py::none(), py::arg("gate") = py::none(),
        py::arg("gate_rows") = 0, py::arg("epi") = 0, py::arg("force_bn") = 0);
  m.def("ln_modulate", &ln_modulate, py::arg("x"), py::arg("y"), py::arg("weight") = py::none(),
        py::arg("bias") = py::none(), py::arg("scale") = py::none(), py::arg("shift") = py::none(),
        py::arg("mod_rows") = 0, py::arg("eps") = 1e-6);
  m.def("rmsnorm", &rmsnorm, py::arg("x"), py::arg("y"), py::arg("weight") = py::none(), py::arg("cos") = py::none(),
        py::arg("sin") = py::none(), py::arg("head_dim") = 0, py::arg("seq_len") = 0, py::arg("eps") = 1e-6);
  m.def("attention", &attention, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("scale"),
        py::arg("causal") = false, py::arg("diag_mode") = 0, py::arg("trace") = py::none());
  m.def("device_error", &device_error, py::arg("reset") = false);
  m.def("p2p_gather_raw", &p2p_gather_raw);
  m.def("attention_cp", &attention_cp);
  m.def("decode_attention", &decode_attention, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("out"),
        py::arg("seqlens"), py::arg("kv_len"), py::arg("max_len"), py::arg("scale"), py::arg("n_split") = 0);
  m.def("decode_splits", [](int B, int Hk, int max_len, int num_sms) { return ft::decode_splits(B, Hk, max_len, num_sms); });
  m.def("p2p_publish_raw", &p2p_publish_raw);
  m.def("tp_ag_gemm", &tp_ag_gemm, py::arg("a_full"), py::arg("w"), py::arg("out"), py::arg("bias"), py::arg("epi"),
        py::arg("peer_a"), py::arg("flags"), py::arg("flag_stride"), py::arg("peer_acks"), py::arg("rank"),
        py::arg("epoch"), py::arg("counters"), py::arg("pair") = false);
  m.def("tp_ag_counter_words", [](int64_t M, int64_t world) { return ft::tp_ag_counter_words((int)M, (int)world); });
  m.def("tp_gemm_rs", &tp_gemm_rs, py::arg("a"), py::arg("w"), py::arg("stage"), py::arg("peer_flags"),
        py::arg("rank"), py::arg("epoch"), py::arg("counters"), py::arg("pair") = false);
  m.def("tp_reduce", &tp_reduce, py::arg("stage"), py::arg("world"), py::arg("rows"), py::arg("out"),
        py::arg("residual"), py::arg("flags"), py::arg("flag_stride"), py::arg("epoch"), py::arg("peer_acks"),
        py::arg("rank"), py::arg("out_peers") = std::vector<uint64_t>{}, py::arg("row_base") = 0,
        py::arg("stage_rows") = 0, py::arg("bias") = py::none(), py::arg("gate") = py::none(),
        py::arg("gate_rows") = 0, py::arg("grow0") = 0);
  m.def("tp_rmsnorm", &tp_rmsnorm, py::arg("x"), py::arg("y"), py::arg("weight"), py::arg("cos"), py::arg("sin"),
        py::arg("head_dim"), py::arg("seq_len"), py::arg("eps"), py::arg("d_full"), py::arg("part_peers"),
        py::arg("stage_rows"), py::arg("peer_flags"), py::arg("flags"), py::arg("flag_stride"), py::arg("peer_acks"),
        py::arg("rank"), py::arg("epoch"), py::arg("counter"), py::arg("phases") = 3);
  m.def("moe_gemm", &moe_gemm);
  m.def("moe_reduce", &moe_reduce);
  m.def("p2p_wait_acks_raw", &p2p_wait_acks_raw);
  m.def("pinned_empty", &pinned_empty, py::arg("nbytes"));
  m.def("host_register", [](uintptr_t p, size_t n) { ft::host_register(reinterpret_cast<void*>(p), n); });
  m.def("host_unregister", [](uintptr_t p) { ft::host_unregister(reinterpret_cast<void*>(p)); });
  m.def("device_malloc", [](size_t n) { return reinterpret_cast<uintptr_t>(ft::device_malloc(n)); });
  m.def("device_free", [](uintptr_t p) { ft::device_free(reinterpret_cast<void*>(p)); });
  m.def("ipc_handle", [](uintptr_t p) { return py::bytes(ft::ipc_handle(reinterpret_cast<void*>(p))); });
  m.def("ipc_open", [](py::bytes h) { return reinterpret_cast<uintptr_t>(ft::ipc_open(std::string(h))); });
  m.def("ipc_close", [](uintptr_t p) { ft::ipc_close(reinterpret_cast<void*>(p)); });
  py::class_<PyEngine>(m, "TransferEngine")
      .def(py::init<int, int, int, bool>())
      .def("begin", &PyEngine::begin)
      .def("submit", &PyEngine::submit)
      .def("wait_ready", &PyEngine::wait_ready)
      .def("finish_use", &PyEngine::finish_use)
      .def("join", &PyEngine::join)
      .def("enable_striping", &PyEngine::enable_striping)
      .def("submit_striped", &PyEngine::submit_striped, py::arg("slot"), py::arg("src"), py::arg("key"),
           py::arg("total_bytes") = -1)
      .def("stripe_bytes", &PyEngine::stripe_bytes)
      .def("drain_striped", &PyEngine::drain_striped)
      .def("kernel_launches", [](const PyEngine& p) { return p.e->kernel_launches(); })
      .def("synchronize", &PyEngine::synchronize)
      .def("take_samples", &PyEngine::take_samples)
      .def("take_phase_samples", &PyEngine::take_phase_samples);
}
