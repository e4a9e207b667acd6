// Native runtime pieces: TMA descriptor encoding, host-page registration and
// the ring-slot transfer engine (dedicated copy stream, per-slot "free" events,
// per-ticket "ready" events, optional timing events).
//
// The engine is the hot path of weight streaming: one call per trap boundary,
// each a handful of CUDA runtime calls with no Python objects involved. It is
// CUDA-graph aware: when the compute stream is capturing, events recorded
// before the capture are forgotten so every wait inside the graph refers to an
// event recorded in the same capture (cross-replay ordering is implied by
// graph launches on one stream).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "ft_ops.h"
#include "ft_runtime.h"

namespace ft {

// ------------------------------------------------------------------ TMA descriptors
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap_2d_bf16_swz(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                           int box_inner, int box_outer, int swizzle_bytes) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld_elems * 2) & 15)) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_2d_bf16(CUtensorMap* map, const void* base, int inner, int outer, int ld, int box_inner,
                       int box_outer) {
  return make_tmap_2d_bf16_swz(map, base, (uint64_t)inner, (uint64_t)outer, (uint64_t)ld, box_inner, box_outer,
                               box_inner * 2 == 128 ? 128 : 0);
}

bool make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t batches,
                       uint64_t row_stride_elems, uint64_t batch_stride_elems, int box_inner, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((row_stride_elems * 2) & 15) || ((batch_stride_elems * 2) & 15))
    return false;
  if (batches > 1 && batch_stride_elems == 0) return false;
  cuuint64_t dims[3] = {inner, rows, batches};
  cuuint64_t strides[2] = {row_stride_elems * 2, (batches > 1 ? batch_stride_elems : rows * row_stride_elems) * 2};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, box_inner * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                                      : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_4d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3,
                       uint64_t s1, uint64_t s2, uint64_t s3, int b0, int b1, int b2, int b3) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((s1 * 2) & 15) || ((s2 * 2) & 15) || ((s3 * 2) & 15)) return false;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1 * 2, s2 * 2, s3 * 2};
  cuuint32_t box[4] = {(cuuint32_t)b0, (cuuint32_t)b1, (cuuint32_t)b2, (cuuint32_t)b3};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, b0 * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------------ host registration
void host_register(void* ptr, size_t bytes) {
  cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterPortable);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaHostRegister failed: ") + cudaGetErrorString(e));
}

void host_unregister(void* ptr) {
  cudaError_t e = cudaHostUnregister(ptr);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaHostUnregister failed: ") + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ symmetric heap (CUDA IPC)
void* device_malloc(size_t bytes) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaMemset failed: ") + cudaGetErrorString(e));
  return p;
}

void device_free(void* p) { cudaFree(p); }

std::string ipc_handle(void* p) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcGetMemHandle failed: ") + cudaGetErrorString(e));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void* ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcOpenMemHandle failed: ") + cudaGetErrorString(e));
  return p;
}

void ipc_close(void* p) { cudaIpcCloseMemHandle(p); }

// ------------------------------------------------------------------ transfer engine
#define FT_CHECK(x)                                                                                \
  do {                                                                                             \
    cudaError_t _e = (x);                                                                          \
    if (_e != cudaSuccess) throw std::runtime_error(std::string(#x " failed: ") + cudaGetErrorString(_e)); \
  } while (0)

TransferEngine::TransferEngine(int device, int n_slots, int n_keys, bool timing)
    : device_(device), timing_(timing) {
  int prev;
  FT_CHECK(cudaGetDevice(&prev));
  FT_CHECK(cudaSetDevice(device));
  int lo, hi;
  FT_CHECK(cudaDeviceGetStreamPriorityRange(&lo, &hi));
  FT_CHECK(cudaStreamCreateWithPriority(&copy_, cudaStreamNonBlocking, hi));
  slot_free_.resize(n_slots);
  slot_recorded_.assign(n_slots, 0);
  ready_.resize(n_keys);
  ready_recorded_.assign(n_keys, 0);
  for (auto& e : slot_free_) FT_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  for (auto& e : ready_) FT_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  FT_CHECK(cudaEventCreateWithFlags(&fork_, cudaEventDisableTiming));
  FT_CHECK(cudaEventCreateWithFlags(&join_, cudaEventDisableTiming));
  if (timing_) {
    t_start_.resize(n_keys);
    t_end_.resize(n_keys);
    w_start_.resize(n_keys);
    w_end_.resize(n_keys);
    for (int i = 0; i < n_keys; i++) {
      FT_CHECK(cudaEventCreate(&t_start_[i]));
      FT_CHECK(cudaEventCreate(&t_end_[i]));
      FT_CHECK(cudaEventCreate(&w_start_[i]));
      FT_CHECK(cudaEventCreate(&w_end_[i]));
    }
    bytes_.assign(n_keys, 0);
    t_valid_.assign(n_keys, 0);
    w_valid_.assign(n_keys, 0);
  }
  cudaSetDevice(prev);
}

TransferEngine::~TransferEngine() {
  int prev;
  if (cudaGetDevice(&prev) != cudaSuccess) return;
  cudaSetDevice(device_);
  cudaStreamSynchronize(copy_);
  for (auto e : slot_free_) cudaEventDestroy(e);
  for (auto e : ready_) cudaEventDestroy(e);
  for (auto* v : {&t_start_, &t_end_, &w_start_, &w_end_, &ph_acked_, &ph_h2d_})
    for (auto e : *v) cudaEventDestroy(e);
  cudaEventDestroy(fork_);
  cudaEventDestroy(join_);
  cudaStreamDestroy(copy_);
  cudaSetDevice(prev);
}

void TransferEngine::begin(cudaStream_t compute) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  FT_CHECK(cudaStreamIsCapturing(compute, &st));
  const bool capturing = st != cudaStreamCaptureStatusNone;
  if (capturing != capturing_) {
    // entering or leaving a capture: events recorded on the other side are not waitable
    std::fill(slot_recorded_.begin(), slot_recorded_.end(), 0);
    std::fill(ready_recorded_.begin(), ready_recorded_.end(), 0);
    capturing_ = capturing;
  }
  FT_CHECK(cudaEventRecord(fork_, compute));
  FT_CHECK(cudaStreamWaitEvent(copy_, fork_, 0));
}

void TransferEngine::submit(int slot, void* dst, const void* src, size_t bytes, int key) {
  if (slot_recorded_[slot]) FT_CHECK(cudaStreamWaitEvent(copy_, slot_free_[slot], 0));
  const bool t = timing_ && !capturing_;
  if (t) FT_CHECK(cudaEventRecord(t_start_[key], copy_));
  FT_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, copy_));
  FT_CHECK(cudaEventRecord(ready_[key], copy_));
  ready_recorded_[key] = 1;
  if (t) {
    FT_CHECK(cudaEventRecord(t_end_[key], copy_));
    bytes_[key] = bytes;
    t_valid_[key] = 1;
  }
}

void TransferEngine::wait_ready(int key, cudaStream_t compute) {
  if (!ready_recorded_[key]) return;
  const bool t = timing_ && !capturing_;
  if (t) FT_CHECK(cudaEventRecord(w_start_[key], compute));
  FT_CHECK(cudaStreamWaitEvent(compute, ready_[key], 0));
  if (t) {
    FT_CHECK(cudaEventRecord(w_end_[key], compute));
    w_valid_[key] = 1;
  }
}

void TransferEngine::finish_use(int slot, cudaStream_t compute) {
  FT_CHECK(cudaEventRecord(slot_free_[slot], compute));
  slot_recorded_[slot] = 1;
}

void TransferEngine::join(cudaStream_t compute) {
  FT_CHECK(cudaEventRecord(join_, copy_));
  FT_CHECK(cudaStreamWaitEvent(compute, join_, 0));
}

void TransferEngine::synchronize() { FT_CHECK(cudaStreamSynchronize(copy_)); }

void TransferEngine::enable_striping(const PeerTable& t, const std::vector<uint64_t>& slot_offsets,
                                     unsigned int* counters, int gather_ctas, int gather_mode) {
  if (gather_mode != 0 && gather_mode != 1) throw std::runtime_error("gather_mode must be 0 (SM) or 1 (copy engine)");
  peers_ = t;
  slot_offsets_ = slot_offsets;
  epochs_.assign(slot_offsets.size(), 0);
  counters_ = counters;
  gather_ctas_ = gather_ctas;
  gather_mode_ = gather_mode;
  striped_ = t.world > 1;
  if (timing_ && ph_acked_.empty()) {
    int prev;
    FT_CHECK(cudaGetDevice(&prev));
    FT_CHECK(cudaSetDevice(device_));
    ph_acked_.resize(t_start_.size());
    ph_h2d_.resize(t_start_.size());
    ph_valid_.assign(t_start_.size(), 0);
    for (auto& e : ph_acked_) FT_CHECK(cudaEventCreate(&e));
    for (auto& e : ph_h2d_) FT_CHECK(cudaEventCreate(&e));
    cudaSetDevice(prev);
  }
}

void TransferEngine::drain_striped() {
  if (!striped_) return;
  for (size_t slot = 0; slot < epochs_.size(); slot++)
    if (epochs_[slot] > 0) FT_CHECK(p2p_wait_acks(peers_, (int)slot, epochs_[slot], copy_));
  FT_CHECK(cudaStreamSynchronize(copy_));
}

size_t TransferEngine::stripe_len(size_t total) const {
  const size_t W = (size_t)std::max(1, peers_.world);
  return ((total + W - 1) / W + 255) / 256 * 256;
}

size_t TransferEngine::stripe_bytes(size_t total) const {
  const size_t s = stripe_len(total);
  const size_t b0 = std::min<size_t>((size_t)peers_.rank * s, total);
  return std::min<size_t>(b0 + s, total) - b0;
}

void TransferEngine::submit_striped(int slot, const void* host_src, size_t bytes, int key, bool stripe_only) {
  if (!striped_) throw std::runtime_error("submit_striped without enable_striping");
  if (slot_recorded_[slot]) FT_CHECK(cudaStreamWaitEvent(copy_, slot_free_[slot], 0));
  const uint64_t epoch = ++epochs_[slot];
  const bool t = timing_ && !capturing_;
  if (t) FT_CHECK(cudaEventRecord(t_start_[key], copy_));
  // peers must have finished reading this slot's previous contents (our stripe) before we overwrite it
  FT_CHECK(p2p_wait_acks(peers_, slot, epoch - 1, copy_));
  const bool ph = t && !ph_acked_.empty();
  if (ph) FT_CHECK(cudaEventRecord(ph_acked_[key], copy_));
  const int r = peers_.rank;
  const uint64_t stripe = stripe_len(bytes);
  const uint64_t b0 = std::min<uint64_t>((uint64_t)r * stripe, bytes);
  const uint64_t b1 = std::min<uint64_t>(b0 + stripe, bytes);
  uint8_t* dst = peers_.heap[r] + slot_offsets_[slot];
  if (b1 > b0)
    FT_CHECK(cudaMemcpyAsync(dst + b0, static_cast<const uint8_t*>(host_src) + (stripe_only ? 0 : b0), b1 - b0,
                             cudaMemcpyHostToDevice, copy_));
  if (ph) FT_CHECK(cudaEventRecord(ph_h2d_[key], copy_));
  FT_CHECK(p2p_publish(peers_, slot, epoch, copy_));
  if (gather_mode_ == 0) {
    kernel_launches_ += (epoch > 1) ? 3 : 2;  // [wait_acks], publish, gather
    FT_CHECK(p2p_gather(peers_, slot, epoch, slot_offsets_[slot], stripe, bytes, counters_, gather_ctas_, copy_));
  } else {
    // copy engine: wait for every peer's stripe, DMA each one over NVLink, acknowledge
    kernel_launches_ += (epoch > 1) ? 4 : 3;  // [wait_acks], publish, wait_flags, ack
    FT_CHECK(p2p_wait_flags(peers_, slot, epoch, copy_));
    for (int pi = 1; pi < peers_.world; pi++) {
      const int p = (r + pi) % peers_.world;  // staggered like the SM gather
      const uint64_t c0 = std::min<uint64_t>((uint64_t)p * stripe, bytes);
      const uint64_t c1 = std::min<uint64_t>(c0 + stripe, bytes);
      if (c1 > c0)
        FT_CHECK(cudaMemcpyAsync(dst + c0, peers_.heap[p] + slot_offsets_[slot] + c0, c1 - c0,
                                 cudaMemcpyDeviceToDevice, copy_));
    }
    FT_CHECK(p2p_ack(peers_, slot, epoch, copy_));
  }
  if (ph) ph_valid_[key] = 1;
  FT_CHECK(cudaEventRecord(ready_[key], copy_));
  ready_recorded_[key] = 1;
  if (t) {
    FT_CHECK(cudaEventRecord(t_end_[key], copy_));
    bytes_[key] = bytes;
    t_valid_[key] = 1;
  }
}

// Moves the phase timings of key k (whose transfer events are valid) into phase_pending_.
void TransferEngine::collect_phase(size_t k) {
  if (k >= ph_valid_.size() || !ph_valid_[k]) return;
  PhaseSample s;
  s.key = (int)k;
  FT_CHECK(cudaEventSynchronize(t_end_[k]));
  FT_CHECK(cudaEventElapsedTime(&s.acks_ms, t_start_[k], ph_acked_[k]));
  FT_CHECK(cudaEventElapsedTime(&s.h2d_ms, ph_acked_[k], ph_h2d_[k]));
  FT_CHECK(cudaEventElapsedTime(&s.gather_ms, ph_h2d_[k], t_end_[k]));
  phase_pending_.push_back(s);
  ph_valid_[k] = 0;
}

std::vector<PhaseSample> TransferEngine::take_phase_samples() {
  if (!ph_valid_.empty()) {
    FT_CHECK(cudaStreamSynchronize(copy_));
    for (size_t k = 0; k < ph_valid_.size(); k++)
      if (t_valid_[k]) collect_phase(k);
  }
  std::vector<PhaseSample> out;
  out.swap(phase_pending_);
  return out;
}

std::vector<TransferSample> TransferEngine::take_samples() {
  std::vector<TransferSample> out;
  if (!timing_) return out;
  FT_CHECK(cudaStreamSynchronize(copy_));
  for (size_t k = 0; k < t_valid_.size(); k++) {
    if (!t_valid_[k]) continue;
    TransferSample s;
    s.key = (int)k;
    s.bytes = bytes_[k];
    FT_CHECK(cudaEventSynchronize(t_end_[k]));
    FT_CHECK(cudaEventElapsedTime(&s.transfer_ms, t_start_[k], t_end_[k]));
    if (w_valid_[k]) {
      FT_CHECK(cudaEventSynchronize(w_end_[k]));
      FT_CHECK(cudaEventElapsedTime(&s.wait_ms, w_start_[k], w_end_[k]));
    }
    out.push_back(s);
    collect_phase(k);  // before the transfer events are recycled
    t_valid_[k] = 0;
    w_valid_[k] = 0;
  }
  return out;
}

}  // namespace ft
