// Native transfer engine and host-memory helpers (runtime.cpp).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <string>
#include <vector>

#include "ft_p2p.h"

namespace ft {

void host_register(void* ptr, size_t bytes);
void host_unregister(void* ptr);

struct TransferSample {
  int key = 0;
  size_t bytes = 0;
  float transfer_ms = 0.f;
  float wait_ms = 0.f;
};

// Striped transfers, per phase on the copy stream (timing mode only): waiting for the peers'
// acknowledgements of the slot's previous epoch, this rank's H2D stripe, and the gather of the
// peers' stripes (including the wait for their publish flags).
struct PhaseSample {
  int key = 0;
  float acks_ms = 0.f;
  float h2d_ms = 0.f;
  float gather_ms = 0.f;
};

// Symmetric heap: cudaMalloc'd on this device, exported with CUDA IPC.
void* device_malloc(size_t bytes);
void device_free(void* p);
std::string ipc_handle(void* p);
void* ipc_open(const std::string& handle);
void ipc_close(void* p);

class TransferEngine {
 public:
  TransferEngine(int device, int n_slots, int n_keys, bool timing);
  ~TransferEngine();
  void begin(cudaStream_t compute);
  void submit(int slot, void* dst, const void* src, size_t bytes, int key);
  void wait_ready(int key, cudaStream_t compute);
  void finish_use(int slot, cudaStream_t compute);
  void join(cudaStream_t compute);
  void synchronize();
  std::vector<TransferSample> take_samples();
  cudaStream_t copy_stream() const { return copy_; }
  // Striped mode: slot `s` lives at heap offset slot_offsets[s] of every rank's symmetric heap;
  // submit() then copies only this rank's stripe and gathers the others from peers.
  // gather_mode 0: the SM pull kernel (gather_ctas CTAs); 1: copy engine (one cudaMemcpyAsync
  // per peer stripe between a bounded flag-wait kernel and an ack kernel).
  void enable_striping(const PeerTable& t, const std::vector<uint64_t>& slot_offsets, unsigned int* counters,
                       int gather_ctas, int gather_mode = 0);
  std::vector<PhaseSample> take_phase_samples();
  // host_src is the whole packed block, or (stripe_only) just this rank's stripe of it.
  void submit_striped(int slot, const void* host_src, size_t bytes, int key, bool stripe_only);
  // Wait (bounded, on the copy stream) until every peer acknowledged the latest epoch of every
  // slot, i.e. finished reading this rank's stripes; then synchronize. Call before freeing the heap.
  void drain_striped();
  // Kernels this engine launched (striped publish / wait / gather), for launch accounting.
  uint64_t kernel_launches() const { return kernel_launches_; }
  // Bytes of the stripe this rank holds for a packed block of `total` bytes (0 past the end).
  size_t stripe_bytes(size_t total) const;
  // Stripe length for a packed block of `total` bytes: ceil(total / world) rounded up to 256.
  size_t stripe_len(size_t total) const;

 private:
  int device_;
  bool timing_;
  bool capturing_ = false;
  cudaStream_t copy_ = nullptr;
  cudaEvent_t fork_ = nullptr, join_ = nullptr;
  std::vector<cudaEvent_t> slot_free_, ready_;
  std::vector<char> slot_recorded_, ready_recorded_;
  std::vector<cudaEvent_t> t_start_, t_end_, w_start_, w_end_;
  std::vector<size_t> bytes_;
  std::vector<char> t_valid_, w_valid_;
  bool striped_ = false;
  uint64_t kernel_launches_ = 0;
  PeerTable peers_;
  std::vector<uint64_t> slot_offsets_;
  std::vector<uint64_t> epochs_;
  unsigned int* counters_ = nullptr;
  int gather_ctas_ = 32;
  int gather_mode_ = 0;
  std::vector<cudaEvent_t> ph_acked_, ph_h2d_;  // per key: after wait_acks, after the H2D stripe
  std::vector<char> ph_valid_;
  std::vector<PhaseSample> phase_pending_;
  void collect_phase(size_t k);
};

}  // namespace ft
