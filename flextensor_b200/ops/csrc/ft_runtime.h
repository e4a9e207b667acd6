// Native transfer engine and host-memory helpers (runtime.cpp).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <vector>

namespace ft {

void host_register(void* ptr, size_t bytes);
void host_unregister(void* ptr);

struct TransferSample {
  int key = 0;
  size_t bytes = 0;
  float transfer_ms = 0.f;
  float wait_ms = 0.f;
};

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
};

}  // namespace ft
