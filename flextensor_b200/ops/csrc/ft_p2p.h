// Peer-memory data plane (p2p.cu) and symmetric-heap helpers (runtime.cpp).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ft {

constexpr int kMaxRanks = 8;

// Device pointers, valid in this process, into every rank's symmetric heap.
struct PeerTable {
  uint8_t* heap[kMaxRanks];   // base of rank p's heap (own heap at [rank])
  uint64_t* flags[kMaxRanks]; // rank p's flag array [world][n_slots]: flags[src][slot] = last published epoch
  uint64_t* acks[kMaxRanks];  // rank p's ack array  [world][n_slots]: acks[src][slot] = last epoch src finished reading
  int rank = 0;
  int world = 1;
  int n_slots = 0;
};

cudaError_t p2p_publish(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s);
cudaError_t p2p_wait_acks(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s);
cudaError_t p2p_gather(const PeerTable& t, int slot, uint64_t epoch, uint64_t slot_offset, uint64_t stripe_bytes,
                       uint64_t total_bytes, unsigned int* done_counter, int ctas, cudaStream_t s);
cudaError_t p2p_wait_flags(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s);
cudaError_t p2p_ack(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s);
int p2p_device_error(bool reset);

}  // namespace ft

// No-allocation striped gather (defined in p2p.cu): the arrival counters live in a file-scope
// device array of 256 entries instead of a caller buffer, so a call allocates no device memory.
// heap_ptrs / flag_ptrs / ack_ptrs hold `world` device addresses each (valid in this process).
// Returns a cudaError_t value; sizes beyond the array are rejected with cudaErrorInvalidValue.
extern "C" int ft_p2p_gather_noalloc(const uint64_t* heap_ptrs, const uint64_t* flag_ptrs,
                                     const uint64_t* ack_ptrs, int world, int rank, int n_slots, int slot,
                                     uint64_t epoch, uint64_t slot_offset, uint64_t stripe_bytes,
                                     uint64_t total_bytes, int ctas, void* stream);
