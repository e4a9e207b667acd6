// Peer-memory data plane for striped weight streaming (NVLink 5 / NVSwitch).
//
// Every rank owns a symmetric device heap (same layout on every rank, mapped into
// every peer through CUDA IPC). A weight block is streamed as N stripes: rank r
// copies stripe r host->device into its own slot, then
//   publish  : one thread stores epoch into flags[r][slot] of EVERY rank
//              (st.release.sys, so the stripe bytes are visible before the flag);
//   gather   : CTAs wait (ld.acquire.sys, bounded) until flags[p][slot] >= epoch for each
//              peer p, pull stripe p from p's slot with 16-byte loads over NVLink into the
//              local slot, and the last CTA to finish stores epoch into acks[r][slot] of
//              every peer (so p may overwrite its slot for the next epoch);
//   wait_acks: before the next H2D into a slot, wait until every peer acked the previous
//              epoch of that slot.
// Copy-engine variant of the gather (gather mode 1): wait_flags (one warp, bounded) ->
// one cudaMemcpyAsync per peer stripe on the copy stream (DMA over NVLink, no SM time) ->
// ack (one thread stores the acknowledgements).
// These kernels wait on OTHER GPUs only (never on another launch on the same GPU). No
// TMA and no multicast is used: plain peer loads and stores. Every wait has a clock64
// bound; on timeout the kernel records kErrPeerTimeout in the device error word and returns.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "ft_p2p.h"
#include "sm100_common.cuh"

namespace ft {

FT_DEFINE_ERROR_READER(p2p_device_error)

namespace {

constexpr int kGatherThreads = 256;

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ bool wait_geq(const uint64_t* p, uint64_t target) {
  const long long t0 = clock64();
  while (ld_acquire_sys(p) < target) {
    if ((unsigned long long)(clock64() - t0) > FT_WAIT_LIMIT_CYCLES) {
      record_error(kErrPeerTimeout);
      return false;
    }
    if (error_raised()) return false;
    __nanosleep(200);
  }
  return true;
}

__global__ void publish_kernel(PeerTable t, int slot, uint64_t epoch) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < t.world; p++) st_release_sys(t.flags[p] + (size_t)t.rank * t.n_slots + slot, epoch);
  }
}

__global__ void wait_acks_kernel(PeerTable t, int slot, uint64_t epoch) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const uint64_t* mine = t.acks[t.rank];
    for (int p = 0; p < t.world; p++) {
      if (p == t.rank) continue;
      if (!wait_geq(mine + (size_t)p * t.n_slots + slot, epoch)) return;
    }
  }
}

// Small CTAs with a low register cap (launch bounds: 5 x 256 threads per SM) so a gather CTA
// fits beside one resident CTA of the persistent GEMM / attention kernels on the same SM and
// the NVLink pull overlaps compute instead of queueing it. Four 16-byte loads in flight per thread.
__global__ void __launch_bounds__(kGatherThreads, 5)
gather_kernel(PeerTable t, int slot, uint64_t epoch, uint64_t slot_offset, uint64_t stripe_bytes,
              uint64_t total_bytes, unsigned int* done_counter) {
  __shared__ int ok;
  const uint64_t* myflags = t.flags[t.rank];
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (int pi = 1; pi < t.world; pi++) {
    const int p = (t.rank + pi) % t.world;  // stagger peers so ranks do not all hit the same source
    if (threadIdx.x == 0) ok = wait_geq(myflags + (size_t)p * t.n_slots + slot, epoch) ? 1 : 0;
    __syncthreads();
    if (!ok) return;
    const uint64_t begin = (uint64_t)p * stripe_bytes;
    const uint64_t end = begin + stripe_bytes < total_bytes ? begin + stripe_bytes : total_bytes;
    if (begin >= end) continue;
    const uint4* src = reinterpret_cast<const uint4*>(t.heap[p] + slot_offset + begin);
    uint4* dst = reinterpret_cast<uint4*>(t.heap[t.rank] + slot_offset + begin);
    const uint64_t n16 = (end - begin) / 16;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n16; i += 4 * stride) {  // streaming: each peer byte is read exactly once
      const uint4 v0 = __ldcs(src + i), v1 = __ldcs(src + i + stride);
      const uint4 v2 = __ldcs(src + i + 2 * stride), v3 = __ldcs(src + i + 3 * stride);
      __stcg(dst + i, v0);
      __stcg(dst + i + stride, v1);
      __stcg(dst + i + 2 * stride, v2);
      __stcg(dst + i + 3 * stride, v3);
    }
    for (; i < n16; i += stride) __stcg(dst + i, __ldcs(src + i));
  }
  // last CTA out acknowledges every peer's stripe for this epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(done_counter + slot, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(done_counter + slot, 0u);
      for (int p = 0; p < t.world; p++) {
        if (p == t.rank) continue;
        st_release_sys(t.acks[p] + (size_t)t.rank * t.n_slots + slot, epoch);
      }
    }
  }
}

// Copy-engine gather, step 1: one warp waits (bounded) until every peer published `epoch` for
// `slot`, so the copies queued behind it on the stream read complete stripes.
__global__ void wait_flags_kernel(PeerTable t, int slot, uint64_t epoch) {
  if (blockIdx.x == 0 && threadIdx.x < t.world && threadIdx.x != t.rank)
    wait_geq(t.flags[t.rank] + (size_t)threadIdx.x * t.n_slots + slot, epoch);
}

// Copy-engine gather, step 3 (after the peer copies on the stream): tell every peer we are done
// reading its stripe of this epoch.
__global__ void ack_kernel(PeerTable t, int slot, uint64_t epoch) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < t.world; p++) {
      if (p == t.rank) continue;
      st_release_sys(t.acks[p] + (size_t)t.rank * t.n_slots + slot, epoch);
    }
  }
}

}  // namespace

cudaError_t p2p_wait_flags(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s) {
  if (t.world <= 1) return cudaSuccess;
  wait_flags_kernel<<<1, 32, 0, s>>>(t, slot, epoch);
  return cudaGetLastError();
}

cudaError_t p2p_ack(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s) {
  if (t.world <= 1) return cudaSuccess;
  ack_kernel<<<1, 32, 0, s>>>(t, slot, epoch);
  return cudaGetLastError();
}

cudaError_t p2p_publish(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s) {
  publish_kernel<<<1, 32, 0, s>>>(t, slot, epoch);
  return cudaGetLastError();
}

cudaError_t p2p_wait_acks(const PeerTable& t, int slot, uint64_t epoch, cudaStream_t s) {
  if (t.world <= 1 || epoch == 0) return cudaSuccess;
  wait_acks_kernel<<<1, 32, 0, s>>>(t, slot, epoch);
  return cudaGetLastError();
}

cudaError_t p2p_gather(const PeerTable& t, int slot, uint64_t epoch, uint64_t slot_offset, uint64_t stripe_bytes,
                       uint64_t total_bytes, unsigned int* done_counter, int ctas, cudaStream_t s) {
  if (t.world <= 1) return cudaSuccess;
  if ((slot_offset | stripe_bytes | total_bytes) & 15) return cudaErrorInvalidValue;
  gather_kernel<<<ctas, kGatherThreads, 0, s>>>(t, slot, epoch, slot_offset, stripe_bytes, total_bytes, done_counter);
  return cudaGetLastError();
}

}  // namespace ft

// ======================================================================================
// No-allocation C entry point for the striped gather.
//
// This entry point has no counterpart in the reference (which has no native code). It serves
// callers that must not allocate device memory on the call path: code driving the gather from
// plain C or from a foreign runtime with no torch allocator at hand, and engines whose device
// memory is planned up front, where an allocation on the call path could fail or fragment the
// pool mid-run.
//
// The gather's only scratch is one arrival counter per ring slot (the last CTA out acknowledges
// the peers and re-zeroes it). Here those counters live in the file-scope device array
// `g_gather_noalloc_counters` (kGatherNoAllocMaxSlots = 256 counters, 1 KiB) instead of a
// caller buffer, so a call allocates nothing: no cudaMalloc / cudaFree, no library call that
// allocates. Slot indices or slot counts beyond 256 are rejected with cudaErrorInvalidValue.
//
// Device address: in host code `g_gather_noalloc_counters` names only a host-side stand-in
// for the symbol, so the kernel never receives it directly. The first call on each device
// (with that device current) looks the address up with cudaGetSymbolAddress, checks the
// result and caches it; make that first call on a device before any stream capture begins.
// The cached address is not refreshed after a device reset (see the cache below).
//
// Every call on a device shares the one array, and the array keeps whatever the previous call
// left. The counter of the slot in use is therefore cleared (cudaMemsetAsync on the caller's
// stream) before each launch, so a call that timed out earlier cannot leave a stale count.
// Calls whose executions overlap on the GPU (several streams, or several host threads on one
// device) race on the shared counters and must be serialised by the caller.
// ======================================================================================
namespace ft {
namespace {

constexpr int kGatherNoAllocMaxSlots = 256;
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) unsigned int g_gather_noalloc_counters[kGatherNoAllocMaxSlots];

// Per-device cache of the array's device address. Entries are atomics (relaxed): two host
// threads making the first call on one device at once may both look the address up, and both
// store the same value. The cache does not survive a device reset: after cudaDeviceReset (or a
// reset of the primary context) on a device, the cached address is stale, so callers that reset
// a device must not use this entry point on it again in the same process.
std::atomic<unsigned int*> g_noalloc_addr_cache[kNoAllocMaxDevices];

unsigned int* noalloc_counters_for_current_device(cudaError_t* err) {
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  unsigned int* cached = g_noalloc_addr_cache[dev].load(std::memory_order_relaxed);
  if (cached == nullptr) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_gather_noalloc_counters);
    if (*err != cudaSuccess) return nullptr;
    cached = static_cast<unsigned int*>(p);
    g_noalloc_addr_cache[dev].store(cached, std::memory_order_relaxed);
  }
  return cached;
}

}  // namespace
}  // namespace ft

// Arguments: per-rank device pointers (heap base, flag array, ack array) for `world` ranks,
// this rank's index, slots per heap, the slot to gather, its epoch, the slot's byte offset in
// every heap, the stripe length, the packed block size, the grid size and a cudaStream_t.
// Returns a cudaError_t value (cudaSuccess = 0).
extern "C" int ft_p2p_gather_noalloc(const uint64_t* heap_ptrs, const uint64_t* flag_ptrs,
                                     const uint64_t* ack_ptrs, int world, int rank, int n_slots, int slot,
                                     uint64_t epoch, uint64_t slot_offset, uint64_t stripe_bytes,
                                     uint64_t total_bytes, int ctas, void* stream) {
  using namespace ft;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return (int)cudaErrorInvalidValue;
  if (n_slots < 1 || n_slots > ft::kGatherNoAllocMaxSlots || slot < 0 || slot >= n_slots) return (int)cudaErrorInvalidValue;
  if (ctas < 1 || !heap_ptrs || !flag_ptrs || !ack_ptrs) return (int)cudaErrorInvalidValue;
  cudaError_t err = cudaSuccess;
  unsigned int* counters = noalloc_counters_for_current_device(&err);
  if (counters == nullptr) return (int)err;
  PeerTable t;
  for (int p = 0; p < world; p++) {
    t.heap[p] = reinterpret_cast<uint8_t*>(heap_ptrs[p]);
    t.flags[p] = reinterpret_cast<uint64_t*>(flag_ptrs[p]);
    t.acks[p] = reinterpret_cast<uint64_t*>(ack_ptrs[p]);
  }
  t.rank = rank;
  t.world = world;
  t.n_slots = n_slots;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  err = cudaMemsetAsync(counters + slot, 0, sizeof(unsigned int), s);
  if (err != cudaSuccess) return (int)err;
  return (int)p2p_gather(t, slot, epoch, slot_offset, stripe_bytes, total_bytes, counters, ctas, s);
}
