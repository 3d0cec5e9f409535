// noalloc.cu — a sum fold that allocates nothing.
//
// mapal_gpu_fold_sum_f32 takes its scratch (one f64 partial per block and a
// block-arrival counter) from its context, which allocates it with cudaMalloc
// when the context is created. Some callers cannot allocate device memory at
// all: a host runtime that hands every byte of device memory out of one
// arena it sized up front (the emitted program's per-function arena model)
// and must not have a library allocate behind it, a process already at the
// edge of HBM where one more allocation fails, or a latency-bound loop that
// cannot absorb cudaMalloc's device-wide synchronisation. This entry point
// serves them: it needs no context, and its scratch is a fixed array in the
// library's own device data, which every GPU that loads the library holds
// until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents, so the counter that must start at zero is cleared on the stream
// before each launch. Two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the array and give wrong sums;
// calls on one stream, or otherwise ordered, are safe.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace {

// One f64 partial per block of the fold kernel (it launches at most 4 blocks
// per SM, so 1024 slots cover devices of up to 256 SMs), plus one slot whose
// first 4 bytes hold the block-arrival counter. 8 KiB + 8 bytes.
constexpr int kNoAllocSlots = 1024;
static __device__ __align__(256) double g_fold_noalloc_scratch[kNoAllocSlots + 1];

// Host-side addresses of the array, one per device ordinal, filled by the
// first call on that device. In host code the symbol itself is only a
// stand-in, never a device address: passing it to a kernel would fault, or
// silently use the wrong memory where the GPU can reach host memory.
//
// Host threads may make their first calls at the same time: the table is
// filled under a mutex, and an entry's address is published (release) only
// after its SM count is written, so a reader that sees the address (acquire)
// also sees the count. An address is looked up once per device for the life
// of the process; after cudaDeviceReset on a device it is stale, so calls
// that follow a reset are not supported.
constexpr int kMaxDevices = 64;
struct ScratchEntry {
  std::atomic<double*> ptr{nullptr};
  int sm_count = 0;
};
ScratchEntry g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// `device` is current on the calling thread.
int setup(int device, double** ptr, int* sm_count) {
  ScratchEntry& e = g_scratch[device];
  double* p = e.ptr.load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    p = e.ptr.load(std::memory_order_relaxed);
    if (!p) {
      void* addr = nullptr;
      cudaError_t err = cudaGetSymbolAddress(&addr, g_fold_noalloc_scratch);
      if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(g_fold_noalloc_scratch)");
      int sms = 0;
      err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(MultiProcessorCount)");
      e.sm_count = sms;
      p = static_cast<double*>(addr);
      e.ptr.store(p, std::memory_order_release);
    }
  }
  *ptr = p;
  *sm_count = e.sm_count;
  return 0;
}

}  // namespace

extern "C" int mapal_gpu_fold_sum_f32_noalloc(float seed, const float* x, uint64_t n, float* out,
                                              void* stream) {
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  if (n && !x) return set_error(MAPAL_ERR_INVALID, "x is null");
  int device = -1;
  MAPAL_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices)
    return set_error(MAPAL_ERR_INVALID, "device ordinal beyond the no-alloc table (64 devices)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The scratch address is the current device's; a stream of another device
  // would run the kernel there against this device's array, so it is refused.
  if (s != nullptr) {
    int stream_device = -1;
    MAPAL_CUDA(cudaStreamGetDevice(s, &stream_device));
    if (stream_device != device)
      return set_error(MAPAL_ERR_INVALID, "stream belongs to device " + std::to_string(stream_device) +
                                              ", the calling thread's current device is " + std::to_string(device));
  }
  double* partials = nullptr;
  int sm_count = 0;
  MAPAL_TRY(setup(device, &partials, &sm_count));
  // The fold kernel uses one partial slot per block, at most 4 blocks per SM
  // (capped at kFoldMaxBlocks): a device needing more slots than the static
  // array holds is refused rather than overrun.
  int max_blocks = 4 * sm_count;
  if (max_blocks > kFoldMaxBlocks) max_blocks = kFoldMaxBlocks;
  if (max_blocks > kNoAllocSlots)
    return set_error(MAPAL_ERR_INVALID,
                     "the no-alloc sum keeps 1024 partial slots; this device needs " +
                         std::to_string(max_blocks) + " (4 per SM)");
  unsigned* counter = reinterpret_cast<unsigned*>(partials + kNoAllocSlots);
  MAPAL_CUDA(cudaMemsetAsync(counter, 0, sizeof(unsigned), s));
  MAPAL_TRY(launch_fold_sum(s, sm_count, x, n, seed, partials, counter, out, nullptr));
  MAPAL_CUDA(cudaGetLastError());
  return 0;
}
