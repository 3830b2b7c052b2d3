// noalloc.cu — the fixed device scratch behind the no-allocation entry point
// tarmac_dense_attention_backward_noalloc (abi.cu).
//
// The dense-attention gradient needs two fp32 row statistics per query row
// (log-sum-exp and D) between its two kernels. The regular entry point takes
// that workspace from the caller; this file provides it instead as one
// file-scope device array, so a caller that cannot allocate device memory
// still gets gradients. The array is part of the library image: every GPU
// that loads the library holds it until the process exits.
#include <mutex>

#include "backward.cuh"

namespace tarmac {

// 2^20 floats (4 MiB): the row statistics of up to B * N = 2^19 query rows.
constexpr size_t NOALLOC_SCRATCH_FLOATS = size_t(1) << 20;

static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];

// In host code g_noalloc_scratch names a host-side stand-in, not device
// memory; the device address comes from cudaGetSymbolAddress, once per
// device, with that device current.
constexpr int NOALLOC_MAX_DEVICES = 64;
static float* g_scratch_addr[NOALLOC_MAX_DEVICES];
static std::mutex g_scratch_mu;

size_t noalloc_scratch_floats() { return NOALLOC_SCRATCH_FLOATS; }

// Device address of the scratch array on the current device.
cudaError_t noalloc_scratch(float** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = static_cast<float*>(addr);
  }
  *ptr = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace tarmac
