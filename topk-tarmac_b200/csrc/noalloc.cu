// noalloc.cu — the fixed device scratch behind the no-allocation entry point
// tarmac_dense_attention_backward_noalloc (abi.cu).
//
// The dense-attention gradient needs two fp32 row statistics per query row
// (log-sum-exp and D) between its two kernels. The regular entry point takes
// that workspace from the caller; this file provides it instead as one
// file-scope device array, so a caller that cannot allocate device memory
// still gets gradients. The array is part of the library image: every GPU
// that loads the library holds it until the process exits.
#include <cuda.h>  // CUcontext / CUresult types only; no driver library link

#include <mutex>

#include "backward.cuh"

namespace tarmac {

// 2^20 floats (4 MiB): the row statistics of up to B * N = 2^19 query rows.
constexpr size_t NOALLOC_SCRATCH_FLOATS = size_t(1) << 20;

static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];

// In host code g_noalloc_scratch names a host-side stand-in, not device
// memory; its device address comes from cudaGetSymbolAddress with the
// device current. That address belongs to the CUDA context the module was
// loaded into, not to the device: after cudaDeviceReset, or under a context
// the caller created and made current through the driver API, the module
// lives at another address. So the address is cached per context, keyed by
// the driver's process-unique context id (cuCtxGetId), and looked up again
// the first time a call runs in a context not seen before.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct ScratchEntry {
  unsigned long long ctx_id;
  float* addr;
};
constexpr int NOALLOC_CACHE_SLOTS = 64;
static ScratchEntry g_cache[NOALLOC_CACHE_SLOTS];
static int g_cache_used = 0, g_cache_next = 0;
static std::mutex g_scratch_mu;
static std::once_flag g_entry_once;
static CtxGetCurrentFn g_ctx_get_current = nullptr;
static CtxGetIdFn g_ctx_get_id = nullptr;

static void resolve_driver_entry_points() {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) ==
          cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f);
  f = nullptr;
  if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) ==
          cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f);
}

// Process-unique id of the calling thread's current context; false when it
// cannot be read (no context current yet, or no driver entry point). Also
// keys the per-kernel shared-memory limits that abi.cu sets.
bool current_context_id(unsigned long long* id) {
  std::call_once(g_entry_once, resolve_driver_entry_points);
  if (!g_ctx_get_current || !g_ctx_get_id) return false;
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return g_ctx_get_id(ctx, id) == CUDA_SUCCESS;
}

size_t noalloc_scratch_floats() { return NOALLOC_SCRATCH_FLOATS; }

// Device address of the scratch array in the current context.
cudaError_t noalloc_scratch(float** ptr) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  unsigned long long id = 0;
  bool have_id = current_context_id(&id);
  if (have_id) {
    for (int i = 0; i < g_cache_used; ++i) {
      if (g_cache[i].ctx_id == id) {
        *ptr = g_cache[i].addr;
        return cudaSuccess;
      }
    }
  }
  // Not seen in this context: look the symbol up (this also binds the
  // device's primary context when none was current).
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  if (!have_id) have_id = current_context_id(&id);
  if (have_id) {
    // ring of the most recent contexts; an evicted one is looked up again
    g_cache[g_cache_next] = ScratchEntry{id, static_cast<float*>(addr)};
    g_cache_next = (g_cache_next + 1) % NOALLOC_CACHE_SLOTS;
    if (g_cache_used < NOALLOC_CACHE_SLOTS) ++g_cache_used;
  }
  *ptr = static_cast<float*>(addr);
  return cudaSuccess;
}

}  // namespace tarmac
