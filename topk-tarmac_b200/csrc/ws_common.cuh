// ws_common.cuh — helpers of the persistent warp-specialized kernels
// (topk_ws.cu, dense_ws.cu): bounded mbarrier waits with a shared abort
// flag, arrivals, and cp.async staging of bf16 tiles into the no-swizzle
// K-major core-matrix layout.
#pragma once

#include "tc_common.cuh"

namespace tarmac {

// polls per bounded wait (each try_wait may suspend the thread for a while)
constexpr uint32_t WS_WAIT_LIMIT = 1u << 22;

namespace ws {

// Bounded mbarrier wait that also gives up once another role aborted.
__device__ __forceinline__ bool wait(uint64_t* mbar, uint32_t parity,
                                     volatile int* abort_flag) {
  const uint32_t a = tc::smem_addr(mbar);
  for (uint32_t it = 0; it < WS_WAIT_LIMIT; ++it) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], "
        "%2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 63) == 63 && *abort_flag) return false;
  }
  *abort_flag = 1;
  return false;
}

// Non-blocking: has the mbarrier phase `parity` completed?
__device__ __forceinline__ bool test(uint64_t* mbar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], "
      "%2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(tc::smem_addr(mbar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                   tc::smem_addr(mbar))
               : "memory");
}

// 16-byte piece e of an R-row tile with KCH chunks per row, in the K-major
// core-matrix order: it sits at byte 16 e and holds row
// ((e / 8) / KCH) * 8 + e % 8, columns 8 c .. 8 c + 7 with c = (e / 8) % KCH.
template <int KCH>
__device__ __forceinline__ void piece_rc(int e, int& r, int& c) {
  r = ((e >> 3) / KCH) * 8 + (e & 7);
  c = (e >> 3) % KCH;
}

__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
               "l"(src), "r"(ok ? 16u : 0u)
               : "memory");
}

// bf16: rows [0, R) of src (row stride rs, d % 8 == 0) straight into a
// K-major tile of DP columns by NT threads; rows >= nvalid and columns >= d
// zero-filled.
template <int DP, int R, int NT>
__device__ __forceinline__ void copy_tile_bf16(uint32_t base,
                                               const __nv_bfloat16* src,
                                               int64_t rs, int nvalid, int d,
                                               int tid) {
  constexpr int KCH = DP / 8;
#pragma unroll 4
  for (int e = tid; e < R * KCH; e += NT) {
    int r, c;
    piece_rc<KCH>(e, r, c);
    const bool ok = r < nvalid && c * 8 < d;
    cp16(base + (uint32_t)e * 16u, ok ? src + (int64_t)r * rs + c * 8 : src, ok);
  }
}

}  // namespace ws
}  // namespace tarmac
