// common.cuh — device helpers shared by the TarMAC attention-core kernels.
//
// Layout convention (see include/tarmac_b200.h): Q, K, V, O are [B, N, d]
// arrays of fp32 or bf16 with unit innermost stride; batch and row strides are
// given in elements. Inside the kernels every row is widened to fp32 and padded
// with zeros to DP (a power of two >= d), so all arithmetic is fp32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tarmac_b200.h"

namespace tarmac {

// Element strides (in elements) of the four [B, N, d] operands.
struct Strides {
  int64_t qb, qn, kb, kn, vb, vn, ob, on;
};

// Everything an attention kernel needs; passed by value (kernel parameter).
struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  Strides st;
  int B, N, d;
  int topk;            // retained peers (top-k kernels)
  int mode;            // TARMAC_SELECT_* (resident-row kernel)
  float qscale;        // folded into q at load time (exact: a power of two)
  float post_scale;    // applied to the retained scores (1 when folded)
  int32_t* idx_out;    // optional [B, N, topk] rank-ordered retained peers
  int vec;             // 1: rows may be moved with 16-byte vector accesses
};

__host__ __device__ constexpr int cdiv(int a, int b) { return (a + b - 1) / b; }

// Raise kernel `fn`'s dynamic shared-memory limit to at least `bytes` in the
// current CUDA context. The attribute lasts as long as the context, so it is
// set only when this process has not yet set that much for this kernel in
// this context (a cudaFuncSetAttribute on every launch costs host time that
// small problems notice); a new context (after cudaDeviceReset, or one the
// caller made current through the driver API) sets it again. Safe from
// several host threads (abi.cu).
cudaError_t raise_smem_limit(const void* fn, size_t bytes);

// Process-unique id of the calling thread's current CUDA context (the
// driver's cuCtxGetId); false when no context is current or the driver does
// not offer the call (noalloc.cu).
bool current_context_id(unsigned long long* id);

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Load 4 consecutive elements starting at p (p is 16-byte aligned for fp32,
// 8-byte aligned for bf16 when `vec` holds) into fp32.
__device__ __forceinline__ float4 load4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 a = __bfloat1622float2(lo);
  float2 b = __bfloat1622float2(hi);
  return make_float4(a.x, a.y, b.x, b.y);
}

// Load the first `d` elements of a row into x[0..DP), zero beyond d.
// vec: d is a multiple of 4 (fp32) / 8 (bf16) and the row is 16-byte aligned.
template <int DP, typename T>
__device__ __forceinline__ void load_row(float (&x)[DP], const T* p, int d,
                                         bool vec) {
  if (vec) {
#pragma unroll
    for (int c = 0; c < DP; c += 4) {
      if (c < d) {
        float4 f = load4(p + c);
        x[c] = f.x; x[c + 1] = f.y; x[c + 2] = f.z; x[c + 3] = f.w;
      } else {
        x[c] = 0.f; x[c + 1] = 0.f; x[c + 2] = 0.f; x[c + 3] = 0.f;
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < DP; ++c) x[c] = (c < d) ? to_f32<T>(p[c]) : 0.f;
  }
}

// Store the first `d` values of x to a row.
template <int DP, typename T>
__device__ __forceinline__ void store_row(T* p, const float (&x)[DP], int d,
                                          bool vec) {
  if constexpr (sizeof(T) == 4) {
    if (vec) {
#pragma unroll
      for (int c = 0; c < DP; c += 4)
        if (c < d)
          *reinterpret_cast<float4*>(p + c) =
              make_float4(x[c], x[c + 1], x[c + 2], x[c + 3]);
      return;
    }
  } else {
    if (vec) {
#pragma unroll
      for (int c = 0; c < DP; c += 4)
        if (c < d) {
          __nv_bfloat162 lo = __floats2bfloat162_rn(x[c], x[c + 1]);
          __nv_bfloat162 hi = __floats2bfloat162_rn(x[c + 2], x[c + 3]);
          uint2 u;
          u.x = *reinterpret_cast<uint32_t*>(&lo);
          u.y = *reinterpret_cast<uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(p + c) = u;
        }
      return;
    }
  }
#pragma unroll
  for (int c = 0; c < DP; ++c)
    if (c < d) p[c] = from_f32<T>(x[c]);
}

// ---------------------------------------------------------------------------
// packed fp32x2 arithmetic (sm_100): one instruction performs two IEEE fp32
// FMAs, which halves the issue slots the FMA-bound loops spend on arithmetic
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float2 unpack2(uint64_t x) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(x));
  return make_float2(lo, hi);
}
__device__ __forceinline__ float hsum2(uint64_t x) {
  const float2 f = unpack2(x);
  return f.x + f.y;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Maximum of CH (8 or 16) consecutive values as a shallow tree of
// three-input maxima (dependency depth 2 or 3 instead of a chain); max is
// exact, so the result equals the chain's (NaN inputs are skipped alike).
template <int CH>
__device__ __forceinline__ float chunk_max(const float* v) {
  static_assert(CH == 8 || CH == 16, "8- or 16-value chunks");
  if constexpr (CH == 8) {
    return max3f(max3f(v[0], v[1], v[2]), max3f(v[3], v[4], v[5]),
                 fmaxf(v[6], v[7]));
  } else {
    const float a = max3f(v[0], v[1], v[2]), b = max3f(v[3], v[4], v[5]);
    const float c = max3f(v[6], v[7], v[8]), e = max3f(v[9], v[10], v[11]);
    const float f = max3f(v[12], v[13], v[14]);
    return fmaxf(max3f(a, b, c), max3f(e, f, v[15]));
  }
}

// q (as DP/2 column pairs) . one fp32 row in shared memory (16-byte aligned):
// even and odd columns accumulate in the two halves, added at the end. Every
// caller forms a given score through this one function, so a score is
// bit-identical wherever it is recomputed.
template <int DP>
__device__ __forceinline__ float dot_pairs(const uint64_t (&qp)[DP / 2],
                                           const float* kr) {
  uint64_t acc = 0ull;
#pragma unroll
  for (int c = 0; c < DP; c += 4) {
    const ulonglong2 kv = *reinterpret_cast<const ulonglong2*>(kr + c);
    acc = ffma2(qp[c / 2], kv.x, acc);
    acc = ffma2(qp[c / 2 + 1], kv.y, acc);
  }
  return hsum2(acc);
}

// Monotone map fp32 -> uint32: a < b (as non-NaN floats) iff key(a) < key(b).
// Restates _float_to_ordered_int (fused_topk_attention.py:113-124) in unsigned
// form (offset by 2^31, so the order is the same).
__device__ __forceinline__ uint32_t ordered_key(float x) {
  uint32_t u = __float_as_uint(x);
  return u ^ ((u & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
  return __uint_as_float(u);
}

// 16-byte global -> shared copy that does not pass through registers
// (cp.async, L2 only); completes at cp_async_wait_all().
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc)
               : "memory");
}
// cp.async of 16 bytes to a shared-memory address (as a 32-bit shared
// window offset)
__device__ __forceinline__ void cp_async16_addr(uint32_t smem_dst,
                                                const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_dst),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void st_shared_zero16(uint32_t smem_dst) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(smem_dst),
               "r"(0u)
               : "memory");
}
__device__ __forceinline__ uint32_t tc_smem_base(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int PENDING>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(PENDING) : "memory");
}

// Stage rows [0, nrows) of a [N, d] episode slice (first row `r0`, row
// stride `rs`) into shared fp32 rows of `sstride` floats, zero-padding rows
// >= N and columns >= d. fp32 rows on the vector path move with cp.async
// (the caller waits with cp_async_wait_all / cp_async_wait<n>); other rows
// are converted through registers, four 16-byte loads in flight per thread.
// All threads of the block participate.
template <int DP, typename T>
__device__ __forceinline__ void stage_rows(float* __restrict__ dst, int sstride,
                                           const T* __restrict__ base,
                                           int64_t rs, int r0, int nrows, int N,
                                           int d, bool vec) {
  constexpr int C4 = DP / 4;
  const int total = nrows * C4;
  if constexpr (sizeof(T) == 4) {
    if (vec) {
      for (int e = threadIdx.x; e < total; e += blockDim.x) {
        const int row = e / C4;
        const int c = (e - row * C4) * 4;
        float* sp = dst + (size_t)row * sstride + c;
        const int r = r0 + row;
        if (r < N && c < d)
          cp_async16(sp, base + (int64_t)r * rs + c);
        else
          *reinterpret_cast<float4*>(sp) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      return;
    }
  }
  constexpr int U = 4;
  for (int e0 = threadIdx.x; e0 < total; e0 += U * blockDim.x) {
    float4 f[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * blockDim.x;
      const int row = e / C4;
      const int c = (e - row * C4) * 4;
      const int r = r0 + row;
      f[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < total && r < N && c < d) {
        const T* src = base + (int64_t)r * rs + c;
        if (vec) {
          f[u] = load4(src);
        } else {
          f[u].x = to_f32<T>(src[0]);
          f[u].y = (c + 1 < d) ? to_f32<T>(src[1]) : 0.f;
          f[u].z = (c + 2 < d) ? to_f32<T>(src[2]) : 0.f;
          f[u].w = (c + 3 < d) ? to_f32<T>(src[3]) : 0.f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < total) {
        const int row = e / C4;
        const int c = (e - row * C4) * 4;
        *reinterpret_cast<float4*>(dst + (size_t)row * sstride + c) = f[u];
      }
    }
  }
}

}  // namespace tarmac
