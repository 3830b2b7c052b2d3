// episode.cuh — per-episode position helpers shared by the Morton and the
// kNN selectors: block-wide coordinate bounds and the reference's
// normalise-and-truncate quantisation.
#pragma once

#include "common.cuh"

namespace tarmac {

// trunc(((x - lo) / span) * scale_q) clamped to [0, qmax], every step an
// explicitly rounded fp32 operation (no contraction), as the reference's
// elementwise tensor arithmetic evaluates it; `.long()` truncates toward zero.
__device__ __forceinline__ uint32_t quantise(float x, float lo, float span,
                                             float scale_q, uint32_t qmax) {
  const float g = __fmul_rn(__fdiv_rn(__fsub_rn(x, lo), span), scale_q);
  // .long() truncates toward zero, then clamp_(0, qmax)
  long long t = (g >= 9.0e18f) ? (long long)qmax : (long long)g;
  if (g != g) t = 0;  // NaN position: quantise to 0 (no defined cell)
  if (t < 0) t = 0;
  if (t > (long long)qmax) t = qmax;
  return (uint32_t)t;
}

// Block-wide min/max of both coordinates of one episode into sm[0..3]
// (lo_x, lo_y, hi_x, hi_y). red must hold 4 * (blockDim/32) floats.
__device__ __forceinline__ void episode_bounds(const float* pos, int N,
                                               float* red, float* out4) {
  float lx = INFINITY, ly = INFINITY, hx = -INFINITY, hy = -INFINITY;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const float2 pxy = reinterpret_cast<const float2*>(pos)[i];
    lx = fminf(lx, pxy.x); ly = fminf(ly, pxy.y);
    hx = fmaxf(hx, pxy.x); hy = fmaxf(hy, pxy.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lx = fminf(lx, __shfl_xor_sync(0xffffffffu, lx, o));
    ly = fminf(ly, __shfl_xor_sync(0xffffffffu, ly, o));
    hx = fmaxf(hx, __shfl_xor_sync(0xffffffffu, hx, o));
    hy = fmaxf(hy, __shfl_xor_sync(0xffffffffu, hy, o));
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[w] = lx; red[nw + w] = ly; red[2 * nw + w] = hx; red[3 * nw + w] = hy;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int u = 1; u < nw; ++u) {
      lx = fminf(lx, red[u]); ly = fminf(ly, red[nw + u]);
      hx = fmaxf(hx, red[2 * nw + u]); hy = fmaxf(hy, red[3 * nw + u]);
    }
    out4[0] = lx; out4[1] = ly; out4[2] = hx; out4[3] = hy;
  }
  __syncthreads();
}

}  // namespace tarmac
