// prescore.cuh — one query row's online-softmax attention over given peers,
// spread over a group of DP/4 lanes (each owns 4 consecutive columns). Shared
// by the stand-alone prescore kernel and the fused Morton + prescore kernel.
#pragma once

#include "common.cuh"

namespace tarmac {

// 4 columns [c, c+4) of a row, zero beyond d.
template <typename T>
__device__ __forceinline__ float4 load_cols4(const T* row, int c, int d,
                                             bool vec) {
  float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c < d) {
    if (vec) {
      f = load4(row + c);
    } else {
      f.x = to_f32<T>(row[c]);
      f.y = (c + 1 < d) ? to_f32<T>(row[c + 1]) : 0.f;
      f.z = (c + 2 < d) ? to_f32<T>(row[c + 2]) : 0.f;
      f.w = (c + 3 < d) ? to_f32<T>(row[c + 3]) : 0.f;
    }
  }
  return f;
}

template <int DP, typename T>
struct PrescoreRow {
  static constexpr int L = DP / 4;
  float4 q, acc;
  float run_max, den;

  __device__ __forceinline__ void init(const AttnParams& p, int b, int i,
                                       int sub, bool live) {
    const bool vec = p.vec != 0;
    q = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) {
      const T* qr = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb +
                    (int64_t)i * p.st.qn;
      q = load_cols4<T>(qr, sub * 4, p.d, vec);
      q.x *= p.qscale; q.y *= p.qscale; q.z *= p.qscale; q.w *= p.qscale;
    }
    acc = make_float4(0.f, 0.f, 0.f, 0.f);
    run_max = -INFINITY;
    den = 0.f;
  }

  // One peer j (already range-checked). Every lane of the warp must call it.
  __device__ __forceinline__ void step(const AttnParams& p, int b, int j,
                                       int sub) {
    const bool vec = p.vec != 0;
    const T* kr = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb +
                  (int64_t)j * p.st.kn;
    const T* vr = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb +
                  (int64_t)j * p.st.vn;
    const float4 kv = load_cols4<T>(kr, sub * 4, p.d, vec);
    const float4 vv = load_cols4<T>(vr, sub * 4, p.d, vec);
    float s = q.x * kv.x;
    s = fmaf(q.y, kv.y, s);
    s = fmaf(q.z, kv.z, s);
    s = fmaf(q.w, kv.w, s);
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= p.post_scale;
    const float m_new = fmaxf(run_max, s);
    const float alpha = (run_max == -INFINITY) ? 0.f : expf(run_max - m_new);
    const float pe = expf(s - m_new);
    den = den * alpha + pe;
    acc.x = acc.x * alpha + pe * vv.x;
    acc.y = acc.y * alpha + pe * vv.y;
    acc.z = acc.z * alpha + pe * vv.z;
    acc.w = acc.w * alpha + pe * vv.w;
    run_max = m_new;
  }

  __device__ __forceinline__ void finish(const AttnParams& p, int b, int i,
                                         int sub, bool bad) {
    const int c = sub * 4;
    if (c >= p.d) return;
    T* orow = static_cast<T*>(p.o) + (int64_t)b * p.st.ob + (int64_t)i * p.st.on;
    float o[4] = {acc.x / den, acc.y / den, acc.z / den, acc.w / den};
    if (bad) o[0] = o[1] = o[2] = o[3] = __int_as_float(0x7fc00000);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (c + e < p.d) orow[c + e] = from_f32<T>(o[e]);
  }
};

}  // namespace tarmac
