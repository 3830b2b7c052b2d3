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
    apply(p, kv, vv);
  }

  // Up to G peers js[0..cnt) (range-checked) in order: every K and V piece
  // is loaded before the first score is formed, so a row waits for one
  // memory round trip per G peers instead of one per peer; the online
  // softmax then takes them in the same order as step(). Every lane of the
  // warp must call it with the same cnt.
  template <int G>
  __device__ __forceinline__ void steps(const AttnParams& p, int b,
                                        const int (&js)[G], int cnt,
                                        int sub) {
    const bool vec = p.vec != 0;
    float4 kv[G], vv[G];
#pragma unroll
    for (int m = 0; m < G; ++m) {
      if (m < cnt) {
        const T* kr = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb +
                      (int64_t)js[m] * p.st.kn;
        const T* vr = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb +
                      (int64_t)js[m] * p.st.vn;
        kv[m] = load_cols4<T>(kr, sub * 4, p.d, vec);
        vv[m] = load_cols4<T>(vr, sub * 4, p.d, vec);
      }
    }
#pragma unroll
    for (int m = 0; m < G; ++m)
      if (m < cnt) apply(p, kv[m], vv[m]);
  }

  // one online-softmax step with a loaded K and V piece
  __device__ __forceinline__ void apply(const AttnParams& p, const float4 kv,
                                        const float4 vv) {
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
    if (p.vec != 0) {  // c + 4 <= d and the piece is 16-byte (8-byte) aligned
      if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(orow + c) = make_float4(o[0], o[1], o[2], o[3]);
      } else {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(o[2], o[3]);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&lo);
        u.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(orow + c) = u;
      }
      return;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (c + e < p.d) orow[c + e] = from_f32<T>(o[e]);
  }
};

// One query row per thread, d <= DT (DT = 8 or 16): the whole row's
// softmax runs once (no lanes repeating it, no shuffles), peers are taken
// two at a time with all their K and V pieces loaded before the first
// score. The dot product adds the four 4-column partial sums as
// (s0 + s2) + (s1 + s3), the order the lane-split form produces.
template <int DT, typename T>
struct PrescoreRowThread {
  float q[DT], acc[DT];
  float run_max, den;

  __device__ __forceinline__ static void load_row(float (&x)[DT], const T* r,
                                                  int d, bool vec) {
#pragma unroll
    for (int c = 0; c < DT; c += 4) {
      const float4 f = load_cols4<T>(r, c, d, vec);
      x[c] = f.x; x[c + 1] = f.y; x[c + 2] = f.z; x[c + 3] = f.w;
    }
  }

  __device__ __forceinline__ void init(const AttnParams& p, const T* qr,
                                       bool live) {
#pragma unroll
    for (int c = 0; c < DT; ++c) { q[c] = 0.f; acc[c] = 0.f; }
    if (live) {
      load_row(q, qr, p.d, p.vec != 0);
#pragma unroll
      for (int c = 0; c < DT; ++c) q[c] *= p.qscale;
    }
    run_max = -INFINITY;
    den = 0.f;
  }

  // peers kr[0..cnt), vr[0..cnt) (cnt <= 2), rows already range-checked
  __device__ __forceinline__ void steps2(const AttnParams& p,
                                         const T* const (&kr)[2],
                                         const T* const (&vr)[2], int cnt) {
    const bool vec = p.vec != 0;
    float kx[2][DT], vx[2][DT];
#pragma unroll
    for (int m = 0; m < 2; ++m)
      if (m < cnt) {
        load_row(kx[m], kr[m], p.d, vec);
        load_row(vx[m], vr[m], p.d, vec);
      }
    apply2(p, kx, vx, cnt);
  }

  // The same with the peer rows js[0..cnt) read from shared memory: K rows
  // at sK, V rows at sV, 16-byte piece c of row j at byte off(j, c) (pieces
  // beyond d hold zeros).
  template <typename Off>
  __device__ __forceinline__ void steps2_shared(const AttnParams& p,
                                                uint32_t sK, uint32_t sV,
                                                const int (&js)[2], int cnt,
                                                Off off) {
    constexpr int EP = 16 / (int)sizeof(T);
    float kx[2][DT], vx[2][DT];
#pragma unroll
    for (int m = 0; m < 2; ++m)
      if (m < cnt) {
#pragma unroll
        for (int c = 0; c < DT / EP; ++c) {
          const uint32_t o = off(js[m], c);
          load_piece(kx[m], c * EP, sK + o);
          load_piece(vx[m], c * EP, sV + o);
        }
      }
    apply2(p, kx, vx, cnt);
  }

  // One peer row j from shared memory (K rows at sK, V rows at sV, piece c
  // of row j at byte off(j, c), zeros beyond d): the score from K pieces,
  // then the accumulator from V pieces, so only one piece is held at a
  // time. Same arithmetic as apply2.
  template <typename Off>
  __device__ __forceinline__ void step_shared(const AttnParams& p, uint32_t sK,
                                              uint32_t sV, int j, Off off) {
    constexpr int EP = 16 / (int)sizeof(T);
    float part[DT / 4];
#pragma unroll
    for (int c = 0; c < DT / EP; ++c) {
      float x[DT];
      load_piece(x, c * EP, sK + off(j, c));
#pragma unroll
      for (int g = c * EP / 4; g < (c + 1) * EP / 4; ++g) {
        float t = q[4 * g] * x[4 * g];
        t = fmaf(q[4 * g + 1], x[4 * g + 1], t);
        t = fmaf(q[4 * g + 2], x[4 * g + 2], t);
        part[g] = fmaf(q[4 * g + 3], x[4 * g + 3], t);
      }
    }
    float s;
    if constexpr (DT == 16)
      s = (part[0] + part[2]) + (part[1] + part[3]);
    else
      s = part[0] + part[1];
    s *= p.post_scale;
    const float m_new = fmaxf(run_max, s);
    const float alpha = (run_max == -INFINITY) ? 0.f : expf(run_max - m_new);
    const float pe = expf(s - m_new);
    den = den * alpha + pe;
#pragma unroll
    for (int c = 0; c < DT / EP; ++c) {
      float x[DT];
      load_piece(x, c * EP, sV + off(j, c));
#pragma unroll
      for (int e = c * EP; e < (c + 1) * EP; ++e)
        acc[e] = acc[e] * alpha + pe * x[e];
    }
    run_max = m_new;
  }

  // 16 bytes of shared memory -> EP values at x[c0..c0+EP)
  __device__ __forceinline__ static void load_piece(float (&x)[DT], int c0,
                                                    uint32_t addr) {
    uint32_t u[4];
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3])
                 : "r"(addr));
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int e = 0; e < 4; ++e) x[c0 + e] = __uint_as_float(u[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(
            *reinterpret_cast<const __nv_bfloat162*>(&u[e]));
        x[c0 + 2 * e] = f.x;
        x[c0 + 2 * e + 1] = f.y;
      }
    }
  }

  __device__ __forceinline__ void apply2(const AttnParams& p,
                                         const float (&kx)[2][DT],
                                         const float (&vx)[2][DT], int cnt) {
#pragma unroll
    for (int m = 0; m < 2; ++m)
      if (m < cnt) {
        float part[DT / 4];
#pragma unroll
        for (int g = 0; g < DT / 4; ++g) {
          float t = q[4 * g] * kx[m][4 * g];
          t = fmaf(q[4 * g + 1], kx[m][4 * g + 1], t);
          t = fmaf(q[4 * g + 2], kx[m][4 * g + 2], t);
          part[g] = fmaf(q[4 * g + 3], kx[m][4 * g + 3], t);
        }
        float s;
        if constexpr (DT == 16)
          s = (part[0] + part[2]) + (part[1] + part[3]);
        else
          s = part[0] + part[1];
        s *= p.post_scale;
        const float m_new = fmaxf(run_max, s);
        const float alpha = (run_max == -INFINITY) ? 0.f : expf(run_max - m_new);
        const float pe = expf(s - m_new);
        den = den * alpha + pe;
#pragma unroll
        for (int c = 0; c < DT; ++c) acc[c] = acc[c] * alpha + pe * vx[m][c];
        run_max = m_new;
      }
  }

  __device__ __forceinline__ void finish(const AttnParams& p, T* orow,
                                         bool bad) {
    float o[DT];
#pragma unroll
    for (int c = 0; c < DT; ++c)
      o[c] = bad ? __int_as_float(0x7fc00000) : acc[c] / den;
    if (p.vec != 0) {  // d % 4 == 0, 16-byte (8-byte) aligned rows
#pragma unroll
      for (int c = 0; c < DT; c += 4) {
        if (c < p.d) {
          if constexpr (sizeof(T) == 4) {
            *reinterpret_cast<float4*>(orow + c) =
                make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
          } else {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(o[c], o[c + 1]);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(o[c + 2], o[c + 3]);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&lo);
            u.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(orow + c) = u;
          }
        }
      }
      return;
    }
#pragma unroll
    for (int c = 0; c < DT; ++c)
      if (c < p.d) orow[c] = from_f32<T>(o[c]);
  }
};

// ---------------------------------------------------------------------------
// One episode's K and V rows in shared memory (d <= DT <= 16, 16-byte rows)
// ---------------------------------------------------------------------------
// Byte offset of 16-byte piece c of row `row`: the pieces of a row are
// XOR-swizzled by bits of the row index, so the pieces a warp gathers from
// 32 random rows spread over all 8 bank groups (64-byte fp32 rows: bits 1-2;
// 32-byte bf16 rows: bit 2).
template <int DT, typename T>
__device__ __forceinline__ uint32_t kv_piece_off(int row, int c) {
  constexpr int CPR = DT * (int)sizeof(T) / 16;  // 16-byte pieces per row
  const int sw = CPR == 4 ? ((row >> 1) & 3) : (CPR == 2 ? ((row >> 2) & 1) : 0);
  return (uint32_t)(row * CPR + (c ^ sw)) * 16u;
}

// Start 16-byte cp.async copies of episode b's N K rows to sK and V rows to
// sV (shared-window addresses, N * DT * sizeof(T) bytes each); pieces beyond
// d are zero-filled. NT threads; the caller waits (cp_async_wait<0>) and
// synchronises the block before reading.
template <int DT, typename T, int NT>
__device__ __forceinline__ void stage_kv_episode(const AttnParams& p, int b,
                                                 uint32_t sK, uint32_t sV) {
  constexpr int CPR = DT * (int)sizeof(T) / 16;
  constexpr int EP = 16 / (int)sizeof(T);
  const T* Kb = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* Vb = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  for (int e = threadIdx.x; e < p.N * CPR; e += NT) {
    const int r = e / CPR, c = e - r * CPR;
    const uint32_t off = kv_piece_off<DT, T>(r, c);
    if (c * EP < p.d) {
      cp_async16_addr(sK + off, Kb + (int64_t)r * p.st.kn + c * EP);
      cp_async16_addr(sV + off, Vb + (int64_t)r * p.st.vn + c * EP);
    } else {
      st_shared_zero16(sK + off);
      st_shared_zero16(sV + off);
    }
  }
  cp_async_commit();
}

// K and V rows can be staged by whole 16-byte pieces with cp.async
template <typename T>
inline bool kv_stageable(const AttnParams& p) {
  constexpr int EP = 16 / (int)sizeof(T);
  const auto a16 = [](const void* x) {
    return reinterpret_cast<uintptr_t>(x) % 16 == 0;
  };
  return p.vec != 0 && p.d % EP == 0 && a16(p.k) && a16(p.v) &&
         p.st.kb % EP == 0 && p.st.kn % EP == 0 && p.st.vb % EP == 0 &&
         p.st.vn % EP == 0;
}

}  // namespace tarmac
