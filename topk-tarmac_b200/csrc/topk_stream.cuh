// topk_stream.cuh — streaming register-buffer top-k attention (k <= 8).
//
// Restates the fused score-then-select top-k of the reference
// (src/kernels/fused_topk_attention.py:211-289 and
// src/kernels/streaming_topk_attention.py:66-179) with a different design:
// one thread owns QPT query rows of one episode and keeps, in registers, a
// sorted buffer of the KM best (score, index) pairs seen so far. Keys stream
// through shared memory in tiles and are read with broadcast loads, so every
// lane of a warp scores the same key against its own queries; no score row is
// ever resident or written. After the last tile the first k buffer entries are
// the retained set; a softmax over them and a gather-aggregate of their V rows
// produce the output row.
//
// Tie rule. Keys arrive in increasing index order. With a strict compare a
// later key never displaces an equal earlier one, so the lowest index wins a
// tie (the argmax-round and streaming kernels of the reference); with a
// non-strict compare the highest index wins (the reference's sort kernel).
// Instantiated per element type by topk_stream_f32.cu / topk_stream_bf16.cu.
#pragma once

#include "common.cuh"

namespace tarmac {

template <bool TIE_HIGH>
__device__ __forceinline__ bool beats(float a, float b) {
  return TIE_HIGH ? (a >= b) : (a > b);
}

// Insert (s, j) into the descending buffer (bs, bi) of KM entries; entries at
// and below the insertion point shift down by one and the last one drops.
template <int KM, bool TIE_HIGH>
__device__ __forceinline__ void buf_insert(float (&bs)[KM], int (&bi)[KM],
                                           float s, int j) {
#pragma unroll
  for (int p = KM - 1; p >= 1; --p) {
    const bool here = beats<TIE_HIGH>(s, bs[p]);
    const bool above = beats<TIE_HIGH>(s, bs[p - 1]);
    const float ns = above ? bs[p - 1] : (here ? s : bs[p]);
    const int ni = above ? bi[p - 1] : (here ? j : bi[p]);
    bs[p] = ns;
    bi[p] = ni;
  }
  if (beats<TIE_HIGH>(s, bs[0])) {
    bs[0] = s;
    bi[0] = j;
  }
}

template <int DP>
__host__ __device__ constexpr int stream_tile_keys() {
  return 16384 / (DP * 4);  // 16 KB of fp32 keys per tile
}

template <int DP, int QPT, int KM, bool TIE_HIGH, typename T>
__global__ void __launch_bounds__(128) topk_stream_kernel(AttnParams p) {
  constexpr int TK = stream_tile_keys<DP>();
  __shared__ __align__(16) float sk[TK * DP];

  const int N = p.N, d = p.d;
  const int groups = cdiv(N, 32 * QPT);  // warp groups per episode
  const int wpb = blockDim.x >> 5;       // warps per block
  const int cpe = cdiv(groups, wpb);     // blocks per episode
  const int b = blockIdx.x / cpe;
  const int chunk = blockIdx.x - b * cpe;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = chunk * wpb + warp;  // this warp's group
  const bool vec = p.vec != 0;
  const bool active = g < groups;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  int qi[QPT];
  float q[QPT][DP];
  float bs[QPT][KM];
  int bi[QPT][KM];
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    qi[r] = g * 32 * QPT + r * 32 + lane;
    if (active && qi[r] < N) {
      load_row<DP, T>(q[r], Q + (int64_t)qi[r] * p.st.qn, d, vec);
#pragma unroll
      for (int c = 0; c < DP; ++c) q[r][c] *= p.qscale;
    } else {
#pragma unroll
      for (int c = 0; c < DP; ++c) q[r][c] = 0.f;
    }
#pragma unroll
    for (int m = 0; m < KM; ++m) {
      bs[r][m] = -INFINITY;
      bi[r][m] = -1;
    }
  }

  for (int t0 = 0; t0 < N; t0 += TK) {
    __syncthreads();
    stage_rows<DP, T>(sk, DP, K, p.st.kn, t0, TK, N, d, vec);
    cp_async_wait_all();
    __syncthreads();
    if (!active) continue;
    const int nk = min(TK, N - t0);
#pragma unroll 2
    for (int jj = 0; jj < nk; ++jj) {
      const float* kr = sk + jj * DP;
      float s[QPT];
#pragma unroll
      for (int r = 0; r < QPT; ++r) s[r] = 0.f;
#pragma unroll
      for (int c = 0; c < DP; c += 4) {
        const float4 kv = *reinterpret_cast<const float4*>(kr + c);
#pragma unroll
        for (int r = 0; r < QPT; ++r) {
          s[r] = fmaf(q[r][c], kv.x, s[r]);
          s[r] = fmaf(q[r][c + 1], kv.y, s[r]);
          s[r] = fmaf(q[r][c + 2], kv.z, s[r]);
          s[r] = fmaf(q[r][c + 3], kv.w, s[r]);
        }
      }
      const int j = t0 + jj;
#pragma unroll
      for (int r = 0; r < QPT; ++r) {
        if (beats<TIE_HIGH>(s[r], bs[r][KM - 1]) && j != qi[r])
          buf_insert<KM, TIE_HIGH>(bs[r], bi[r], s[r], j);
      }
    }
  }
  if (!active) return;

  const int kk = p.topk;
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    if (qi[r] >= N) continue;
    // softmax over the k retained scores, scaled as the reference scales
    const float mx = bs[r][0] * p.post_scale;
    float den = 0.f;
    float e[KM];
#pragma unroll
    for (int m = 0; m < KM; ++m) {
      e[m] = (m < kk) ? expf(bs[r][m] * p.post_scale - mx) : 0.f;
      den += e[m];
    }
    float acc[DP];
#pragma unroll
    for (int c = 0; c < DP; ++c) acc[c] = 0.f;
    // A slot left empty (index -1) means fewer than k comparable scores (NaN
    // scores never enter the buffer): the row is NaN, nothing is read.
    bool empty = false;
#pragma unroll
    for (int m = 0; m < KM; ++m) empty |= (m < kk) && (bi[r][m] < 0);
#pragma unroll
    for (int m = 0; m < KM; ++m) {
      if (m < kk && !empty) {
        const float w = e[m] / den;
        const T* vr = V + (int64_t)bi[r][m] * p.st.vn;
#pragma unroll
        for (int c = 0; c < DP; c += 4) {
          if (c < d) {
            float4 f;
            if (vec) {
              f = load4(vr + c);
            } else {
              f.x = to_f32<T>(vr[c]);
              f.y = (c + 1 < d) ? to_f32<T>(vr[c + 1]) : 0.f;
              f.z = (c + 2 < d) ? to_f32<T>(vr[c + 2]) : 0.f;
              f.w = (c + 3 < d) ? to_f32<T>(vr[c + 3]) : 0.f;
            }
            acc[c] = fmaf(w, f.x, acc[c]);
            acc[c + 1] = fmaf(w, f.y, acc[c + 1]);
            acc[c + 2] = fmaf(w, f.z, acc[c + 2]);
            acc[c + 3] = fmaf(w, f.w, acc[c + 3]);
          }
        }
      }
    }
    if (empty) {
#pragma unroll
      for (int c = 0; c < DP; ++c) acc[c] = __int_as_float(0x7fc00000);
    }
    store_row<DP, T>(O + (int64_t)qi[r] * p.st.on, acc, d, vec);
    if (p.idx_out != nullptr) {
      int32_t* io = p.idx_out + ((int64_t)b * N + qi[r]) * kk;
#pragma unroll
      for (int m = 0; m < KM; ++m)
        if (m < kk) io[m] = bi[r][m];
    }
  }
}

// QPT query rows per thread: register budget for q (QPT * DP) and buffers.
template <int DP>
constexpr int stream_qpt() {
  return DP >= 64 ? 1 : (DP >= 32 ? 2 : 4);
}

template <int DP, int KM, bool TIE_HIGH, typename T>
cudaError_t launch_stream_t(const AttnParams& p, cudaStream_t s) {
  constexpr int QPT = stream_qpt<DP>();
  const int groups = cdiv(p.N, 32 * QPT);
  const int wpb = groups < 4 ? groups : 4;
  const int cpe = cdiv(groups, wpb);
  const int64_t blocks = (int64_t)p.B * cpe;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  topk_stream_kernel<DP, QPT, KM, TIE_HIGH, T>
      <<<(unsigned)blocks, 32 * wpb, 0, s>>>(p);
  return cudaGetLastError();
}

template <int DP, bool TIE_HIGH, typename T>
cudaError_t launch_stream_km(const AttnParams& p, cudaStream_t s) {
  const int k = p.topk;
  if (k <= 1) return launch_stream_t<DP, 1, TIE_HIGH, T>(p, s);
  if (k <= 2) return launch_stream_t<DP, 2, TIE_HIGH, T>(p, s);
  if (k <= 4) return launch_stream_t<DP, 4, TIE_HIGH, T>(p, s);
  return launch_stream_t<DP, 8, TIE_HIGH, T>(p, s);
}

template <typename T>
cudaError_t launch_stream_dt(const AttnParams& p, bool tie_high,
                             cudaStream_t s) {
  if (p.d <= 16)
    return tie_high ? launch_stream_km<16, true, T>(p, s)
                    : launch_stream_km<16, false, T>(p, s);
  if (p.d <= 32)
    return tie_high ? launch_stream_km<32, true, T>(p, s)
                    : launch_stream_km<32, false, T>(p, s);
  if (p.d <= 64)
    return tie_high ? launch_stream_km<64, true, T>(p, s)
                    : launch_stream_km<64, false, T>(p, s);
  return tie_high ? launch_stream_km<128, true, T>(p, s)
                  : launch_stream_km<128, false, T>(p, s);
}

}  // namespace tarmac
