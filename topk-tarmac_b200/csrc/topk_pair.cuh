// topk_pair.cuh — key-pair chunked top-k attention (k <= 8, d <= 32) on sm_100a.
//
// Same function and selection scheme as topk_chunk.cuh (chunk maxima, a
// running buffer of the k best chunks, exact recompute of the candidates; the
// reference kernels are src/kernels/fused_topk_attention.py:211-289 and
// src/kernels/streaming_topk_attention.py:66-179), with the score loop laid
// out for the packed fp32x2 FMA so that one 64-bit operand is shared by
// consecutive instructions:
//
// * Keys sit in shared memory as interleaved pairs: for keys 2p and 2p+1 the
//   row holds (k_2p[c], k_2p+1[c]) for every column c, padded to 2*DP+4
//   floats. One 16-byte broadcast load yields the operands for columns c and
//   c+1 of both keys.
// * A lane keeps each of its QPT query rows duplicated into both halves,
//   (q[c], q[c]), so fma.rn.f32x2 advances the scores of two keys at once:
//   each half is one ordinary fp32 FMA chain over the columns in order, and
//   the key-pair operand is reused by the QPT queries in a row.
// * A block holds WQ query groups of 32*QPT queries; in each group 4 warps
//   split the keys. The recompute runs the same FMA chains, so candidate
//   scores are bit-identical to the main loop's.
#pragma once

#include "topk_chunk.cuh"

namespace tarmac {

constexpr int PAIR_WQ = 2;                      // query groups per block
constexpr int PAIR_WARPS = PAIR_WQ * CH_WARPS;  // 8 warps

template <int DP>
__host__ __device__ constexpr int pair_row_stride() {
  return 2 * DP + 4;
}

template <int DP, int QPT, int KC, int CH>
__host__ __device__ constexpr size_t pair_smem_bytes(int NC) {
  return (size_t)(NC * CH / 2) * pair_row_stride<DP>() * 4 +
         (size_t)PAIR_WQ * QPT * CH_WARPS * 32 * KC * 8;
}

// Stage key rows [0, 2*npairs) of one episode as interleaved pairs, zero
// beyond N and d; all threads of the block take part, four pair-columns of
// 16-byte loads in flight per thread.
template <int DP, typename T>
__device__ __forceinline__ void stage_pairs(float* __restrict__ sk,
                                            const T* __restrict__ K,
                                            int64_t rs, int npairs, int N,
                                            int d, bool vec) {
  constexpr int C4 = DP / 4;
  constexpr int PS = pair_row_stride<DP>();
  const int total = npairs * C4;
  constexpr int U = 4;
  for (int e0 = threadIdx.x; e0 < total; e0 += U * blockDim.x) {
    float4 a[U], b[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * blockDim.x;
      const int pr = e / C4;
      const int c = (e - pr * C4) * 4;
      a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < total && c < d) {
        const int j = 2 * pr;
        if (j < N) {
          const T* src = K + (int64_t)j * rs + c;
          if (vec) {
            a[u] = load4(src);
          } else {
            a[u].x = to_f32<T>(src[0]);
            a[u].y = (c + 1 < d) ? to_f32<T>(src[1]) : 0.f;
            a[u].z = (c + 2 < d) ? to_f32<T>(src[2]) : 0.f;
            a[u].w = (c + 3 < d) ? to_f32<T>(src[3]) : 0.f;
          }
        }
        if (j + 1 < N) {
          const T* src = K + (int64_t)(j + 1) * rs + c;
          if (vec) {
            b[u] = load4(src);
          } else {
            b[u].x = to_f32<T>(src[0]);
            b[u].y = (c + 1 < d) ? to_f32<T>(src[1]) : 0.f;
            b[u].z = (c + 2 < d) ? to_f32<T>(src[2]) : 0.f;
            b[u].w = (c + 3 < d) ? to_f32<T>(src[3]) : 0.f;
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < total) {
        const int pr = e / C4;
        const int c = (e - pr * C4) * 4;
        float* dst = sk + (size_t)pr * PS + 2 * c;
        *reinterpret_cast<float4*>(dst) = make_float4(a[u].x, b[u].x, a[u].y, b[u].y);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(a[u].z, b[u].z, a[u].w, b[u].w);
      }
    }
  }
}

// Scores of keys (2p, 2p+1) for QPT duplicated query rows: acc[r] holds the
// two scores of query r. `kp` points at the pair's row in shared memory.
template <int DP, int QPT>
__device__ __forceinline__ void pair_scores(const uint64_t (&qd)[QPT][DP],
                                            const float* kp,
                                            uint64_t (&acc)[QPT]) {
#pragma unroll
  for (int r = 0; r < QPT; ++r) acc[r] = 0ull;
#pragma unroll
  for (int c = 0; c < DP; c += 2) {
    const ulonglong2 kv = *reinterpret_cast<const ulonglong2*>(kp + 2 * c);
#pragma unroll
    for (int r = 0; r < QPT; ++r) acc[r] = ffma2(qd[r][c], kv.x, acc[r]);
#pragma unroll
    for (int r = 0; r < QPT; ++r) acc[r] = ffma2(qd[r][c + 1], kv.y, acc[r]);
  }
}

// Two key pairs at once: 2*QPT independent chains in program order.
template <int DP, int QPT>
__device__ __forceinline__ void pair_scores2(const uint64_t (&qd)[QPT][DP],
                                             const float* kp0, const float* kp1,
                                             uint64_t (&a0)[QPT],
                                             uint64_t (&a1)[QPT]) {
#pragma unroll
  for (int r = 0; r < QPT; ++r) a0[r] = a1[r] = 0ull;
#pragma unroll
  for (int c = 0; c < DP; c += 2) {
    const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(kp0 + 2 * c);
    const ulonglong2 y = *reinterpret_cast<const ulonglong2*>(kp1 + 2 * c);
#pragma unroll
    for (int r = 0; r < QPT; ++r) {
      a0[r] = ffma2(qd[r][c], x.x, a0[r]);
      a1[r] = ffma2(qd[r][c], y.x, a1[r]);
    }
#pragma unroll
    for (int r = 0; r < QPT; ++r) {
      a0[r] = ffma2(qd[r][c + 1], x.y, a0[r]);
      a1[r] = ffma2(qd[r][c + 1], y.y, a1[r]);
    }
  }
}

template <int DP, int QPT, int KC, int CH, bool TIE_HIGH, typename T>
__global__ void __launch_bounds__(PAIR_WARPS * 32, 2)
    topk_pair_kernel(AttnParams p, int NC) {
  constexpr int PS = pair_row_stride<DP>();
  constexpr int PPC = CH / 2;  // key pairs per chunk
  constexpr int GQ = 32 * QPT; // queries per group
  extern __shared__ __align__(16) float smem[];
  float* sK = smem;
  float* lv = sK + (size_t)(NC * PPC) * PS;  // [WQ][QPT][warps][32][KC]
  int* li = reinterpret_cast<int*>(lv + PAIR_WQ * QPT * CH_WARPS * 32 * KC);

  const int N = p.N, d = p.d;
  const int bpe = cdiv(N, PAIR_WQ * GQ);  // blocks per episode
  const int b = blockIdx.x / bpe;
  const int qb = (blockIdx.x - b * bpe) * PAIR_WQ * GQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / CH_WARPS, ks = warp % CH_WARPS;
  const int q0 = qb + grp * GQ;  // this warp's query group
  const bool vec = p.vec != 0;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  stage_pairs<DP, T>(sK, K, p.st.kn, NC * PPC, N, d, vec);

  // ---- queries, duplicated into both halves (power-of-two scale folded) ---
  uint64_t qd[QPT][DP];
  int qi[QPT];
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    qi[r] = q0 + r * 32 + lane;
    float qr[DP];
    if (qi[r] < N) {
      load_row<DP, T>(qr, Q + (int64_t)qi[r] * p.st.qn, d, vec);
    } else {
#pragma unroll
      for (int c = 0; c < DP; ++c) qr[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < DP; ++c) {
      const float x = qr[c] * p.qscale;
      qd[r][c] = pack2(x, x);
    }
  }
  __syncthreads();

  // ---- main loop: chunk maxima, running k best chunks --------------------
  float cbv[QPT][KC];
  int cbi[QPT][KC];
#pragma unroll
  for (int r = 0; r < QPT; ++r)
#pragma unroll
    for (int m = 0; m < KC; ++m) {
      cbv[r][m] = -INFINITY;
      cbi[r][m] = -1;
    }
  const int c0 = (ks * NC) / CH_WARPS;
  const int c1 = ((ks + 1) * NC) / CH_WARPS;
  const int diag0 = q0 / CH;                     // chunks holding the group's
  const int diag1 = (q0 + GQ + CH - 1) / CH;     // own keys (the diagonal)
  for (int c = c0; c < c1; ++c) {
    const float* kb = sK + (size_t)c * PPC * PS;
    float cm[QPT];
#pragma unroll
    for (int r = 0; r < QPT; ++r) cm[r] = -INFINITY;
    if ((c + 1) * CH <= N && (c < diag0 || c >= diag1)) {
#pragma unroll
      for (int pp = 0; pp < PPC; pp += 2) {
        uint64_t a0[QPT], a1[QPT];
        pair_scores2<DP, QPT>(qd, kb + pp * PS, kb + (pp + 1) * PS, a0, a1);
#pragma unroll
        for (int r = 0; r < QPT; ++r) {
          const float2 x = unpack2(a0[r]), y = unpack2(a1[r]);
          cm[r] = max3f(cm[r], max3f(x.x, x.y, y.x), y.y);
        }
      }
    } else {
      // partial last chunk or a diagonal chunk: keys >= N (zero rows) and
      // the query's own key do not count
      for (int pp = 0; pp < PPC; ++pp) {
        uint64_t a[QPT];
        pair_scores<DP, QPT>(qd, kb + pp * PS, a);
        const int j0 = c * CH + 2 * pp;
#pragma unroll
        for (int r = 0; r < QPT; ++r) {
          const float2 x = unpack2(a[r]);
          const float s0 = (j0 < N && j0 != qi[r]) ? x.x : -INFINITY;
          const float s1 = (j0 + 1 < N && j0 + 1 != qi[r]) ? x.y : -INFINITY;
          cm[r] = max3f(cm[r], s0, s1);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < QPT; ++r)
      buf_insert<KC, TIE_HIGH>(cbv[r], cbi[r], cm[r], c);
  }

  // ---- publish each warp's chunk lists ------------------------------------
#pragma unroll
  for (int r = 0; r < QPT; ++r)
#pragma unroll
    for (int m = 0; m < KC; ++m) {
      const int o = (((grp * QPT + r) * CH_WARPS + ks) * 32 + lane) * KC + m;
      lv[o] = cbv[r][m];
      li[o] = cbi[r][m];
    }
  __syncthreads();
  if (ks >= QPT) return;

  // ---- finalize: warp ks of the group owns query row r = ks ---------------
  const int r = ks;
  const int i = q0 + r * 32 + lane;
  if (i >= N) return;
  uint64_t qf[1][DP];
  {
    float qr[DP];
    load_row<DP, T>(qr, Q + (int64_t)i * p.st.qn, d, vec);
#pragma unroll
    for (int c = 0; c < DP; ++c) {
      const float x = qr[c] * p.qscale;
      qf[0][c] = pack2(x, x);
    }
  }
  float mv[KC];
  int mi[KC];
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    mv[m] = -INFINITY;
    mi[m] = -1;
  }
  for (int w2 = 0; w2 < CH_WARPS; ++w2) {
#pragma unroll
    for (int m = 0; m < KC; ++m) {
      const int o = (((grp * QPT + r) * CH_WARPS + w2) * 32 + lane) * KC + m;
      const int id = li[o];
      if (id >= 0) ins_idx<KC, TIE_HIGH>(mv, mi, lv[o], id);
    }
  }
  const float thr = mv[KC - 1];  // <= the k-th best score of the row
  float bs[KC];
  int bi[KC];
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    bs[m] = -INFINITY;
    bi[m] = -1;
  }
  // ins_idx orders by (score, index) explicitly, so the visiting order of the
  // candidate pairs does not matter; lanes start at different pairs of their
  // chunk to spread the shared-memory gathers over banks.
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    const int cid = mi[m];
    if (cid < 0) continue;
#pragma unroll
    for (int pp = 0; pp < PPC; ++pp) {
      const int pr = (pp + lane) & (PPC - 1);
      uint64_t a[1];
      pair_scores<DP, 1>(qf, sK + (size_t)(cid * PPC + pr) * PS, a);
      const float2 x = unpack2(a[0]);
      const int j0 = cid * CH + 2 * pr;
      if (j0 < N && j0 != i && x.x >= thr) ins_idx<KC, TIE_HIGH>(bs, bi, x.x, j0);
      if (j0 + 1 < N && j0 + 1 != i && x.y >= thr)
        ins_idx<KC, TIE_HIGH>(bs, bi, x.y, j0 + 1);
    }
  }

  // ---- softmax over the k retained scores, V gather-aggregate -------------
  const int kk = p.topk;
  const float mx = bs[0] * p.post_scale;
  float den = 0.f;
  float e[KC];
  bool empty = false;
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    e[m] = (m < kk) ? expf(bs[m] * p.post_scale - mx) : 0.f;
    den += e[m];
    empty |= (m < kk) && (bi[m] < 0);
  }
  float acc[DP];
#pragma unroll
  for (int c = 0; c < DP; ++c) acc[c] = 0.f;
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    if (m < kk && !empty) {
      const float w = e[m] / den;
      const T* vr = V + (int64_t)bi[m] * p.st.vn;
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
  store_row<DP, T>(O + (int64_t)i * p.st.on, acc, d, vec);
  if (p.idx_out != nullptr) {
    int32_t* io = p.idx_out + ((int64_t)b * N + i) * kk;
#pragma unroll
    for (int m = 0; m < KC; ++m)
      if (m < kk) io[m] = bi[m];
  }
}

// two query rows per lane at d <= 16 (64 registers of duplicated q), one at
// d <= 32 or when 8 chunk slots are kept
template <int DP, int KC>
constexpr int pair_qpt() {
  return (DP >= 32 || KC >= 8) ? 1 : 2;
}

template <int DP, int KC>
size_t pair_smem_for(int N) {
  constexpr int CH = chunk_len(KC);
  return pair_smem_bytes<DP, pair_qpt<DP, KC>(), KC, CH>(cdiv(N, CH));
}

template <int DP>
size_t pair_smem_dp(int N, int topk) {
  switch (chunk_slots(topk)) {
    case 1: return pair_smem_for<DP, 1>(N);
    case 2: return pair_smem_for<DP, 2>(N);
    case 4: return pair_smem_for<DP, 4>(N);
    default: return pair_smem_for<DP, 8>(N);
  }
}

// true when the key-pair kernel serves (d <= 32) and the keys fit
inline bool pair_fits(int N, int d, int topk) {
  if (d > 32) return false;
  const size_t sm = d <= 16 ? pair_smem_dp<16>(N, topk) : pair_smem_dp<32>(N, topk);
  return sm <= CHUNK_SMEM_MAX;
}

template <int DP, int KC, bool TIE_HIGH, typename T>
cudaError_t launch_pair_t(const AttnParams& p, cudaStream_t s) {
  constexpr int QPT = pair_qpt<DP, KC>();
  constexpr int CH = chunk_len(KC);
  const int NC = cdiv(p.N, CH);
  const size_t sm = pair_smem_bytes<DP, QPT, KC, CH>(NC);
  cudaError_t e = cudaFuncSetAttribute(
      topk_pair_kernel<DP, QPT, KC, CH, TIE_HIGH, T>,
      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.B * cdiv(p.N, PAIR_WQ * 32 * QPT);
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  topk_pair_kernel<DP, QPT, KC, CH, TIE_HIGH, T>
      <<<(unsigned)blocks, PAIR_WARPS * 32, sm, s>>>(p, NC);
  return cudaGetLastError();
}

template <int DP, bool TIE_HIGH, typename T>
cudaError_t launch_pair_kc(const AttnParams& p, cudaStream_t s) {
  switch (chunk_slots(p.topk)) {
    case 1: return launch_pair_t<DP, 1, TIE_HIGH, T>(p, s);
    case 2: return launch_pair_t<DP, 2, TIE_HIGH, T>(p, s);
    case 4: return launch_pair_t<DP, 4, TIE_HIGH, T>(p, s);
    default: return launch_pair_t<DP, 8, TIE_HIGH, T>(p, s);
  }
}

// Resident-key top-k for one element type and tie rule (one translation unit
// each, compiled in parallel): the key-pair kernel for d <= 32, the
// column-pair chunked kernel above; the caller has checked resident_fits.
template <bool TIE_HIGH, typename T>
cudaError_t launch_resident_dt(const AttnParams& p, cudaStream_t s) {
  if (pair_fits(p.N, p.d, p.topk)) {
    if (p.d <= 16) return launch_pair_kc<16, TIE_HIGH, T>(p, s);
    return launch_pair_kc<32, TIE_HIGH, T>(p, s);
  }
  if (p.d <= 16) return launch_chunk_kc<16, TIE_HIGH, T>(p, s);
  if (p.d <= 32) return launch_chunk_kc<32, TIE_HIGH, T>(p, s);
  if (p.d <= 64) return launch_chunk_kc<64, TIE_HIGH, T>(p, s);
  return launch_chunk_kc<128, TIE_HIGH, T>(p, s);
}

// true when one of the resident-key kernels can hold the episode's keys
inline bool resident_fits(int N, int d, int topk) {
  return pair_fits(N, d, topk) || chunk_fits(N, d, topk);
}

}  // namespace tarmac
