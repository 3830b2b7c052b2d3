// topk_chunk.cuh — resident-key chunked top-k attention (k <= 8) on sm_100a.
//
// Same function as the streaming register-buffer kernel (reference:
// src/kernels/fused_topk_attention.py:211-289, streaming_topk_attention.py:
// 66-179; lowest or highest index wins a tie at the k-th score), organised so
// that selection costs about one instruction per score instead of a compare,
// a branch and a divergent buffer insertion:
//
// * The episode's K rows are staged once into shared memory (fp32, rows padded
//   to DP+4 floats). A block owns 32*QPT queries (QPT per lane, q in
//   registers as fp32 pairs) and its 4 warps split the keys into contiguous
//   ranges of CH-key chunks (CH = 4, 8 or 16 for k <= 2, 4, 8).
// * Scores use the packed fp32x2 FMA (fma.rn.f32x2): even and odd columns
//   accumulate in the two halves and are added at the end. Two keys are
//   scored against all QPT queries in lock-step, so 2*QPT independent FMA
//   chains are interleaved in program order.
// * Per query and chunk only the chunk maximum is formed (three-input max),
//   and a branch-free running buffer keeps the k best chunks, ordered by
//   (maximum, chunk index) with the tie rule. The k best scores of the row lie
//   in those k chunks: any other chunk has k chunk maxima above its own, each
//   the maximum of a distinct score that beats all of its scores. The
//   diagonal is masked only in the chunks that can hold it for this block's
//   queries (a warp-uniform test per chunk).
// * The warps' chunk lists are merged through shared memory; each lane then
//   recomputes — bit-identically — the scores of its query's k candidate
//   chunks and keeps the k best by (score, index) with the tie rule. Only
//   scores >= the k-th chunk maximum (a lower bound of the k-th score) reach
//   the exact buffer.
#pragma once

#include "topk_stream.cuh"

namespace tarmac {

constexpr int CH_WARPS = 4;  // warps per block (they split the keys)

// (a, ia) precedes (b, ib) in the retained order: score descending, ties by
// index ascending (lowest wins) or descending (highest wins); an empty slot
// (ib < 0) is preceded by everything.
template <bool TIE_HIGH>
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  return ib < 0 || a > b || (a == b && (TIE_HIGH ? ia > ib : ia < ib));
}

template <int KM, bool TIE_HIGH>
__device__ __forceinline__ void ins_idx(float (&bs)[KM], int (&bi)[KM],
                                        float s, int j) {
#pragma unroll
  for (int p = KM - 1; p >= 1; --p) {
    const bool here = better<TIE_HIGH>(s, j, bs[p], bi[p]);
    const bool above = better<TIE_HIGH>(s, j, bs[p - 1], bi[p - 1]);
    const float ns = above ? bs[p - 1] : (here ? s : bs[p]);
    const int ni = above ? bi[p - 1] : (here ? j : bi[p]);
    bs[p] = ns;
    bi[p] = ni;
  }
  if (better<TIE_HIGH>(s, j, bs[0], bi[0])) {
    bs[0] = s;
    bi[0] = j;
  }
}

// Scores of two key rows (shared memory, 16-byte aligned) against QPT query
// rows, chains interleaved; each score is accumulated in exactly the order
// of dot_pairs, so the final recompute reproduces it bit for bit.
template <int DP, int QPT>
__device__ __forceinline__ void dot2keys(const uint64_t (&qp)[QPT][DP / 2],
                                         const float* k0, const float* k1,
                                         float (&s0)[QPT], float (&s1)[QPT]) {
  uint64_t a0[QPT], a1[QPT];
#pragma unroll
  for (int r = 0; r < QPT; ++r) a0[r] = a1[r] = 0ull;
#pragma unroll
  for (int c = 0; c < DP; c += 4) {
    const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(k0 + c);
    const ulonglong2 y = *reinterpret_cast<const ulonglong2*>(k1 + c);
#pragma unroll
    for (int r = 0; r < QPT; ++r) {
      a0[r] = ffma2(qp[r][c / 2], x.x, a0[r]);
      a1[r] = ffma2(qp[r][c / 2], y.x, a1[r]);
    }
#pragma unroll
    for (int r = 0; r < QPT; ++r) {
      a0[r] = ffma2(qp[r][c / 2 + 1], x.y, a0[r]);
      a1[r] = ffma2(qp[r][c / 2 + 1], y.y, a1[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    s0[r] = hsum2(a0[r]);
    s1[r] = hsum2(a1[r]);
  }
}

template <int DP>
__host__ __device__ constexpr int chunk_row_stride() {
  return DP + 4;  // padding spreads the recompute's row gathers over banks
}

template <int DP, int QPT, int KC, int CH>
__host__ __device__ constexpr size_t chunk_smem_bytes(int NC) {
  return (size_t)NC * CH * chunk_row_stride<DP>() * 4 +
         (size_t)QPT * CH_WARPS * 32 * KC * 8;
}

template <int DP, int QPT, int KC, int CH, bool TIE_HIGH, typename T>
__global__ void __launch_bounds__(CH_WARPS * 32, DP >= 128 ? 2 : 4)
    topk_chunk_kernel(AttnParams p, int NC) {
  constexpr int KS = chunk_row_stride<DP>();
  extern __shared__ __align__(16) float smem[];
  float* sK = smem;
  float* lv = sK + (size_t)NC * CH * KS;          // [QPT][warps][32][KC]
  int* li = reinterpret_cast<int*>(lv + QPT * CH_WARPS * 32 * KC);

  const int N = p.N, d = p.d;
  const int gpe = cdiv(N, 32 * QPT);
  const int b = blockIdx.x / gpe;
  const int g = blockIdx.x - b * gpe;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool vec = p.vec != 0;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  // ---- stage the episode's keys: rows [0, NC*CH), zero beyond N and d ----
  stage_rows<DP, T>(sK, KS, K, p.st.kn, 0, NC * CH, N, d, vec);

  // ---- queries as column pairs -------------------------------------------
  uint64_t qp[QPT][DP / 2];
  int qi[QPT];
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    qi[r] = g * 32 * QPT + r * 32 + lane;
    float qr[DP];
    if (qi[r] < N) {
      load_row<DP, T>(qr, Q + (int64_t)qi[r] * p.st.qn, d, vec);
    } else {
#pragma unroll
      for (int c = 0; c < DP; ++c) qr[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < DP; c += 2)
      qp[r][c / 2] = pack2(qr[c] * p.qscale, qr[c + 1] * p.qscale);
  }
  cp_async_wait_all();
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
  const int c0 = (warp * NC) / CH_WARPS;
  const int c1 = ((warp + 1) * NC) / CH_WARPS;
  // chunks holding this block's diagonal (keys g*32*QPT ... +32*QPT-1)
  const int diag0 = (g * 32 * QPT) / CH;
  const int diag1 = (g * 32 * QPT + 32 * QPT + CH - 1) / CH;
  for (int c = c0; c < c1; ++c) {
    const float* kb = sK + (size_t)c * CH * KS;
    float cm[QPT];
#pragma unroll
    for (int r = 0; r < QPT; ++r) cm[r] = -INFINITY;
    const bool plain = (c + 1) * CH <= N && (c < diag0 || c >= diag1);
    if (plain) {
#pragma unroll
      for (int jj = 0; jj < CH; jj += 2) {
        float s0[QPT], s1[QPT];
        dot2keys<DP, QPT>(qp, kb + jj * KS, kb + (jj + 1) * KS, s0, s1);
#pragma unroll
        for (int r = 0; r < QPT; ++r) cm[r] = max3f(cm[r], s0[r], s1[r]);
      }
    } else {
      // partial last chunk or a diagonal chunk: keys >= N (zero rows in
      // shared memory) and the query's own key do not count
      for (int jj = 0; jj < CH; jj += 2) {
        float s0[QPT], s1[QPT];
        dot2keys<DP, QPT>(qp, kb + jj * KS, kb + (jj + 1) * KS, s0, s1);
        const int j0 = c * CH + jj;
#pragma unroll
        for (int r = 0; r < QPT; ++r) {
          const float a = (j0 < N && j0 != qi[r]) ? s0[r] : -INFINITY;
          const float e = (j0 + 1 < N && j0 + 1 != qi[r]) ? s1[r] : -INFINITY;
          cm[r] = max3f(cm[r], a, e);
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
      const int o = ((r * CH_WARPS + warp) * 32 + lane) * KC + m;
      lv[o] = cbv[r][m];
      li[o] = cbi[r][m];
    }
  __syncthreads();
  if (warp >= QPT) return;

  // ---- finalize: warp w owns query row r = w of this lane -----------------
  const int r = warp;
  const int i = g * 32 * QPT + r * 32 + lane;
  if (i >= N) return;
  uint64_t qf[DP / 2];
  {
    float qr[DP];
    load_row<DP, T>(qr, Q + (int64_t)i * p.st.qn, d, vec);
#pragma unroll
    for (int c = 0; c < DP; c += 2)
      qf[c / 2] = pack2(qr[c] * p.qscale, qr[c + 1] * p.qscale);
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
      const int o = ((r * CH_WARPS + w2) * 32 + lane) * KC + m;
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
  // Each lane walks its own candidate chunks. Chunk bases are bank-aligned,
  // so every lane starts at a different row of its chunk ((jj + lane) mod CH):
  // rows r and r+1 sit DP+4 floats apart, which puts 8 consecutive lanes on 8
  // distinct 4-bank groups. ins_idx orders by (score, index) explicitly, so
  // the visiting order does not matter.
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    const int cid = mi[m];
    if (cid < 0) continue;
    const int nk = min(CH, N - cid * CH);
#pragma unroll 4
    for (int jj = 0; jj < CH; ++jj) {
      const int jr = (jj + lane) & (CH - 1);
      const int j = cid * CH + jr;
      const float s = dot_pairs<DP>(qf, sK + (size_t)j * KS);
      if (jr < nk && j != i && s >= thr) ins_idx<KC, TIE_HIGH>(bs, bi, s, j);
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

// QPT query rows per lane: q pairs (QPT * DP regs) plus 2 * QPT * KC chunk
// slots must stay within the register budget.
template <int DP, int KC>
constexpr int chunk_qpt() {
  return DP >= 64 ? 1 : (DP >= 32 ? (KC >= 8 ? 1 : 2) : (KC >= 8 ? 2 : 4));
}

// Keys per chunk for KC chunk slots: short chunks keep the final recompute
// (KC * CH scores per query) small; the per-chunk buffer update (about 4 KC
// instructions per query) must stay well below the chunk's FMA-pipe time.
constexpr int chunk_len(int KC) { return KC <= 2 ? 4 : (KC <= 4 ? 8 : 16); }

// Largest dynamic shared memory the chunked kernel may take per block.
constexpr size_t CHUNK_SMEM_MAX = 200 * 1024;

// chunk slots: the k-bucket {1, 2, 4, 8} holding k
constexpr int chunk_slots(int topk) {
  return topk <= 1 ? 1 : (topk <= 2 ? 2 : (topk <= 4 ? 4 : 8));
}

template <int DP, int KC>
size_t chunk_smem_for(int N) {
  constexpr int CH = chunk_len(KC);
  return chunk_smem_bytes<DP, chunk_qpt<DP, KC>(), KC, CH>(cdiv(N, CH));
}

template <int DP>
size_t chunk_smem_dp(int N, int topk) {
  switch (chunk_slots(topk)) {
    case 1: return chunk_smem_for<DP, 1>(N);
    case 2: return chunk_smem_for<DP, 2>(N);
    case 4: return chunk_smem_for<DP, 4>(N);
    default: return chunk_smem_for<DP, 8>(N);
  }
}

// true when the episode's keys fit the chunked kernel's shared memory
inline bool chunk_fits(int N, int d, int topk) {
  size_t sm;
  if (d <= 16) sm = chunk_smem_dp<16>(N, topk);
  else if (d <= 32) sm = chunk_smem_dp<32>(N, topk);
  else if (d <= 64) sm = chunk_smem_dp<64>(N, topk);
  else sm = chunk_smem_dp<128>(N, topk);
  return sm <= CHUNK_SMEM_MAX;
}

template <int DP, int KC, bool TIE_HIGH, typename T, int QPT>
cudaError_t launch_chunk_q(const AttnParams& p, cudaStream_t s) {
  constexpr int CH = chunk_len(KC);
  const int NC = cdiv(p.N, CH);
  const size_t sm = chunk_smem_bytes<DP, QPT, KC, CH>(NC);
  cudaError_t e = raise_smem_limit(
      (const void*)topk_chunk_kernel<DP, QPT, KC, CH, TIE_HIGH, T>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.B * cdiv(p.N, 32 * QPT);
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  topk_chunk_kernel<DP, QPT, KC, CH, TIE_HIGH, T>
      <<<(unsigned)blocks, CH_WARPS * 32, sm, s>>>(p, NC);
  return cudaGetLastError();
}

// Queries per lane: the register-budget maximum, lowered for short episodes
// at d <= 16 so that a block's 32 * QPT query rows do not run far past N
// (every warp issues the work of all QPT rows per key, live or not, and
// fewer rows per lane take fewer registers, so more blocks fit an SM).
template <int DP, int KC, bool TIE_HIGH, typename T>
cudaError_t launch_chunk_t(const AttnParams& p, cudaStream_t s) {
  constexpr int QMAX = chunk_qpt<DP, KC>();
  if constexpr (DP <= 16 && QMAX >= 2) {
    if (p.N <= 32) return launch_chunk_q<DP, KC, TIE_HIGH, T, 1>(p, s);
    if constexpr (QMAX >= 4)
      if (p.N <= 64) return launch_chunk_q<DP, KC, TIE_HIGH, T, 2>(p, s);
  }
  return launch_chunk_q<DP, KC, TIE_HIGH, T, QMAX>(p, s);
}

template <int DP, bool TIE_HIGH, typename T>
cudaError_t launch_chunk_kc(const AttnParams& p, cudaStream_t s) {
  switch (chunk_slots(p.topk)) {
    case 1: return launch_chunk_t<DP, 1, TIE_HIGH, T>(p, s);
    case 2: return launch_chunk_t<DP, 2, TIE_HIGH, T>(p, s);
    case 4: return launch_chunk_t<DP, 4, TIE_HIGH, T>(p, s);
    default: return launch_chunk_t<DP, 8, TIE_HIGH, T>(p, s);
  }
}

// One element type and tie rule per translation unit (compile in parallel).
template <bool TIE_HIGH, typename T>
cudaError_t launch_chunk_dt(const AttnParams& p, cudaStream_t s) {
  if (p.d <= 16) return launch_chunk_kc<16, TIE_HIGH, T>(p, s);
  if (p.d <= 32) return launch_chunk_kc<32, TIE_HIGH, T>(p, s);
  if (p.d <= 64) return launch_chunk_kc<64, TIE_HIGH, T>(p, s);
  return launch_chunk_kc<128, TIE_HIGH, T>(p, s);
}

}  // namespace tarmac
