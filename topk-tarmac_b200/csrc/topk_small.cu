// topk_small.cu — fused top-k attention for short episodes on sm_100a:
// N <= 128, d <= 16, k <= 8, one or two lanes per query row.
//
// Same function as topk_chunk_kernel and the tensor-core kernel (reference:
// src/kernels/fused_topk_attention.py:211-289, streaming_topk_attention.py:
// 66-179; the lowest or the highest index wins a tie at the k-th score). For
// short episodes the chunked kernel's organisation (four warps splitting one
// episode's keys, a merge, then a finalisation on some of the warps) leaves
// most of each block waiting on memory latency. Here:
//
// * Up to 64 agents, ceil(N / 16) warps own one episode with two lanes per
//   query row (each scores every other key and keeps its own k best; the
//   pair then merges the two buffers by shuffles and each lane stores half
//   the row), and a block of four warps carries 4, 2 or 1 episodes. Above 64
//   agents, four warps own one episode, one lane per row. The episode's
//   warps copy its K and V rows into shared memory (16-byte cp.async for
//   aligned fp32 rows, converted through registers otherwise; rows padded to
//   DP + 4 floats) while each lane's Q row loads into registers.
// * Each lane scores its keys with dot_pairs (the key rows are broadcast
//   reads), the arithmetic of the chunked kernel's exact pass, so
//   every score is bit-identical to it, and keeps the k best by (score,
//   index) with the tie rule in a sorted register buffer. NaN scores are
//   never retained (the chunked kernel's threshold test drops them too).
// * Softmax over the k retained scores, V rows gathered from shared memory,
//   the output row and, if asked, the indices in rank order.
#include "topk_chunk.cuh"

namespace tarmac {

constexpr int SMALL_DP = 16;
constexpr int SMALL_MAX_N = 128;

template <typename T>
__device__ __forceinline__ float4 small_cols4(const T* src, int c, int d,
                                              bool vec) {
  if (vec) return load4(src);
  float4 f;
  f.x = to_f32<T>(src[0]);
  f.y = (c + 1 < d) ? to_f32<T>(src[1]) : 0.f;
  f.z = (c + 2 < d) ? to_f32<T>(src[2]) : 0.f;
  f.w = (c + 3 < d) ? to_f32<T>(src[3]) : 0.f;
  return f;
}

template <int KC, int WPE, int SPLIT, int BW, bool TIE_HIGH, typename T>
__global__ void __launch_bounds__(BW * 32)
    topk_small_kernel(AttnParams p) {
  constexpr int DP = SMALL_DP;
  constexpr int EPB = BW / WPE;           // episodes per block
  constexpr int GT = WPE * 32;            // threads of an episode
  constexpr int ROWS = GT / SPLIT;        // rows (= query rows) it holds
  constexpr int KS = DP + 4;
  constexpr int C4 = DP / 4;
  static_assert(SPLIT == 1 || SPLIT == 2, "one or two lanes per query row");
  __shared__ __align__(16) float sk[EPB][ROWS * KS];
  __shared__ __align__(16) float sv[EPB][ROWS * KS];

  const int N = p.N, d = p.d;
  const int warp = threadIdx.x >> 5;
  const int e = warp / WPE;
  const int64_t b = (int64_t)blockIdx.x * EPB + e;
  const int t = threadIdx.x - e * GT;  // thread within the episode
  const int i = t / SPLIT;             // its query row
  const int h = t % SPLIT;             // its share of the keys
  const bool has = b < p.B;
  const bool live = has && i < N;
  const bool vec = p.vec != 0;
  float* sK = sk[e];
  float* sV = sv[e];
  const int64_t bb = has ? b : 0;
  const T* Q = static_cast<const T*>(p.q) + bb * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + bb * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + bb * p.st.vb;
  T* O = static_cast<T*>(p.o) + bb * p.st.ob;

  // ---- the episode's K and V rows into shared memory ----------------------
  if (has) {
    for (int x = t; x < N * C4; x += GT) {
      const int r = x / C4, c = (x % C4) * 4;
      float* dk = sK + r * KS + c;
      float* dv = sV + r * KS + c;
      if (c >= d) {
        *reinterpret_cast<float4*>(dk) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(dv) = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      const T* gk = K + (int64_t)r * p.st.kn + c;
      const T* gv = V + (int64_t)r * p.st.vn + c;
      if constexpr (sizeof(T) == 4) {
        if (vec) {
          cp_async16(dk, gk);
          cp_async16(dv, gv);
          continue;
        }
      }
      *reinterpret_cast<float4*>(dk) = small_cols4<T>(gk, c, d, vec);
      *reinterpret_cast<float4*>(dv) = small_cols4<T>(gv, c, d, vec);
    }
  }

  // ---- this lane's query row (scaled as the chunked kernel scales it) -----
  uint64_t qf[DP / 2];
  {
    float qr[DP];
    if (live) {
      load_row<DP, T>(qr, Q + (int64_t)i * p.st.qn, d, vec);
    } else {
#pragma unroll
      for (int c = 0; c < DP; ++c) qr[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < DP; c += 2)
      qf[c / 2] = pack2(qr[c] * p.qscale, qr[c + 1] * p.qscale);
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- scores and the k best by (score, index) -----------------------------
  float bs[KC];
  int bi[KC];
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    bs[m] = -INFINITY;
    bi[m] = -1;
  }
  if (live) {
#pragma unroll 4
    for (int j = h; j < N; j += SPLIT) {
      const float s = dot_pairs<DP>(qf, sK + j * KS);
      if (j != i && s == s && better<TIE_HIGH>(s, j, bs[KC - 1], bi[KC - 1]))
        ins_idx<KC, TIE_HIGH>(bs, bi, s, j);
    }
  }
  if constexpr (SPLIT == 2) {
    // The pair's buffers hold disjoint keys: each lane merges its partner's
    // into its own by the same (score, index) order, so both end with the k
    // best of the whole row in the same order. Every lane of the warp takes
    // part in the shuffles (lanes past N carry empty buffers); the two lanes
    // of a pair share one query row, so both are live or neither.
    float ps[KC];
    int pi[KC];
#pragma unroll
    for (int m = 0; m < KC; ++m) {
      ps[m] = __shfl_xor_sync(0xffffffffu, bs[m], 1);
      pi[m] = __shfl_xor_sync(0xffffffffu, bi[m], 1);
    }
#pragma unroll
    for (int m = 0; m < KC; ++m)
      if (pi[m] >= 0 && better<TIE_HIGH>(ps[m], pi[m], bs[KC - 1], bi[KC - 1]))
        ins_idx<KC, TIE_HIGH>(bs, bi, ps[m], pi[m]);
  }
  if (!live) return;

  // ---- softmax over the k retained scores, V gather-aggregate -------------
  const int kk = p.topk;
  const float mx = bs[0] * p.post_scale;
  float den = 0.f;
  float ev[KC];
  bool empty = false;
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    ev[m] = (m < kk) ? expf(bs[m] * p.post_scale - mx) : 0.f;
    den += ev[m];
    empty |= (m < kk) && (bi[m] < 0);
  }
  float acc[DP];
#pragma unroll
  for (int c = 0; c < DP; ++c) acc[c] = 0.f;
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    if (m < kk && !empty) {
      const float w = ev[m] / den;
      const float* vr = sV + bi[m] * KS;
#pragma unroll
      for (int c = 0; c < DP; c += 4) {
        const float4 f = *reinterpret_cast<const float4*>(vr + c);
        acc[c] = fmaf(w, f.x, acc[c]);
        acc[c + 1] = fmaf(w, f.y, acc[c + 1]);
        acc[c + 2] = fmaf(w, f.z, acc[c + 2]);
        acc[c + 3] = fmaf(w, f.w, acc[c + 3]);
      }
    }
  }
  if (empty) {
#pragma unroll
    for (int c = 0; c < DP; ++c) acc[c] = __int_as_float(0x7fc00000);
  }
  if constexpr (SPLIT == 1) {
    store_row<DP, T>(O + (int64_t)i * p.st.on, acc, d, vec);
  } else {
    // each lane of the pair stores half of the row's columns
    constexpr int HW = DP / 2;
    float half[HW];
#pragma unroll
    for (int c = 0; c < HW; ++c) half[c] = h ? acc[HW + c] : acc[c];
    if (d > h * HW)
      store_row<HW, T>(O + (int64_t)i * p.st.on + h * HW, half, d - h * HW,
                       vec);
  }
  if (p.idx_out != nullptr && h == 0) {
    int32_t* io = p.idx_out + ((int64_t)bb * N + i) * kk;
#pragma unroll
    for (int m = 0; m < KC; ++m)
      if (m < kk) io[m] = bi[m];
  }
}

template <int KC, int WPE, int SPLIT, int BW, bool TIE_HIGH, typename T>
static cudaError_t launch_small_w(const AttnParams& p, cudaStream_t s) {
  constexpr int EPB = BW / WPE;
  const int64_t blocks = ((int64_t)p.B + EPB - 1) / EPB;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  topk_small_kernel<KC, WPE, SPLIT, BW, TIE_HIGH, T>
      <<<(unsigned)blocks, BW * 32, 0, s>>>(p);
  return cudaGetLastError();
}

// Up to 64 agents a query row takes two lanes (each scores every other
// key: twice the warps, half the chain per lane) and a block of four warps
// carries 4, 2 or 1 episodes. Above, one lane per row in a four-warp block:
// two lanes per row in eight-warp blocks measured slower there (N=100, k=2:
// 22.7 -> 25.7 us at B=1024).
template <int KC, bool TIE_HIGH, typename T>
static cudaError_t launch_small_n(const AttnParams& p, cudaStream_t s) {
  if (p.N <= 16) return launch_small_w<KC, 1, 2, 4, TIE_HIGH, T>(p, s);
  if (p.N <= 32) return launch_small_w<KC, 2, 2, 4, TIE_HIGH, T>(p, s);
  if (p.N <= 64) return launch_small_w<KC, 4, 2, 4, TIE_HIGH, T>(p, s);
  return launch_small_w<KC, 4, 1, 4, TIE_HIGH, T>(p, s);
}

template <bool TIE_HIGH, typename T>
static cudaError_t launch_small_k(const AttnParams& p, cudaStream_t s) {
  switch (chunk_slots(p.topk)) {
    case 1: return launch_small_n<1, TIE_HIGH, T>(p, s);
    case 2: return launch_small_n<2, TIE_HIGH, T>(p, s);
    case 4: return launch_small_n<4, TIE_HIGH, T>(p, s);
    default: return launch_small_n<8, TIE_HIGH, T>(p, s);
  }
}

bool topk_small_supported(const AttnParams& p) {
  return p.N >= 2 && p.N <= SMALL_MAX_N && p.d <= SMALL_DP && p.topk >= 1 &&
         p.topk <= 8;
}

cudaError_t launch_topk_small(const AttnParams& p, int dtype, bool tie_high,
                              cudaStream_t s) {
  if (dtype == TARMAC_BF16)
    return tie_high ? launch_small_k<true, __nv_bfloat16>(p, s)
                    : launch_small_k<false, __nv_bfloat16>(p, s);
  return tie_high ? launch_small_k<true, float>(p, s)
                  : launch_small_k<false, float>(p, s);
}

}  // namespace tarmac
