// topk_rows.cu — resident-row top-k attention: any k, three tie rules, N <= 1024.
//
// Covers the reference's kernels whose semantics the streaming register
// buffer cannot express: the threshold (bisection) kernel that keeps every
// peer tied with the k-th score (src/kernels/fused_topk_attention.py:127-208)
// and selections with k > 8 for the argmax-round and sort kernels
// (src/kernels/fused_topk_attention.py:211-289, 405-504).
//
// One warp owns one query row. Lane l scores keys l, l+32, ... (the row is
// staged in shared memory), the scores are mapped to order-preserving 32-bit
// keys (the unsigned form of _float_to_ordered_int, fused_topk_attention.py:
// 113-124) and held 32 per lane in registers. An exact bitwise search, from
// the most significant bit down, finds T = the k-th largest key with
// multiplicity; every step counts keys >= candidate with one warp-wide
// integer reduction. Peers above T are retained, and peers tied at T by the
// mode: the lowest-index ones (ARGMAX), the highest-index ones (SORT), or all
// (THRESHOLD). Softmax over the retained scores; each lane gathers its
// retained V rows and a butterfly reduction forms the output row.
#include "common.cuh"

namespace tarmac {

constexpr int ROWS_MAX_N = 1024;
constexpr int ROWS_SLOTS = ROWS_MAX_N / 32;
constexpr int ROWS_WARPS = 4;

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

template <typename T>
__device__ __forceinline__ float4 cols4(const T* row, int c, int d, bool vec) {
  float4 f;
  if (vec) {
    f = load4(row + c);
  } else {
    f.x = to_f32<T>(row[c]);
    f.y = (c + 1 < d) ? to_f32<T>(row[c + 1]) : 0.f;
    f.z = (c + 2 < d) ? to_f32<T>(row[c + 2]) : 0.f;
    f.w = (c + 3 < d) ? to_f32<T>(row[c + 3]) : 0.f;
  }
  return f;
}

template <int DP, typename T>
__global__ void __launch_bounds__(ROWS_WARPS * 32) topk_rows_kernel(AttnParams p) {
  __shared__ __align__(16) float sq[ROWS_WARPS][DP];
  __shared__ float ssc[ROWS_WARPS][ROWS_MAX_N];
  const int N = p.N, d = p.d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * ROWS_WARPS + warp;
  if (row >= (int64_t)p.B * N) return;  // warp-uniform
  const int b = (int)(row / N);
  const int i = (int)(row - (int64_t)b * N);
  const bool vec = p.vec != 0;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  for (int c = lane * 4; c < DP; c += 128) {
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < d) f = cols4<T>(Q + (int64_t)i * p.st.qn, c, d, vec);
    sq[warp][c] = f.x * p.qscale;
    sq[warp][c + 1] = f.y * p.qscale;
    sq[warp][c + 2] = f.z * p.qscale;
    sq[warp][c + 3] = f.w * p.qscale;
  }
  __syncwarp();

  // scores of keys lane + 32 t
  const int slots = cdiv(N, 32);
#pragma unroll 1
  for (int t = 0; t < slots; ++t) {
    const int j = lane + 32 * t;
    if (j < N) {
      const T* kr = K + (int64_t)j * p.st.kn;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < DP; c += 4) {
        if (c < d) {
          const float4 f = cols4<T>(kr, c, d, vec);
          const float4 qv = *reinterpret_cast<const float4*>(&sq[warp][c]);
          s = fmaf(qv.x, f.x, s);
          s = fmaf(qv.y, f.y, s);
          s = fmaf(qv.z, f.z, s);
          s = fmaf(qv.w, f.w, s);
        }
      }
      ssc[warp][j] = s;
    }
  }
  __syncwarp();

  // order-preserving keys; excluded slots (j >= N, j == i) get key 0, which
  // lies below the key of every non-NaN score
  uint32_t key[ROWS_SLOTS];
#pragma unroll
  for (int t = 0; t < ROWS_SLOTS; ++t) {
    const int j = lane + 32 * t;
    key[t] = (t < slots && j < N && j != i) ? ordered_key(ssc[warp][j]) : 0u;
  }

  // T = the largest value with at least k keys >= it
  const int kk = p.topk;
  uint32_t thr = 0u;
#pragma unroll 1
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = thr | (1u << bit);
    int c = 0;
#pragma unroll
    for (int t = 0; t < ROWS_SLOTS; ++t) c += (key[t] >= cand) ? 1 : 0;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= kk) thr = cand;
  }
  int gt = 0, eq = 0;
#pragma unroll
  for (int t = 0; t < ROWS_SLOTS; ++t) {
    gt += (key[t] > thr) ? 1 : 0;
    eq += (key[t] == thr) ? 1 : 0;
  }
  gt = __reduce_add_sync(0xffffffffu, gt);
  eq = __reduce_add_sync(0xffffffffu, eq);
  const int need = kk - gt;  // tied peers to retain (ARGMAX / SORT)

  // retained slots; ties ranked in index order (slot t, then lane)
  uint32_t selmask = 0u;
  int before = 0;
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int t = 0; t < ROWS_SLOTS; ++t) {
    const bool tie = key[t] == thr;
    const uint32_t bal = __ballot_sync(0xffffffffu, tie);
    const int rank = before + __popc(bal & lt);
    before += __popc(bal);
    bool keep = key[t] > thr;
    if (tie) {
      if (p.mode == TARMAC_SELECT_ARGMAX) keep = rank < need;
      else if (p.mode == TARMAC_SELECT_SORT) keep = rank >= eq - need;
      else keep = true;
    }
    if (keep) selmask |= 1u << t;
  }

  // only real peers can be read: drop any slot outside [0, N) or the diagonal
  // (possible only when NaN scores push the threshold down to key 0)
#pragma unroll
  for (int t = 0; t < ROWS_SLOTS; ++t) {
    const int j = lane + 32 * t;
    if (t >= slots || j >= N || j == i) selmask &= ~(1u << t);
  }

  float mx = -INFINITY;
#pragma unroll 1
  for (int t = 0; t < slots; ++t)
    if ((selmask >> t) & 1u) mx = fmaxf(mx, ssc[warp][lane + 32 * t] * p.post_scale);
  mx = warp_max(mx);

  float den = 0.f;
  float acc[DP];
#pragma unroll
  for (int c = 0; c < DP; ++c) acc[c] = 0.f;
#pragma unroll 1
  for (int t = 0; t < slots; ++t) {
    if ((selmask >> t) & 1u) {
      const int j = lane + 32 * t;
      const float e = expf(ssc[warp][j] * p.post_scale - mx);
      den += e;
      const T* vr = V + (int64_t)j * p.st.vn;
#pragma unroll
      for (int c = 0; c < DP; c += 4) {
        if (c < d) {
          const float4 f = cols4<T>(vr, c, d, vec);
          acc[c] = fmaf(e, f.x, acc[c]);
          acc[c + 1] = fmaf(e, f.y, acc[c + 1]);
          acc[c + 2] = fmaf(e, f.z, acc[c + 2]);
          acc[c + 3] = fmaf(e, f.w, acc[c + 3]);
        }
      }
    }
  }
  den = warp_sum(den);
  const float inv = 1.0f / den;
#pragma unroll
  for (int c = 0; c < DP; ++c) acc[c] = warp_sum(acc[c]) * inv;
  if (lane == 0) store_row<DP, T>(O + (int64_t)i * p.st.on, acc, d, vec);
}

template <int DP, typename T>
static cudaError_t launch_rows_dp(const AttnParams& p, cudaStream_t s) {
  const int64_t rows = (int64_t)p.B * p.N;
  const int64_t blocks = (rows + ROWS_WARPS - 1) / ROWS_WARPS;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  topk_rows_kernel<DP, T><<<(unsigned)blocks, ROWS_WARPS * 32, 0, s>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_rows_dt(const AttnParams& p, cudaStream_t s) {
  if (p.d <= 16) return launch_rows_dp<16, T>(p, s);
  if (p.d <= 32) return launch_rows_dp<32, T>(p, s);
  if (p.d <= 64) return launch_rows_dp<64, T>(p, s);
  return launch_rows_dp<128, T>(p, s);
}

cudaError_t launch_topk_rows(const AttnParams& p, int dtype, cudaStream_t s) {
  return dtype == TARMAC_BF16 ? launch_rows_dt<__nv_bfloat16>(p, s)
                              : launch_rows_dt<float>(p, s);
}

}  // namespace tarmac
