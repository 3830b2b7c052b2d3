// dense.cu — dense masked-diagonal attention on sm_100a (fp32 arithmetic).
//
// Restates the reference's _flash_dense_kernel
// (src/kernels/fused_dense_attention.py:38-99): softmax(q k^T * scale) v with
// the diagonal excluded and no score matrix written. The design differs:
// one thread owns QPT query rows; K and V tiles are staged through shared
// memory and read with broadcast loads; both products run on the packed
// fp32x2 FMA (q.k with even/odd column halves, p*v with the weight duplicated
// into both halves); the online softmax works in base 2 and only moves its
// reference maximum when a score exceeds it by more than 2^RESCALE_LOG2 (a
// stale maximum leaves every weight bounded by 2^8, so the normaliser cannot
// overflow, and the final division makes the result independent of the
// reference point).
#include "common.cuh"

namespace tarmac {

constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 8.0f;

template <int DP>
__host__ __device__ constexpr int dense_tile_keys() {
  return 8192 / (DP * 4);  // 8 KB of K plus 8 KB of V per tile
}

// One staged tile of nk keys (rows of DP floats) against QPT query rows;
// with SPLIT = 2 this lane takes the keys of parity h only.
template <int DP, int QPT, int SPLIT>
__device__ __forceinline__ void dense_tile(
    const float* __restrict__ sk, const float* __restrict__ sv, int nk, int t0,
    const int (&qi)[QPT], const uint64_t (&qp)[QPT][DP / 2],
    uint64_t (&acc)[QPT][DP / 2], float (&mc2)[QPT], float (&mth)[QPT],
    float (&l)[QPT], float c2, int h) {
  constexpr int H = DP / 2;
#pragma unroll 2
  for (int jj = h; jj < nk; jj += SPLIT) {
    const float* kr = sk + jj * DP;
    const float* vr = sv + jj * DP;
    const int j = t0 + jj;
    uint64_t pp[QPT];
#pragma unroll
    for (int r = 0; r < QPT; ++r) {
      // m is kept as mc2 = m * c2, rounded once and shared by the whole row:
      // the exponent fma(s, c2, -mc2) then carries one rounding of a small
      // number, and the rounding of mc2 is a common factor the final
      // division cancels.
      const float s = dot_pairs<DP>(qp[r], kr);
      const float sd = (j == qi[r]) ? -INFINITY : s;
      if (sd > mth[r]) {
        const float mc2n = sd * c2;
        const float alpha = exp2f(mc2[r] - mc2n);
        l[r] *= alpha;
        const uint64_t aa = pack2(alpha, alpha);
#pragma unroll
        for (int c = 0; c < H; ++c) acc[r][c] = ffma2(acc[r][c], aa, 0ull);
        mc2[r] = mc2n;
        mth[r] = sd + RESCALE_LOG2 / c2;
      }
      const float pe = exp2f(fmaf(sd, c2, -mc2[r]));
      l[r] += pe;
      pp[r] = pack2(pe, pe);
    }
#pragma unroll
    for (int c = 0; c < DP; c += 4) {
      const ulonglong2 vv = *reinterpret_cast<const ulonglong2*>(vr + c);
#pragma unroll
      for (int r = 0; r < QPT; ++r) {
        acc[r][c / 2] = ffma2(pp[r], vv.x, acc[r][c / 2]);
        acc[r][c / 2 + 1] = ffma2(pp[r], vv.y, acc[r][c / 2 + 1]);
      }
    }
  }
}

// SPLIT = 2: two lanes per query row, each over the keys of one parity; the
// pair merges its two online-softmax states at the end (the larger reference
// maximum, both normalisers and accumulators rescaled to it, the even lane's
// state first in both lanes, so both hold the same values) and each lane
// stores half the row.
template <int DP, int QPT, typename T, int SPLIT = 1>
__global__ void __launch_bounds__(128) dense_kernel(AttnParams p) {
  constexpr int TK = dense_tile_keys<DP>();
  constexpr int H = DP / 2;  // column pairs
  // double-buffered K and V tiles: tile t+1 is in flight while t is used
  __shared__ __align__(16) float sk[2][TK * DP];
  __shared__ __align__(16) float sv[2][TK * DP];

  constexpr int RPW = 32 * QPT / SPLIT;  // query rows per warp
  const int N = p.N, d = p.d;
  const int groups = cdiv(N, RPW);
  const int wpb = blockDim.x >> 5;
  const int cpe = cdiv(groups, wpb);
  const int b = blockIdx.x / cpe;
  const int chunk = blockIdx.x - b * cpe;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = chunk * wpb + warp;
  const bool vec = p.vec != 0;
  const bool active = g < groups;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  // scores enter the exponent as s * scale * log2(e)
  const float c2 = p.post_scale * LOG2E;
  int qi[QPT];
  uint64_t qp[QPT][H];
  uint64_t acc[QPT][H];
  float mc2[QPT];  // reference maximum times c2 (exponent units)
  float mth[QPT];  // raw score above which the reference point moves
  float l[QPT];
  const int h = lane % SPLIT;
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    qi[r] = g * RPW + r * (32 / SPLIT) + lane / SPLIT;
    float qr[DP];
    if (active && qi[r] < N) {
      load_row<DP, T>(qr, Q + (int64_t)qi[r] * p.st.qn, d, vec);
    } else {
#pragma unroll
      for (int c = 0; c < DP; ++c) qr[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < DP; c += 2) {
      qp[r][c / 2] = pack2(qr[c] * p.qscale, qr[c + 1] * p.qscale);
      acc[r][c / 2] = 0ull;
    }
    mc2[r] = -1e30f;     // finite, so exp2(fma(-inf, c2, -mc2)) is 0, not NaN
    mth[r] = -INFINITY;  // the first finite score moves the reference point
    l[r] = 0.f;
  }

  const int ntiles = cdiv(N, TK);
  stage_rows<DP, T>(sk[0], DP, K, p.st.kn, 0, TK, N, d, vec);
  stage_rows<DP, T>(sv[0], DP, V, p.st.vn, 0, TK, N, d, vec);
  cp_async_commit();
  for (int t = 0; t < ntiles; ++t) {
    const int t0 = t * TK;
    const int buf = t & 1;
    if (t + 1 < ntiles) {
      stage_rows<DP, T>(sk[buf ^ 1], DP, K, p.st.kn, t0 + TK, TK, N, d, vec);
      stage_rows<DP, T>(sv[buf ^ 1], DP, V, p.st.vn, t0 + TK, TK, N, d, vec);
      cp_async_commit();
      cp_async_wait<1>();  // tile t has landed; t+1 may still be in flight
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (active)
      dense_tile<DP, QPT, SPLIT>(sk[buf], sv[buf], min(TK, N - t0), t0, qi,
                                 qp, acc, mc2, mth, l, c2, h);
    __syncthreads();  // everyone is done with `buf` before it is refilled
  }
  if (!active) return;  // warp-uniform: the shuffles below see all 32 lanes
  if constexpr (SPLIT == 2) {
#pragma unroll
    for (int r = 0; r < QPT; ++r) {
      const float mo = __shfl_xor_sync(0xffffffffu, mc2[r], 1);
      const float lo = __shfl_xor_sync(0xffffffffu, l[r], 1);
      uint64_t ao[H];
#pragma unroll
      for (int c = 0; c < H; ++c)
        ao[c] = __shfl_xor_sync(0xffffffffu, acc[r][c], 1);
      // (m0, l0, a0): the even lane's state, (m1, l1, a1): the odd lane's
      const float m0 = h ? mo : mc2[r], m1 = h ? mc2[r] : mo;
      const float l0 = h ? lo : l[r], l1 = h ? l[r] : lo;
      const float m = fmaxf(m0, m1);
      const float f0 = exp2f(m0 - m), f1 = exp2f(m1 - m);
      l[r] = fmaf(l1, f1, l0 * f0);
      const uint64_t ff0 = pack2(f0, f0), ff1 = pack2(f1, f1);
#pragma unroll
      for (int c = 0; c < H; ++c) {
        const uint64_t a0 = h ? ao[c] : acc[r][c];
        const uint64_t a1 = h ? acc[r][c] : ao[c];
        acc[r][c] = ffma2(a1, ff1, ffma2(a0, ff0, 0ull));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < QPT; ++r) {
    if (qi[r] >= N) continue;
    const float inv = 1.0f / l[r];
    float o[DP];
#pragma unroll
    for (int c = 0; c < H; ++c) {
      const float2 f = unpack2(acc[r][c]);
      o[2 * c] = f.x * inv;
      o[2 * c + 1] = f.y * inv;
    }
    if constexpr (SPLIT == 1) {
      store_row<DP, T>(O + (int64_t)qi[r] * p.st.on, o, d, vec);
    } else {
      // each lane of the pair stores half of the row's columns
      float half[H];
#pragma unroll
      for (int c = 0; c < H; ++c) half[c] = h ? o[H + c] : o[c];
      if (d > h * H)
        store_row<H, T>(O + (int64_t)qi[r] * p.st.on + h * H, half, d - h * H,
                        vec);
    }
  }
}

template <int DP>
constexpr int dense_qpt() {
  return DP <= 16 ? 2 : 1;
}

template <int DP, int QPT, typename T, int SPLIT = 1>
static cudaError_t launch_dense_q(const AttnParams& p, cudaStream_t s) {
  const int groups = cdiv(p.N, 32 * QPT / SPLIT);
  const int wpb = groups < 4 ? groups : 4;
  const int cpe = cdiv(groups, wpb);
  const int64_t blocks = (int64_t)p.B * cpe;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  dense_kernel<DP, QPT, T, SPLIT><<<(unsigned)blocks, 32 * wpb, 0, s>>>(p);
  return cudaGetLastError();
}

// Short episodes at d <= 16 spread over up to four warps instead of one
// warp walking every key for two rows per lane: up to 64 agents two lanes
// per query row (each over half the keys), below 128 one lane per row (two
// lanes per row measured slower there: N=100 36.5 -> 38.4 us at B=1024).
template <int DP, typename T>
static cudaError_t launch_dense_dp(const AttnParams& p, cudaStream_t s) {
  constexpr int QPT = dense_qpt<DP>();
  if constexpr (QPT > 1) {
    if (p.N <= 64) return launch_dense_q<DP, 1, T, 2>(p, s);
    if (p.N < 128) return launch_dense_q<DP, 1, T, 1>(p, s);
  }
  return launch_dense_q<DP, QPT, T>(p, s);
}

template <typename T>
static cudaError_t launch_dense_dt(const AttnParams& p, cudaStream_t s) {
  if (p.d <= 8) return launch_dense_dp<8, T>(p, s);
  if (p.d <= 16) return launch_dense_dp<16, T>(p, s);
  if (p.d <= 32) return launch_dense_dp<32, T>(p, s);
  if (p.d <= 64) return launch_dense_dp<64, T>(p, s);
  return launch_dense_dp<128, T>(p, s);
}

bool dense_tc_supported(const AttnParams& p);
cudaError_t launch_dense_tc(const AttnParams& p, cudaStream_t s);
bool dense_tc_f32_supported(const AttnParams& p);
cudaError_t launch_dense_tc_f32(const AttnParams& p, cudaStream_t s);
bool dense_ws_supported(const AttnParams& p);
cudaError_t launch_dense_ws(const AttnParams& p, cudaStream_t s);

// Episodes of 128 or more agents run on the tensor cores: bf16 directly —
// batches of at least four episodes per SM of 320-512 agents with d from 24
// to 64 in the persistent warp-specialized kernel (dense_ws.cu), others one
// 128-query block at a time (dense_tc.cu), the same bits either way — and fp32 with d
// in {8, 16} and 16-byte rows as three exact bf16 planes; other shapes on
// the packed-FMA kernel above.
// 0: persistent warp-specialized, 1: tensor-core per block (bf16), 2:
// tensor-core per block (fp32 planes), 3: packed FMA
int dense_plan(const AttnParams& p, int dtype) {
  if (dtype == TARMAC_BF16 && dense_ws_supported(p)) return 0;
  if (dtype == TARMAC_BF16 && dense_tc_supported(p)) return 1;
  if (dtype == TARMAC_F32 && dense_tc_f32_supported(p)) return 2;
  return 3;
}

cudaError_t launch_dense(const AttnParams& p, int dtype, cudaStream_t s) {
  switch (dense_plan(p, dtype)) {
    case 0: return launch_dense_ws(p, s);
    case 1: return launch_dense_tc(p, s);
    case 2: return launch_dense_tc_f32(p, s);
    default:
      return dtype == TARMAC_BF16 ? launch_dense_dt<__nv_bfloat16>(p, s)
                                  : launch_dense_dt<float>(p, s);
  }
}

}  // namespace tarmac
