// morton.cu — Z-order (Morton) peer selection and the fused select-before-
// scoring kernel on sm_100a.
//
// Restates src/kernels/prescore_selection.py:313-342:
//   _morton_code: per-episode min/max normalise, quantise to `bits` per axis
//     ((pos - lo) / span * (2^bits - 1), truncated, clamped), interleave;
//   select_morton_window: argsort of the codes, rank, and the peers at ranks
//     r+1..r+h, r-1..r-(k-h) (mod N), h = (k+1)/2.
// One block owns one episode. The codes are paired with the agent index into
// a 64-bit key (code << 32 | i), so a plain ascending sort of distinct keys is
// the stable argsort (equal codes keep index order). The sort is a bitonic
// network in shared memory. The quantisation uses explicitly rounded fp32
// operations (no contraction into fused multiply-adds), matching the
// reference's elementwise tensor arithmetic bit for bit.
#include "episode.cuh"
#include "prescore.cuh"

namespace tarmac {

constexpr int MORTON_THREADS = 512;

__device__ __forceinline__ uint32_t spread_bits(uint32_t v) {
  // insert a zero between consecutive bits of a 16-bit value
  v = (v | (v << 8)) & 0x00FF00FFu;
  v = (v | (v << 4)) & 0x0F0F0F0Fu;
  v = (v | (v << 2)) & 0x33333333u;
  v = (v | (v << 1)) & 0x55555555u;
  return v;
}

__device__ __forceinline__ uint32_t morton_of(float2 pxy, const float* bnd,
                                              int bits) {
  const uint32_t qmax = (1u << bits) - 1u;
  const float scale_q = (float)qmax;
  // span = (hi - lo).clamp_min(1e-6)
  const float sx = fmaxf(__fsub_rn(bnd[2], bnd[0]), 1e-6f);
  const float sy = fmaxf(__fsub_rn(bnd[3], bnd[1]), 1e-6f);
  const uint32_t gx = quantise(pxy.x, bnd[0], sx, scale_q, qmax);
  const uint32_t gy = quantise(pxy.y, bnd[1], sy, scale_q, qmax);
  return spread_bits(gx) | (spread_bits(gy) << 1);
}

__global__ void __launch_bounds__(MORTON_THREADS) morton_code_kernel(
    const float* __restrict__ pos, int N, int bits, int64_t* __restrict__ out) {
  __shared__ float red[4 * (MORTON_THREADS / 32)];
  __shared__ float bnd[4];
  const int b = blockIdx.x;
  const float* pe = pos + (int64_t)b * N * 2;
  episode_bounds(pe, N, red, bnd);
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const float2 pxy = reinterpret_cast<const float2*>(pe)[i];
    out[(int64_t)b * N + i] = (int64_t)morton_of(pxy, bnd, bits);
  }
}

// Shared prologue of the selector kernels: sorted keys of the episode in
// keys[0..NP), rank[i] = position of agent i in curve order.
// Dynamic shared memory: NP uint64 keys followed by N int32 ranks.
__device__ __forceinline__ void morton_sort_episode(const float* pe, int N,
                                                    int NP, int bits,
                                                    unsigned long long* keys,
                                                    int* rank, float* red,
                                                    float* bnd) {
  episode_bounds(pe, N, red, bnd);
  for (int i = threadIdx.x; i < NP; i += blockDim.x) {
    unsigned long long key = ~0ull;
    if (i < N) {
      const float2 pxy = reinterpret_cast<const float2*>(pe)[i];
      key = ((unsigned long long)morton_of(pxy, bnd, bits) << 32) |
            (unsigned long long)i;
    }
    keys[i] = key;
  }
  // bitonic sort, ascending
  for (int size = 2; size <= NP; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < (NP >> 1); t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long a = keys[lo], c = keys[hi];
        if ((a > c) == up) {
          keys[lo] = c;
          keys[hi] = a;
        }
      }
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < N; r += blockDim.x)
    rank[(int)(keys[r] & 0xffffffffu)] = r;
  __syncthreads();
}

// peer o (0 <= o < k) of the agent at curve rank r
__device__ __forceinline__ int window_peer(const unsigned long long* keys,
                                           int r, int o, int k, int N) {
  const int h = (k + 1) / 2;
  const int off = (o < h) ? (o + 1) : -(o - h + 1);
  int nr = (r + off) % N;
  if (nr < 0) nr += N;
  return (int)(keys[nr] & 0xffffffffu);
}

__global__ void __launch_bounds__(MORTON_THREADS) morton_select_kernel(
    const float* __restrict__ pos, int N, int NP, int k, int bits,
    int64_t* __restrict__ idx_out) {
  extern __shared__ __align__(16) unsigned char dsm[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(dsm);
  int* rank = reinterpret_cast<int*>(keys + NP);
  __shared__ float red[4 * (MORTON_THREADS / 32)];
  __shared__ float bnd[4];
  const int b = blockIdx.x;
  morton_sort_episode(pos + (int64_t)b * N * 2, N, NP, bits, keys, rank, red,
                      bnd);
  int64_t* ob = idx_out + (int64_t)b * N * k;
  for (int e = threadIdx.x; e < N * k; e += blockDim.x) {
    const int i = e / k, o = e - i * k;
    ob[e] = window_peer(keys, rank[i], o, k, N);
  }
}

template <int DP, typename T>
__global__ void __launch_bounds__(MORTON_THREADS) morton_prescore_kernel(
    AttnParams p, const float* __restrict__ pos, int NP, int bits,
    int64_t* __restrict__ idx_out) {
  extern __shared__ __align__(16) unsigned char dsm[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(dsm);
  int* rank = reinterpret_cast<int*>(keys + NP);
  __shared__ float red[4 * (MORTON_THREADS / 32)];
  __shared__ float bnd[4];
  const int N = p.N, k = p.topk;
  const int b = blockIdx.x;
  morton_sort_episode(pos + (int64_t)b * N * 2, N, NP, bits, keys, rank, red,
                      bnd);
  constexpr int L = DP / 4;
  constexpr int GROUPS = MORTON_THREADS / L;
  const int sub = threadIdx.x % L;
  const int grp = threadIdx.x / L;
  // every lane of a warp runs the same number of iterations (shuffles inside)
  const int iters = cdiv(N, GROUPS);
  for (int it = 0; it < iters; ++it) {
    const int i = it * GROUPS + grp;
    const bool live = i < N;
    PrescoreRow<DP, T> pr;
    pr.init(p, b, live ? i : 0, sub, live);
    const int r = live ? rank[i] : 0;
    for (int o = 0; o < k; ++o) {
      const int j = window_peer(keys, r, o, k, N);
      pr.step(p, b, j, sub);
      if (live && idx_out != nullptr && sub == 0)
        idx_out[((int64_t)b * N + i) * k + o] = j;
    }
    if (live) pr.finish(p, b, i, sub, false);
  }
}

static int next_pow2(int x) {
  int v = 1;
  while (v < x) v <<= 1;
  return v;
}

static size_t sort_smem(int N) {
  return (size_t)next_pow2(N) * 8 + (size_t)N * 4;
}

cudaError_t launch_morton_code(const float* pos, int B, int N, int bits,
                               int64_t* out, cudaStream_t s) {
  morton_code_kernel<<<B, MORTON_THREADS, 0, s>>>(pos, N, bits, out);
  return cudaGetLastError();
}

cudaError_t launch_morton_select(const float* pos, int B, int N, int k,
                                 int bits, int64_t* idx_out, cudaStream_t s) {
  const size_t sm = sort_smem(N);
  cudaError_t e = cudaFuncSetAttribute(
      morton_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
      (int)sm);
  if (e != cudaSuccess) return e;
  morton_select_kernel<<<B, MORTON_THREADS, sm, s>>>(pos, N, next_pow2(N), k,
                                                     bits, idx_out);
  return cudaGetLastError();
}

template <int DP, typename T>
static cudaError_t launch_mp_t(const AttnParams& p, const float* pos, int bits,
                               int64_t* idx_out, cudaStream_t s) {
  const size_t sm = sort_smem(p.N);
  cudaError_t e = cudaFuncSetAttribute(
      morton_prescore_kernel<DP, T>,
      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  morton_prescore_kernel<DP, T><<<p.B, MORTON_THREADS, sm, s>>>(
      p, pos, next_pow2(p.N), bits, idx_out);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_mp_dt(const AttnParams& p, const float* pos, int bits,
                                int64_t* idx_out, cudaStream_t s) {
  if (p.d <= 8) return launch_mp_t<8, T>(p, pos, bits, idx_out, s);
  if (p.d <= 16) return launch_mp_t<16, T>(p, pos, bits, idx_out, s);
  if (p.d <= 32) return launch_mp_t<32, T>(p, pos, bits, idx_out, s);
  if (p.d <= 64) return launch_mp_t<64, T>(p, pos, bits, idx_out, s);
  return launch_mp_t<128, T>(p, pos, bits, idx_out, s);
}

cudaError_t launch_morton_prescore(const AttnParams& p, int dtype,
                                   const float* pos, int bits,
                                   int64_t* idx_out, cudaStream_t s) {
  return dtype == TARMAC_BF16
             ? launch_mp_dt<__nv_bfloat16>(p, pos, bits, idx_out, s)
             : launch_mp_dt<float>(p, pos, bits, idx_out, s);
}

}  // namespace tarmac
