// selectors.cu — positional and random peer selectors on sm_100a.
//
// Restates src/kernels/prescore_selection.py:35-172 and the random_k arm of
// src/agents/mappo.py:233-263:
// * select_radius_knn: the k spatially nearest peers of every agent (squared
//   distance (dx^2 + dy^2) in fp32, self excluded), lowest index first on an
//   exact tie. One block per episode; positions in shared memory, read by
//   broadcast; a sorted k-best register buffer per agent.
// * select_grid_knn: the k nearest among the 3 x 3 grid cells around each
//   agent, with the reference's grid side G and per-cell capacity M
//   (grid_knn_shape). Per episode: cell ids with the reference's
//   normalise-and-truncate arithmetic, a stable counting sort of the agents
//   by cell (counts, a warp prefix sum, and a warp-synchronous placement in
//   index order: equal cells keep agent order, the deterministic member of
//   the reference's unstable argsort), then each agent ranks the three
//   contiguous runs of sorted agents (x-1..x+1, y-1..y+1), each cut at 3M
//   entries. When the 3 x 3 neighbourhood can hold N or more candidates
//   (3 * 3M >= N) the exact selector runs instead, as in the reference. An
//   agent whose runs hold fewer than k candidates takes the exact k nearest.
// * random_k: k distinct peers per agent, uniform over the k-subsets of the
//   other N - 1 agents (Floyd's sampling on a Philox stream keyed by the row),
//   the distribution of the reference's rank-the-uniform-noise rule.
// Output: int64 [B, N, k]; the kNN selectors list peers by increasing
// (distance, index).
#include <curand_kernel.h>

#include "episode.cuh"
#include "topk_chunk.cuh"

namespace tarmac {

constexpr int SEL_THREADS = 256;

__device__ __forceinline__ float dist2(float2 a, float2 b) {
  const float dx = __fsub_rn(b.x, a.x), dy = __fsub_rn(b.y, a.y);
  return __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
}

// exact k nearest of agent i among all N (buffers hold negated distances)
template <int KM>
__device__ __forceinline__ void knn_row(const float2* sp, int N, int i,
                                        float (&bs)[KM], int (&bi)[KM]) {
#pragma unroll
  for (int m = 0; m < KM; ++m) {
    bs[m] = -INFINITY;
    bi[m] = -1;
  }
  const float2 pi = sp[i];
  for (int j = 0; j < N; ++j) {
    const float nd = -dist2(pi, sp[j]);
    // increasing j: a later index enters only strictly closer
    if (j != i && nd > bs[KM - 1]) buf_insert<KM, false>(bs, bi, nd, j);
  }
}

// the same for agents i and i2 in one pass over the positions (each position
// read from shared memory once for both rows); i2 >= N computes nothing
// that is kept
template <int KM>
__device__ __forceinline__ void knn_row2(const float2* sp, int N, int i, int i2,
                                         float (&bs)[KM], int (&bi)[KM],
                                         float (&bs2)[KM], int (&bi2)[KM]) {
#pragma unroll
  for (int m = 0; m < KM; ++m) {
    bs[m] = -INFINITY;
    bi[m] = -1;
    bs2[m] = -INFINITY;
    bi2[m] = -1;
  }
  const float2 pi = sp[i], pi2 = sp[i2 < N ? i2 : i];
#pragma unroll 4
  for (int j = 0; j < N; ++j) {
    const float2 pj = sp[j];
    const float nd = -dist2(pi, pj), nd2 = -dist2(pi2, pj);
    // one test for both rows on the common path (neither enters)
    if (nd > bs[KM - 1] || nd2 > bs2[KM - 1]) {
      if (j != i && nd > bs[KM - 1]) buf_insert<KM, false>(bs, bi, nd, j);
      if (j != i2 && nd2 > bs2[KM - 1]) buf_insert<KM, false>(bs2, bi2, nd2, j);
    }
  }
}

template <int KM>
__global__ void __launch_bounds__(SEL_THREADS) knn_select_kernel(
    const float* __restrict__ pos, int N, int k, int64_t* __restrict__ out) {
  extern __shared__ float2 sel_sp[];
  const int b = blockIdx.x;
  const float2* pe = reinterpret_cast<const float2*>(pos) + (int64_t)b * N;
  for (int i = threadIdx.x; i < N; i += blockDim.x) sel_sp[i] = pe[i];
  __syncthreads();
  // two agents a thread per pass (i and i + blockDim.x)
  for (int i = threadIdx.x; i < N; i += 2 * blockDim.x) {
    const int i2 = i + blockDim.x;
    float bs[KM], bs2[KM];
    int bi[KM], bi2[KM];
    knn_row2<KM>(sel_sp, N, i, i2, bs, bi, bs2, bi2);
    int64_t* o = out + ((int64_t)b * N + i) * k;
#pragma unroll
    for (int m = 0; m < KM; ++m)
      if (m < k) o[m] = bi[m];
    if (i2 < N) {
      int64_t* o2 = out + ((int64_t)b * N + i2) * k;
#pragma unroll
      for (int m = 0; m < KM; ++m)
        if (m < k) o2[m] = bi2[m];
    }
  }
}

// Grid kNN. Dynamic shared memory: N float2 positions, N int cells, N int
// order, C + 1 int run starts, C int fill counters (C = G * G).
template <int KM>
__global__ void __launch_bounds__(SEL_THREADS) grid_knn_kernel(
    const float* __restrict__ pos, int N, int k, int G, int L,
    int64_t* __restrict__ out) {
  extern __shared__ float2 sel_sp[];
  __shared__ float red[4 * (SEL_THREADS / 32)];
  __shared__ float bnd[4];
  const int C = G * G;
  int* cell = reinterpret_cast<int*>(sel_sp + N);
  int* order = cell + N;
  int* start = order + N;
  int* fill = start + C + 1;
  const int b = blockIdx.x;
  const float* pe = pos + (int64_t)b * N * 2;
  for (int i = threadIdx.x; i < N; i += blockDim.x)
    sel_sp[i] = reinterpret_cast<const float2*>(pe)[i];
  for (int c = threadIdx.x; c < C + 1; c += blockDim.x) start[c] = 0;
  episode_bounds(pe, N, red, bnd);  // synchronises
  // cxy = ((pos - lo) / span * G).long().clamp(0, G - 1); cell = x * G + y
  const float sx = fmaxf(__fsub_rn(bnd[2], bnd[0]), 1e-6f);
  const float sy = fmaxf(__fsub_rn(bnd[3], bnd[1]), 1e-6f);
  const float gq = (float)G;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const uint32_t cx = quantise(sel_sp[i].x, bnd[0], sx, gq, (uint32_t)(G - 1));
    const uint32_t cy = quantise(sel_sp[i].y, bnd[1], sy, gq, (uint32_t)(G - 1));
    const int c = (int)(cx * G + cy);
    cell[i] = c;
    atomicAdd(&start[c + 1], 1);
  }
  __syncthreads();
  // inclusive prefix sum of start[1..C] by warp 0: start[c] = first sorted
  // position of cell c, start[C] = N
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = cdiv(C + 1, 32);
    const int c0 = lane * per, c1 = min(C + 1, c0 + per);
    int run = 0;
    for (int c = c0; c < c1; ++c) run += start[c];
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int acc = incl - run;
    for (int c = c0; c < c1; ++c) {
      acc += start[c];
      start[c] = acc;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) fill[c] = start[c];
  __syncthreads();
  // stable placement in index order, 32 agents at a time (warp 0)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const unsigned lt = (1u << lane) - 1u;
    for (int i0 = 0; i0 < N; i0 += 32) {
      const int i = i0 + lane;
      const int c = i < N ? cell[i] : -1 - lane;  // absent lanes match nobody
      const unsigned peers = __match_any_sync(0xffffffffu, c);
      if (i < N) {
        const int base = fill[c];
        order[base + __popc(peers & lt)] = i;
      }
      __syncwarp();
      if (i < N && (peers & lt) == 0) fill[c] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const int ci = cell[i];
    const int cx = ci / G, cy = ci - (ci / G) * G;
    const float2 pi = sel_sp[i];
    float bs[KM];
    int bi[KM];
#pragma unroll
    for (int m = 0; m < KM; ++m) {
      bs[m] = -INFINITY;
      bi[m] = -1;
    }
    int found = 0;
#pragma unroll
    for (int dx = -1; dx <= 1; ++dx) {
      const int x = cx + dx;
      if (x < 0 || x >= G) continue;
      const int lo = start[x * G + max(cy - 1, 0)];
      const int hi = min(start[x * G + min(cy + 1, G - 1) + 1], lo + L);
      for (int s = lo; s < hi; ++s) {
        const int j = order[s];
        if (j == i) continue;
        ++found;
        ins_idx<KM, false>(bs, bi, -dist2(pi, sel_sp[j]), j);
      }
    }
    if (found < k) knn_row<KM>(sel_sp, N, i, bs, bi);
    int64_t* o = out + ((int64_t)b * N + i) * k;
#pragma unroll
    for (int m = 0; m < KM; ++m)
      if (m < k) o[m] = bi[m];
  }
}

__global__ void __launch_bounds__(SEL_THREADS) random_select_kernel(
    int64_t rows, int N, int k, unsigned long long seed,
    unsigned long long offset, int64_t* __restrict__ out) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int i = (int)(row % N);
  curandStatePhilox4_32_10_t st;
  curand_init(seed, (unsigned long long)row, offset, &st);
  int64_t* o = out + row * k;
  const int M = N - 1;  // candidates: the other agents, r -> r < i ? r : r+1
  // Floyd: for j = M-k .. M-1 draw t uniform in [0, j]; take t, or j if t
  // was already taken. Every k-subset of [0, M) is equally likely.
  for (int c = 0; c < k; ++c) {
    const int j = M - k + c;
    const uint32_t t = (uint32_t)(((uint64_t)curand(&st) * (uint64_t)(j + 1)) >> 32);
    bool dup = false;
    for (int u = 0; u < c; ++u) {
      const int64_t prev = o[u];
      const int64_t r = prev > i ? prev - 1 : prev;
      dup |= r == (int64_t)t;
    }
    const int r = dup ? j : (int)t;
    o[c] = r < i ? r : r + 1;
  }
}

// ---------------------------------------------------------------------------

template <int KM>
static cudaError_t launch_knn_t(const float* pos, int B, int N, int k,
                                int64_t* out, cudaStream_t s) {
  const size_t sm = (size_t)N * sizeof(float2);
  cudaError_t e = raise_smem_limit(
      (const void*)knn_select_kernel<KM>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  knn_select_kernel<KM><<<B, SEL_THREADS, sm, s>>>(pos, N, k, out);
  return cudaGetLastError();
}

template <int KM>
static cudaError_t launch_grid_t(const float* pos, int B, int N, int k, int G,
                                 int L, int64_t* out, cudaStream_t s) {
  const int C = G * G;
  const size_t sm = (size_t)N * sizeof(float2) + (size_t)(2 * N + 2 * C + 1) * 4;
  cudaError_t e = raise_smem_limit(
      (const void*)grid_knn_kernel<KM>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  grid_knn_kernel<KM><<<B, SEL_THREADS, sm, s>>>(pos, N, k, G, L, out);
  return cudaGetLastError();
}

#define SEL_DISPATCH(FN, ...)                           \
  switch (k <= 1 ? 1 : k <= 2 ? 2 : k <= 4 ? 4 : k <= 8 ? 8 : k <= 16 ? 16 : 32) { \
    case 1: return FN<1>(__VA_ARGS__);                  \
    case 2: return FN<2>(__VA_ARGS__);                  \
    case 4: return FN<4>(__VA_ARGS__);                  \
    case 8: return FN<8>(__VA_ARGS__);                  \
    case 16: return FN<16>(__VA_ARGS__);                \
    default: return FN<32>(__VA_ARGS__);                \
  }

cudaError_t launch_knn_select(const float* pos, int B, int N, int k,
                              int64_t* out, cudaStream_t s) {
  SEL_DISPATCH(launch_knn_t, pos, B, N, k, out, s)
}

// grid side G and per-cell capacity M as the reference sizes them
// (prescore_selection.py grid_knn_shape)
void grid_knn_shape(int N, int k, int* G, int* M) {
  const int occ = k > 2 ? k : 2;
  int g = (int)sqrt((double)N / occ);
  if (g < 1) g = 1;
  const double mean = (double)N / ((double)g * g);
  *G = g;
  *M = (int)(mean + 3.0 * sqrt(mean) + 2.0);
}

cudaError_t launch_grid_knn_select(const float* pos, int B, int N, int k,
                                   int64_t* out, cudaStream_t s) {
  int G, M;
  grid_knn_shape(N, k, &G, &M);
  const int L = 3 * M;
  if (3 * L >= N) return launch_knn_select(pos, B, N, k, out, s);
  SEL_DISPATCH(launch_grid_t, pos, B, N, k, G, L, out, s)
}

cudaError_t launch_random_select(int B, int N, int k, unsigned long long seed,
                                 unsigned long long offset, int64_t* out,
                                 cudaStream_t s) {
  const int64_t rows = (int64_t)B * N;
  const int64_t blocks = (rows + SEL_THREADS - 1) / SEL_THREADS;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  random_select_kernel<<<(unsigned)blocks, SEL_THREADS, 0, s>>>(rows, N, k, seed,
                                                                offset, out);
  return cudaGetLastError();
}

}  // namespace tarmac
