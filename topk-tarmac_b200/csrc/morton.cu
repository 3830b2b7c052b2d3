// morton.cu — Z-order (Morton) peer selection and the fused select-before-
// scoring kernel on sm_100a.
//
// Restates src/kernels/prescore_selection.py:51-84:
//   _morton_code: per-episode min/max normalise, quantise to `bits` per axis
//     ((pos - lo) / span * (2^bits - 1), truncated, clamped), interleave;
//   select_morton_window: argsort of the codes, rank, and the peers at ranks
//     r+1..r+h, r-1..r-(k-h) (mod N), h = (k+1)/2.
// One block owns one episode. The codes are paired with the agent index into
// a 64-bit key (code << 32 | i), so a plain ascending sort of distinct keys is
// the stable argsort (equal codes keep index order). The quantisation uses
// explicitly rounded fp32 operations (no contraction into fused
// multiply-adds), matching the reference's elementwise tensor arithmetic bit
// for bit.
// * N <= 1024: a block of 4 warps. The curve order comes from a bucket count
//   on the leading code bits (an exclusive scan of the counts, then a rank
//   by (code, index) inside each small bucket). An episode whose codes crowd
//   one bucket falls back to a bitonic network over keys held in registers
//   (up to 8 per lane): strides below 32 on warp shuffles, strides up to
//   16 * keys-per-lane between a lane's own registers, and only the larger
//   strides through shared memory between block barriers. The sorted order
//   and the ranks go to shared memory; the block then writes the window
//   indices or runs the attention rows (one row per thread for d <= 16).
// * Larger N: 512 threads and a bitonic network over shared memory.
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

// ---------------------------------------------------------------------------
// N <= 1024: register bitonic sort over the block's warps
// ---------------------------------------------------------------------------
constexpr int MW_WARPS = 4;  // warps per episode block
constexpr int MW_THREADS = 32 * MW_WARPS;

// Compare-exchange between registers p and p + PS (stride PS*32) of every
// lane; element e of key[p] is ebase + 32 p.
template <int P, int PS>
__device__ __forceinline__ void bitonic_regs(unsigned long long (&key)[P],
                                             int ebase, int size) {
#pragma unroll
  for (int p = 0; p < P; ++p) {
    if ((p & PS) == 0) {
      const int q = p | PS;
      // both elements lie in one size-block: one direction
      const bool up = ((ebase + (p << 5)) & size) == 0;
      const unsigned long long a = key[p], c = key[q];
      const bool sw = (a > c) == up;
      key[p] = sw ? c : a;
      key[q] = sw ? a : c;
    }
  }
}

// Ascending bitonic sort of M = WS*32*P keys held by warps 0..WS-1 of the
// block: warp w, lane l, register p holds element w*32*P + p*32 + l. Strides
// below 32 run on warp shuffles, strides 32 .. 16P between a lane's own
// registers, larger strides (across warps) through `sk` (M keys of shared
// memory) between block barriers. Every thread of the block calls it (the
// others hold no keys and only take part in the barriers).
template <int WS, int P>
__device__ __forceinline__ void block_bitonic_sort(
    unsigned long long (&key)[P], unsigned long long* sk) {
  constexpr int M = WS * 32 * P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool has = warp < WS;
  const int ebase = warp * 32 * P + lane;
#pragma unroll 1
  for (int size = 2; size <= M; size <<= 1) {
#pragma unroll 1
    for (int st = size >> 1; st >= 32 * P; st >>= 1) {
      __syncthreads();
      if (has) {
#pragma unroll
        for (int p = 0; p < P; ++p) sk[ebase + 32 * p] = key[p];
      }
      __syncthreads();
      if (has) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const int e = ebase + 32 * p;
          const unsigned long long o = sk[e ^ st];
          const bool lower = (e & st) == 0, up = (e & size) == 0;
          const unsigned long long mn = key[p] < o ? key[p] : o;
          const unsigned long long mx = key[p] < o ? o : key[p];
          key[p] = (lower == up) ? mn : mx;
        }
      }
    }
    if (has) {
      const int top = (size >> 1) < 16 * P ? (size >> 1) : 16 * P;
#pragma unroll 1
      for (int ps = top >> 5; ps >= 1; ps >>= 1) {
        if constexpr (P >= 2) { if (ps == 1) bitonic_regs<P, 1>(key, ebase, size); }
        if constexpr (P >= 4) { if (ps == 2) bitonic_regs<P, 2>(key, ebase, size); }
        if constexpr (P >= 8) { if (ps == 4) bitonic_regs<P, 4>(key, ebase, size); }
      }
#pragma unroll 1
      for (int st = (size >> 1) < 16 ? (size >> 1) : 16; st > 0; st >>= 1) {
        const bool lower = (lane & st) == 0;
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const unsigned long long o =
              __shfl_xor_sync(0xffffffffu, key[p], st);
          const bool up = ((ebase + (p << 5)) & size) == 0;
          const unsigned long long mn = key[p] < o ? key[p] : o;
          const unsigned long long mx = key[p] < o ? o : key[p];
          key[p] = (lower == up) ? mn : mx;
        }
      }
    }
  }
}

// Bounds, codes and sorted keys of the episode; then ord[r] = agent at curve
// rank r and rank[i] = curve rank of agent i in shared memory, visible to the
// whole block on return. NW: the block's first NW (<= MW_WARPS, >= WS) warps
// hold the agents and exchange the bounds. red: 4 * MW_WARPS floats; sk:
// WS*32*P keys.
template <int WS, int P, int NW = MW_WARPS>
__device__ __forceinline__ void morton_sort_episode_regs(
    const float* pe, int N, int bits, int* ord, int* rank,
    unsigned long long* sk, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool has = warp < WS;
  const int ebase = warp * 32 * P + lane;
  float2 xy[P];
  float lx = INFINITY, ly = INFINITY, hx = -INFINITY, hy = -INFINITY;
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const int e = ebase + 32 * p;
    const bool live = has && e < N;
    xy[p] = live ? reinterpret_cast<const float2*>(pe)[e]
                 : make_float2(0.f, 0.f);
    if (live) {
      lx = fminf(lx, xy[p].x); ly = fminf(ly, xy[p].y);
      hx = fmaxf(hx, xy[p].x); hy = fmaxf(hy, xy[p].y);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lx = fminf(lx, __shfl_xor_sync(0xffffffffu, lx, o));
    ly = fminf(ly, __shfl_xor_sync(0xffffffffu, ly, o));
    hx = fmaxf(hx, __shfl_xor_sync(0xffffffffu, hx, o));
    hy = fmaxf(hy, __shfl_xor_sync(0xffffffffu, hy, o));
  }
  if (lane == 0 && warp < NW) {
    red[warp] = lx; red[NW + warp] = ly;
    red[2 * NW + warp] = hx; red[3 * NW + warp] = hy;
  }
  __syncthreads();
  float bnd[4] = {red[0], red[NW], red[2 * NW], red[3 * NW]};
#pragma unroll
  for (int w = 1; w < NW; ++w) {
    bnd[0] = fminf(bnd[0], red[w]);
    bnd[1] = fminf(bnd[1], red[NW + w]);
    bnd[2] = fmaxf(bnd[2], red[2 * NW + w]);
    bnd[3] = fmaxf(bnd[3], red[3 * NW + w]);
  }
  unsigned long long key[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const int e = ebase + 32 * p;
    key[p] = (has && e < N)
                 ? (((unsigned long long)morton_of(xy[p], bnd, bits) << 32) |
                    (unsigned long long)e)
                 : ~0ull;
  }
  block_bitonic_sort<WS, P>(key, sk);
  if (has) {
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int r = ebase + 32 * p;
      if (r < N) {
        const int a = (int)(key[p] & 0xffffffffu);
        ord[r] = a;
        rank[a] = r;
      }
    }
  }
  __syncthreads();
}

// peer o (0 <= o < k) of the agent at curve rank r, from the sorted order;
// |offset| <= k < N, so one wrap suffices
__device__ __forceinline__ int window_peer_ord(const int* ord, int r, int o,
                                               int k, int N) {
  const int h = (k + 1) / 2;
  const int off = (o < h) ? (o + 1) : -(o - h + 1);
  int nr = r + off;
  nr = nr >= N ? nr - N : (nr < 0 ? nr + N : nr);
  return ord[nr];
}

// ---------------------------------------------------------------------------
// Bucket order (the usual path for N <= 1024)
// ---------------------------------------------------------------------------
// The leading log2(M) bits of a code name its bucket (M = buckets = the
// power of two >= N): buckets follow the curve, so counting the agents per
// bucket, an exclusive scan of the counts and a rank inside the bucket by
// (code, index) give every agent its curve rank — about a hundred
// instructions per agent where the bitonic network takes several hundred.
// An episode whose codes crowd one bucket (more than BUCKET_MAX agents:
// clustered or duplicated positions) takes the bitonic network instead.
constexpr int BUCKET_MAX = 32;

// Exclusive scan of a[0..M) in place by the first 32 * NW threads; every
// thread of the block calls it and gets the largest entry. wsum: 2 *
// MW_WARPS ints of shared memory (NW <= MW_WARPS).
template <int M, int NW = MW_WARPS>
__device__ __forceinline__ int block_scan_max(int* a, int* wsum) {
  constexpr int V = M >= (32 * NW) ? M / (32 * NW) : 1;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int base = t * V;
  const bool has = base < M;
  int loc[V];
  int sum = 0, mx = 0;
#pragma unroll
  for (int u = 0; u < V; ++u) {
    loc[u] = has ? a[base + u] : 0;
    sum += loc[u];
    mx = max(mx, loc[u]);
  }
  int inc = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (warp < NW) {
    if (lane == 31) wsum[warp] = inc;
    if (lane == 0) wsum[NW + warp] = mx;
  }
  __syncthreads();
  int off = 0, gmx = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    off += w < warp ? wsum[w] : 0;
    gmx = max(gmx, wsum[NW + w]);
  }
  int run = off + inc - sum;
  if (has) {
#pragma unroll
    for (int u = 0; u < V; ++u) {
      a[base + u] = run;
      run += loc[u];
    }
  }
  __syncthreads();
  return gmx;
}

// Same result as morton_sort_episode_regs (ord, rank; sk and red as there;
// the block's first NW warps hold the agents). Shared scratch: code[M],
// bst[M], memb[M], wsum[2 * MW_WARPS].
template <int WS, int P, int NW = MW_WARPS>
__device__ __forceinline__ void morton_order_episode(
    const float* pe, int N, int bits, int* ord, int* rank,
    unsigned long long* sk, float* red, uint32_t* code, int* bst, int* memb,
    int* wsum) {
  constexpr int M = WS * 32 * P;
  constexpr int LB = M >= 1024 ? 10 : M >= 512 ? 9 : M >= 256 ? 8
                   : M >= 128 ? 7 : M >= 64 ? 6 : 5;
  constexpr int EPT = (M + (32 * NW) - 1) / (32 * NW);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the first (32 * NW) threads hold the agents; any further threads of a
  // larger block only take part in the barriers
  const bool srt = tid < (32 * NW);
  float2 xy[EPT];
  float lx = INFINITY, ly = INFINITY, hx = -INFINITY, hy = -INFINITY;
#pragma unroll
  for (int t = 0; t < EPT; ++t) {
    const int e = tid + (32 * NW) * t;
    xy[t] = (srt && e < N) ? reinterpret_cast<const float2*>(pe)[e]
                           : make_float2(0.f, 0.f);
    if (srt && e < N) {
      lx = fminf(lx, xy[t].x); ly = fminf(ly, xy[t].y);
      hx = fmaxf(hx, xy[t].x); hy = fmaxf(hy, xy[t].y);
    }
  }
  if (srt)
    for (int e = tid; e < M; e += (32 * NW)) bst[e] = 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lx = fminf(lx, __shfl_xor_sync(0xffffffffu, lx, o));
    ly = fminf(ly, __shfl_xor_sync(0xffffffffu, ly, o));
    hx = fmaxf(hx, __shfl_xor_sync(0xffffffffu, hx, o));
    hy = fmaxf(hy, __shfl_xor_sync(0xffffffffu, hy, o));
  }
  if (lane == 0 && warp < NW) {
    red[warp] = lx; red[NW + warp] = ly;
    red[2 * NW + warp] = hx; red[3 * NW + warp] = hy;
  }
  __syncthreads();
  float bnd[4] = {red[0], red[NW], red[2 * NW], red[3 * NW]};
#pragma unroll
  for (int w = 1; w < NW; ++w) {
    bnd[0] = fminf(bnd[0], red[w]);
    bnd[1] = fminf(bnd[1], red[NW + w]);
    bnd[2] = fmaxf(bnd[2], red[2 * NW + w]);
    bnd[3] = fmaxf(bnd[3], red[3 * NW + w]);
  }
  // the code has 2 * bits significant bits; its leading LB name the bucket
  const int shift = 2 * bits > LB ? 2 * bits - LB : 0;
  uint32_t c[EPT];
  int bk[EPT], slot[EPT];
#pragma unroll
  for (int t = 0; t < EPT; ++t) {
    const int e = tid + (32 * NW) * t;
    if (srt && e < N) {
      c[t] = morton_of(xy[t], bnd, bits);
      code[e] = c[t];
      bk[t] = (int)(c[t] >> shift);
      slot[t] = atomicAdd(&bst[bk[t]], 1);
    }
  }
  __syncthreads();
  const int most = block_scan_max<M, NW>(bst, wsum);
  if (most > BUCKET_MAX) {  // block-uniform
    morton_sort_episode_regs<WS, P, NW>(pe, N, bits, ord, rank, sk, red);
    return;
  }
#pragma unroll
  for (int t = 0; t < EPT; ++t) {
    const int e = tid + (32 * NW) * t;
    if (srt && e < N) memb[bst[bk[t]] + slot[t]] = e;
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < EPT; ++t) {
    const int e = tid + (32 * NW) * t;
    if (srt && e < N) {
      const int lo = bst[bk[t]];
      const int hi = bk[t] + 1 < M ? bst[bk[t] + 1] : N;
      int pos = lo;
      for (int m = lo; m < hi; ++m) {
        const int j = memb[m];
        const uint32_t cj = code[j];
        pos += (cj < c[t] || (cj == c[t] && j < e)) ? 1 : 0;
      }
      ord[pos] = e;
      rank[e] = pos;
    }
  }
  __syncthreads();
}

// Shared scratch of the register-tier sort kernels. The bitonic keys (only
// used when an episode falls back to the bitonic network, after the bucket
// arrays are dead) share their space with the codes and bucket starts.
template <int M>
struct SortScratch {
  union {
    unsigned long long sk[M];
    struct {
      uint32_t code[M];
      int bst[M];
    } b;
  } u;
  int ord[M];
  int rank[M];
  int memb[M];
  int wsum[2 * MW_WARPS];
  float red[4 * MW_WARPS];
};

template <int WS, int P>
__global__ void __launch_bounds__(MW_THREADS) morton_select_regs_kernel(
    const float* __restrict__ pos, int N, int k, int bits,
    int64_t* __restrict__ idx_out) {
  constexpr int M = WS * 32 * P;
  __shared__ SortScratch<M> S;
  unsigned long long* sk = S.u.sk;
  int* ord = S.ord;
  int* rank = S.rank;
  uint32_t* code = S.u.b.code;
  int* bst = S.u.b.bst;
  int* memb = S.memb;
  int* wsum = S.wsum;
  float* red = S.red;
  const int b = blockIdx.x;
  morton_order_episode<WS, P>(pos + (int64_t)b * N * 2, N, bits, ord, rank, sk,
                              red, code, bst, memb, wsum);
  int64_t* ob = idx_out + (int64_t)b * N * k;
  for (int e = threadIdx.x; e < N * k; e += MW_THREADS) {
    const int i = e / k, o = e - i * k;
    ob[e] = window_peer_ord(ord, rank[i], o, k, N);
  }
}

template <int WS, int P, int DP, typename T>
__global__ void __launch_bounds__(MW_THREADS) morton_prescore_regs_kernel(
    AttnParams p, const float* __restrict__ pos, int bits,
    int64_t* __restrict__ idx_out) {
  constexpr int M = WS * 32 * P;
  __shared__ SortScratch<M> S;
  unsigned long long* sk = S.u.sk;
  int* ord = S.ord;
  int* rank = S.rank;
  uint32_t* code = S.u.b.code;
  int* bst = S.u.b.bst;
  int* memb = S.memb;
  int* wsum = S.wsum;
  float* red = S.red;
  const int N = p.N, k = p.topk;
  const int b = blockIdx.x;
  morton_order_episode<WS, P>(pos + (int64_t)b * N * 2, N, bits, ord, rank, sk,
                              red, code, bst, memb, wsum);
  if constexpr (DP <= 16) {
    // one query row per thread
    const T* Qb = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
    const T* Kb = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
    const T* Vb = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
    T* Ob = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;
    for (int i = threadIdx.x; i < N; i += MW_THREADS) {
      PrescoreRowThread<DP, T> pr;
      pr.init(p, Qb + (int64_t)i * p.st.qn, true);
      const int r = rank[i];
      for (int o0 = 0; o0 < k; o0 += 2) {
        const int cnt = min(2, k - o0);
        const T* kr[2];
        const T* vr[2];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const int j = m < cnt ? window_peer_ord(ord, r, o0 + m, k, N) : 0;
          if (m < cnt && idx_out != nullptr)
            idx_out[((int64_t)b * N + i) * k + o0 + m] = j;
          kr[m] = Kb + (int64_t)j * p.st.kn;
          vr[m] = Vb + (int64_t)j * p.st.vn;
        }
        pr.steps2(p, kr, vr, cnt);
      }
      pr.finish(p, Ob + (int64_t)i * p.st.on, false);
    }
    return;
  }
  constexpr int L = DP / 4;
  constexpr int GROUPS = MW_THREADS / L;
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
    for (int o0 = 0; o0 < k; o0 += 4) {
      const int cnt = min(4, k - o0);
      int js[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        js[m] = m < cnt ? window_peer_ord(ord, r, o0 + m, k, N) : 0;
        if (m < cnt && live && idx_out != nullptr && sub == 0)
          idx_out[((int64_t)b * N + i) * k + o0 + m] = js[m];
      }
      pr.template steps<4>(p, b, js, cnt, sub);
    }
    if (live) pr.finish(p, b, i, sub, false);
  }
}

// d <= 16 with 16-byte rows, N <= 512: the episode's K and V rows are copied
// into shared memory (16-byte cp.async, started before the curve order is
// built, so the copy overlaps it) and the window gathers read them there.
// Gathering from global memory, each 16-byte load of a warp touched 32
// different cache lines (one per lane's random row) and the L1 tag stage
// bounded the kernel; from shared memory a gather costs only the bank
// conflicts. A row's 16-byte pieces are stored XOR-swizzled by bits 1-2 of
// the row index, so the pieces a warp gathers from 32 random rows spread
// over all 8 bank groups. Dynamic shared memory: K then V, N rows of DT
// elements each. The block has up to 256 threads, one or two query rows per
// thread; the sort runs on its first four warps (on all of them in the 32-
// and 64-thread blocks of episodes up to 32 and 64 agents).
template <int WS, int P, int DT, typename T, int NT>
__global__ void __launch_bounds__(NT) morton_prescore_smem_kernel(
    AttnParams p, const float* __restrict__ pos, int bits,
    int64_t* __restrict__ idx_out) {
  constexpr int M = WS * 32 * P;
  constexpr int CPR = DT * (int)sizeof(T) / 16;
  __shared__ SortScratch<M> S;
  unsigned long long* sk = S.u.sk;
  int* ord = S.ord;
  int* rank = S.rank;
  uint32_t* code = S.u.b.code;
  int* bst = S.u.b.bst;
  int* memb = S.memb;
  int* wsum = S.wsum;
  float* red = S.red;
  extern __shared__ __align__(16) unsigned char kv_smem[];
  const int N = p.N, k = p.topk;
  const int b = blockIdx.x;
  const uint32_t sK = tc_smem_base(kv_smem);
  const uint32_t sV = sK + (uint32_t)N * CPR * 16u;
  constexpr int NW = NT / 32 < MW_WARPS ? NT / 32 : MW_WARPS;
  static_assert(NW >= WS, "the sorting warps must exist");
  stage_kv_episode<DT, T, NT>(p, b, sK, sV);
  morton_order_episode<WS, P, NW>(pos + (int64_t)b * N * 2, N, bits, ord,
                                  rank, sk, red, code, bst, memb, wsum);
  cp_async_wait<0>();
  __syncthreads();
  const T* Qb = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  T* Ob = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;
  for (int i = threadIdx.x; i < N; i += NT) {
    PrescoreRowThread<DT, T> pr;
    pr.init(p, Qb + (int64_t)i * p.st.qn, true);
    const int r = rank[i];
    for (int o = 0; o < k; ++o) {
      const int j = window_peer_ord(ord, r, o, k, N);
      if (idx_out != nullptr) idx_out[((int64_t)b * N + i) * k + o] = j;
      pr.step_shared(p, sK, sV, j,
                     [](int row, int c) { return kv_piece_off<DT, T>(row, c); });
    }
    pr.finish(p, Ob + (int64_t)i * p.st.on, false);
  }
}

// register-sort tier for N: M = next power of two >= max(N, 32) keys, held
// by WS warps with P keys per lane (0: N above 1024, the shared-memory sort)
static int regs_tier(int N) {
  return N <= 32 ? 1 : N <= 64 ? 2 : N <= 128 ? 4 : N <= 256 ? 8
       : N <= 512 ? 16 : N <= 1024 ? 32 : 0;  // M / 32
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
  switch (regs_tier(N)) {
    case 1: morton_select_regs_kernel<1, 1><<<B, MW_THREADS, 0, s>>>(pos, N, k, bits, idx_out); return cudaGetLastError();
    case 2: morton_select_regs_kernel<2, 1><<<B, MW_THREADS, 0, s>>>(pos, N, k, bits, idx_out); return cudaGetLastError();
    case 4: morton_select_regs_kernel<4, 1><<<B, MW_THREADS, 0, s>>>(pos, N, k, bits, idx_out); return cudaGetLastError();
    case 8: morton_select_regs_kernel<4, 2><<<B, MW_THREADS, 0, s>>>(pos, N, k, bits, idx_out); return cudaGetLastError();
    case 16: morton_select_regs_kernel<4, 4><<<B, MW_THREADS, 0, s>>>(pos, N, k, bits, idx_out); return cudaGetLastError();
    case 32: morton_select_regs_kernel<4, 8><<<B, MW_THREADS, 0, s>>>(pos, N, k, bits, idx_out); return cudaGetLastError();
    default: break;
  }
  const size_t sm = sort_smem(N);
  cudaError_t e = raise_smem_limit(
      (const void*)morton_select_kernel, (size_t)(sm));
  if (e != cudaSuccess) return e;
  morton_select_kernel<<<B, MORTON_THREADS, sm, s>>>(pos, N, next_pow2(N), k,
                                                     bits, idx_out);
  return cudaGetLastError();
}

template <int WS, int P, int DP, typename T>
static cudaError_t launch_mpr(const AttnParams& p, const float* pos, int bits,
                              int64_t* idx_out, cudaStream_t s) {
  morton_prescore_regs_kernel<WS, P, DP, T><<<p.B, MW_THREADS, 0, s>>>(
      p, pos, bits, idx_out);
  return cudaGetLastError();
}

// NT = half the sort's key count, at least 128 threads (one or two query
// rows per thread): with the 64 KB of K and V at N = 512, three blocks fit
// an SM, so one block's sort runs beside another's attention rows. Episodes
// of up to 32 or 64 agents take a block of exactly 32 or 64 threads (one
// row per thread, no idle lanes), so twice or four times as many episodes
// are resident per SM.
template <int WS, int P, int DT, typename T>
static cudaError_t launch_mps(const AttnParams& p, const float* pos, int bits,
                              int64_t* idx_out, cudaStream_t s) {
  constexpr int M = WS * 32 * P;
  constexpr int NT = M <= 64 ? M : (M / 2 < MW_THREADS ? MW_THREADS : M / 2);
  const size_t sm = (size_t)2 * p.N * DT * sizeof(T);
  cudaError_t e = raise_smem_limit(
      (const void*)morton_prescore_smem_kernel<WS, P, DT, T, NT>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  morton_prescore_smem_kernel<WS, P, DT, T, NT><<<p.B, NT, sm, s>>>(
      p, pos, bits, idx_out);
  return cudaGetLastError();
}

template <int DP, typename T>
static cudaError_t launch_mp_t(const AttnParams& p, const float* pos, int bits,
                               int64_t* idx_out, cudaStream_t s) {
  if constexpr (DP <= 16) {
    if (kv_stageable<T>(p)) {
      switch (regs_tier(p.N)) {
        case 1: return launch_mps<1, 1, DP, T>(p, pos, bits, idx_out, s);
        case 2: return launch_mps<2, 1, DP, T>(p, pos, bits, idx_out, s);
        case 4: return launch_mps<4, 1, DP, T>(p, pos, bits, idx_out, s);
        case 8: return launch_mps<4, 2, DP, T>(p, pos, bits, idx_out, s);
        case 16: return launch_mps<4, 4, DP, T>(p, pos, bits, idx_out, s);
        default: break;
      }
    }
  }
  switch (regs_tier(p.N)) {
    case 1: return launch_mpr<1, 1, DP, T>(p, pos, bits, idx_out, s);
    case 2: return launch_mpr<2, 1, DP, T>(p, pos, bits, idx_out, s);
    case 4: return launch_mpr<4, 1, DP, T>(p, pos, bits, idx_out, s);
    case 8: return launch_mpr<4, 2, DP, T>(p, pos, bits, idx_out, s);
    case 16: return launch_mpr<4, 4, DP, T>(p, pos, bits, idx_out, s);
    case 32: return launch_mpr<4, 8, DP, T>(p, pos, bits, idx_out, s);
    default: break;
  }
  const size_t sm = sort_smem(p.N);
  cudaError_t e = raise_smem_limit(
      (const void*)morton_prescore_kernel<DP, T>, (size_t)(sm));
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
