// comm.cu — the whole communication module forward in one kernel:
// qkv projection -> attention core -> GELU -> output projection.
//
// Restates AttentionComm.forward (src/agents/mappo.py:332-353, 361-373,
// 419-420) for the dense and the top-k modes: q, k, v = split(x W_qkv^T +
// b_qkv); msg = attention core over the episode (diagonal excluded; dense
// softmax, or the k best scores with the lowest index kept on a tie, the
// topk / topk_gather function); out = gelu(msg) W_proj^T + b_proj with the
// exact (erf) GELU of torch.nn.functional.gelu.
//
// One block owns one episode. The projections and the episode's Q, K and V
// rows (msg_dim wide) sit in shared memory, so Q, K and V never reach HBM:
// the kernel reads x once and writes the module output once. Phase 1: the
// block projects the episode's x rows (staged through shared memory 32 rows
// at a time, coalesced) into q, k and v, one (row, output) pair per thread
// at a time. Phase 2:
// every thread owns query agents: scores against all keys (fp32 FMA), a
// sorted k-best buffer (top-k) or a base-2 online softmax (dense), the V
// aggregate, GELU and the output projection. Sized for the reference's
// MAPPO shapes (N up to 1024, msg_dim up to 64, in_dim up to 256).
// Batches of at least one episode per SM with short episodes take the
// multi-episode tile form (comm_tile_kernel below), which returns the same
// bits.
#include <algorithm>

#include "comm.cuh"
#include "topk_chunk.cuh"

namespace tarmac {

constexpr int COMM_THREADS = 128;
constexpr int COMM_XTILE = 32;  // x rows staged per step
// resident blocks per SM of the multi-episode tile form for large batches
constexpr int COMM_TILE_BPS = 8;



__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// 4-byte global -> shared copy without a register round trip (cp.async,
// through L1); completes at cp_async_wait_all().
__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(gsrc)
               : "memory");
}

// Copy rows [0, R) of a row-major [R, D] global matrix into shared rows of DS
// floats: rows over warps, columns over lanes (no index division). With VEC
// the rows move as 16-byte pieces (D % 4 == 0, 16-byte aligned source and
// rows), else as 4-byte words. Every copy is in flight at once; the caller
// waits with cp_async_wait_all().
template <bool VEC>
__device__ __forceinline__ void comm_stage(float* dst, int DS, const float* src,
                                           int R, int D) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  if constexpr (VEC) {
    const int D4 = D >> 2;
    for (int r = warp; r < R; r += nw)
      for (int c = lane; c < D4; c += 32)
        cp_async16(dst + r * DS + 4 * c, src + (int64_t)r * D + 4 * c);
  } else {
    for (int r = warp; r < R; r += nw)
      for (int c = lane; c < D; c += 32)
        cp_async4(dst + r * DS + c, src + (int64_t)r * D + c);
  }
}

// Shared row stride of the x tile and of W_qkv: with VEC, D rounded so that
// the row stride is an odd number of 16-byte pieces (eight consecutive rows
// read as 16-byte pieces hit distinct bank groups); else D + 1 (32
// consecutive rows read word by word hit distinct banks).
__host__ __device__ __forceinline__ int comm_row_stride(int D, bool vec) {
  return vec ? 4 * ((D >> 2) | 1) : D + 1;
}

// Dynamic shared memory layout (floats): Q/K/V [N][MP] each (columns
// m..MP-1 zero), x tile [32][DS], GELU buffer [COMM_THREADS], W_qkv
// [3m][DS] when p.w_smem, then W_proj [m][m], b_proj [m], b_qkv [3m].
// Without p.w_smem W_qkv is read from global memory through L1.
//
// Phase 2 runs in one of two forms. An episode with N * MP <= COMM_THREADS
// (the MAPPO shapes: a handful of agents) gives every (agent, message
// column) pair its own thread: each thread of an agent's group forms the
// agent's scores and selection (the same arithmetic in every lane of the
// group), aggregates its own V column and applies GELU; after a barrier
// thread (agent, r) forms output column r. Larger episodes give each thread
// whole query agents. Both forms evaluate every output with the same
// operations in the same order.
// Phase 1 for the staged x rows [r0, r0 + nr) (x tile sx, row stride DS):
// threads take (row, output) pairs, consecutive threads consecutive outputs
// of one row, so the x row is a broadcast read and the weight rows hit
// distinct banks. Each dot product runs over the columns in order, then
// adds the bias.
template <int MP, bool VEC>
__device__ __forceinline__ void comm_project(const CommParams& p, const float* sx,
                                             int DS, const float* sw,
                                             const float* sbq, int r0, int nr,
                                             float* sq, float* sk, float* sv) {
  const int D = p.in_dim, m = p.m, M3 = 3 * m;
  for (int pr = threadIdx.x; pr < nr * M3; pr += blockDim.x) {
    const int rr = pr / M3, o = pr - rr * M3;
    const float* xr = sx + rr * DS;
    float acc = 0.f;
    if constexpr (VEC) {
      if (p.w_smem) {
        const float* wr = sw + o * DS;
        for (int c = 0; c < D; c += 4) {
          const float4 a = *reinterpret_cast<const float4*>(xr + c);
          const float4 w = *reinterpret_cast<const float4*>(wr + c);
          acc = fmaf(a.x, w.x, acc);
          acc = fmaf(a.y, w.y, acc);
          acc = fmaf(a.z, w.z, acc);
          acc = fmaf(a.w, w.w, acc);
        }
      } else {
        const float4* wr = reinterpret_cast<const float4*>(p.wqkv + (int64_t)o * D);
        for (int c = 0; c < D; c += 4) {
          const float4 a = *reinterpret_cast<const float4*>(xr + c);
          const float4 w = __ldg(wr + (c >> 2));
          acc = fmaf(a.x, w.x, acc);
          acc = fmaf(a.y, w.y, acc);
          acc = fmaf(a.z, w.z, acc);
          acc = fmaf(a.w, w.w, acc);
        }
      }
    } else {
      if (p.w_smem) {
        const float* wr = sw + o * DS;
        for (int c = 0; c < D; ++c) acc = fmaf(xr[c], wr[c], acc);
      } else {
        const float* wr = p.wqkv + (int64_t)o * D;
        for (int c = 0; c < D; ++c) acc = fmaf(xr[c], __ldg(wr + c), acc);
      }
    }
    acc += sbq[o];
    const int part = o / m, col = o - part * m;
    float* dst = part == 0 ? sq : (part == 1 ? sk : sv);
    dst[(r0 + rr) * MP + col] = acc;
  }
}

// Phase 2 for episode b: attention over the episode's q, k, v rows, GELU and
// the output projection (both forms described above).
template <int MP, int KM>
__device__ __forceinline__ void comm_attend(const CommParams& p, int b,
                                            const float* sq, const float* sk,
                                            const float* sv, float* sg,
                                            const float* spw, const float* spb) {
  const int N = p.N, m = p.m;
  if (N * MP <= COMM_THREADS) {
    // one thread per (agent i, message column c)
    const int i = threadIdx.x / MP, c = threadIdx.x % MP;
    float g = 0.f;
    if (i < N) {
      float qi[MP];
#pragma unroll
      for (int t = 0; t < MP; t += 4) {
        const float4 f = *reinterpret_cast<const float4*>(sq + i * MP + t);
        qi[t] = f.x; qi[t + 1] = f.y; qi[t + 2] = f.z; qi[t + 3] = f.w;
      }
      float msg = 0.f;
      if constexpr (KM > 0) {
        float bs[KM];
        int bi[KM];
#pragma unroll
        for (int s = 0; s < KM; ++s) {
          bs[s] = -INFINITY;
          bi[s] = -1;
        }
        for (int j = 0; j < N; ++j) {
          float s = 0.f;
#pragma unroll
          for (int t = 0; t < MP; t += 4) {
            const float4 f = *reinterpret_cast<const float4*>(sk + j * MP + t);
            s = fmaf(qi[t], f.x, s);
            s = fmaf(qi[t + 1], f.y, s);
            s = fmaf(qi[t + 2], f.z, s);
            s = fmaf(qi[t + 3], f.w, s);
          }
          if (j != i && s > bs[KM - 1]) buf_insert<KM, false>(bs, bi, s, j);
        }
        const int kk = p.topk;
        const float mx = bs[0] * p.scale;
        float den = 0.f, w[KM];
#pragma unroll
        for (int s = 0; s < KM; ++s) {
          w[s] = (s < kk && bi[s] >= 0) ? expf(bs[s] * p.scale - mx) : 0.f;
          den += w[s];
        }
#pragma unroll
        for (int s = 0; s < KM; ++s)
          if (w[s] > 0.f) msg = fmaf(w[s] / den, sv[bi[s] * MP + c], msg);
      } else {
        float mref = -INFINITY, l = 0.f;
        for (int j = 0; j < N; ++j) {
          if (j == i) continue;
          float s = 0.f;
#pragma unroll
          for (int t = 0; t < MP; t += 4) {
            const float4 f = *reinterpret_cast<const float4*>(sk + j * MP + t);
            s = fmaf(qi[t], f.x, s);
            s = fmaf(qi[t + 1], f.y, s);
            s = fmaf(qi[t + 2], f.z, s);
            s = fmaf(qi[t + 3], f.w, s);
          }
          s *= p.scale;
          if (s > mref) {
            const float a = expf(mref - s);
            l *= a;
            msg *= a;
            mref = s;
          }
          const float e = expf(s - mref);
          l += e;
          msg = fmaf(e, sv[j * MP + c], msg);
        }
        msg *= 1.0f / l;
      }
      g = gelu_erf(msg);
    }
    sg[threadIdx.x] = g;
    __syncthreads();
    if (i < N && c < m) {
      const float* gr = sg + i * MP;
      const float* wr = spw + c * m;
      float acc = 0.f;
      for (int t = 0; t < m; ++t) acc = fmaf(gr[t], wr[t], acc);
      p.out[((int64_t)b * N + i) * m + c] = acc + spb[c];
    }
    return;
  }
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    float qi[MP];
#pragma unroll
    for (int c = 0; c < MP; ++c) qi[c] = c < m ? sq[i * MP + c] : 0.f;
    float msg[MP];
#pragma unroll
    for (int c = 0; c < MP; ++c) msg[c] = 0.f;
    if constexpr (KM > 0) {
      float bs[KM];
      int bi[KM];
#pragma unroll
      for (int s = 0; s < KM; ++s) {
        bs[s] = -INFINITY;
        bi[s] = -1;
      }
      for (int j = 0; j < N; ++j) {
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < MP; ++c) s = fmaf(qi[c], sk[j * MP + c], s);
        if (j != i && s > bs[KM - 1]) buf_insert<KM, false>(bs, bi, s, j);
      }
      const int kk = p.topk;
      const float mx = bs[0] * p.scale;
      float den = 0.f, w[KM];
#pragma unroll
      for (int s = 0; s < KM; ++s) {
        w[s] = (s < kk && bi[s] >= 0) ? expf(bs[s] * p.scale - mx) : 0.f;
        den += w[s];
      }
#pragma unroll
      for (int s = 0; s < KM; ++s) {
        if (w[s] > 0.f) {
          const float ws = w[s] / den;
          const float* vr = sv + bi[s] * MP;
#pragma unroll
          for (int c = 0; c < MP; ++c) msg[c] = fmaf(ws, vr[c], msg[c]);
        }
      }
    } else {
      // dense: online softmax with the maximum tracked exactly
      float mref = -INFINITY, l = 0.f;
      for (int j = 0; j < N; ++j) {
        if (j == i) continue;
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < MP; ++c) s = fmaf(qi[c], sk[j * MP + c], s);
        s *= p.scale;
        if (s > mref) {
          const float a = expf(mref - s);
          l *= a;
#pragma unroll
          for (int c = 0; c < MP; ++c) msg[c] *= a;
          mref = s;
        }
        const float e = expf(s - mref);
        l += e;
        const float* vr = sv + j * MP;
#pragma unroll
        for (int c = 0; c < MP; ++c) msg[c] = fmaf(e, vr[c], msg[c]);
      }
      const float inv = 1.0f / l;
#pragma unroll
      for (int c = 0; c < MP; ++c) msg[c] *= inv;
    }
    float* o = p.out + ((int64_t)b * N + i) * m;
#pragma unroll
    for (int c = 0; c < MP; ++c) msg[c] = gelu_erf(msg[c]);
    for (int r = 0; r < m; ++r) {
      const float* wr = spw + r * m;
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < MP; ++c)
        if (c < m) acc = fmaf(msg[c], wr[c], acc);
      o[r] = acc + spb[r];
    }
  }
}

template <int MP, int KM, bool VEC>
__global__ void __launch_bounds__(COMM_THREADS, 1) comm_forward_kernel(CommParams p) {
  extern __shared__ __align__(16) float comm_sm[];
  const int N = p.N, D = p.in_dim, m = p.m;
  const int DS = comm_row_stride(D, VEC);
  const int M3 = 3 * m;
  float* sq = comm_sm;
  float* sk = sq + (size_t)N * MP;
  float* sv = sk + (size_t)N * MP;
  float* sx = sv + (size_t)N * MP;
  float* sg = sx + (size_t)COMM_XTILE * DS;
  float* sw = sg + COMM_THREADS;
  float* spw = sw + (p.w_smem ? (size_t)M3 * DS : 0);
  float* spb = spw + m * m;
  float* sbq = spb + m;
  const int b = blockIdx.x;
  const float* X = p.x + (int64_t)b * N * D;

  // weights and biases: every copy issued before the first wait
  if (p.w_smem) comm_stage<VEC>(sw, DS, p.wqkv, M3, D);
  for (int e = threadIdx.x; e < m * m; e += blockDim.x) cp_async4(spw + e, p.wproj + e);
  for (int e = threadIdx.x; e < m; e += blockDim.x) cp_async4(spb + e, p.bproj + e);
  for (int e = threadIdx.x; e < M3; e += blockDim.x) cp_async4(sbq + e, p.bqkv + e);
  if (m < MP)
    for (int e = threadIdx.x; e < 3 * N * MP; e += blockDim.x) sq[e] = 0.f;

  // ---- phase 1: q, k, v rows of every agent, 32 staged x rows at a time ----
  for (int r0 = 0; r0 < N; r0 += COMM_XTILE) {
    const int nr = min(COMM_XTILE, N - r0);
    __syncthreads();  // the previous tile is consumed
    comm_stage<VEC>(sx, DS, X + (int64_t)r0 * D, nr, D);
    cp_async_wait_all();
    __syncthreads();
    comm_project<MP, VEC>(p, sx, DS, sw, sbq, r0, nr, sq, sk, sv);
  }
  __syncthreads();

  // ---- phase 2: attention, GELU, projection --------------------------------
  comm_attend<MP, KM>(p, b, sq, sk, sv, sg, spw, spb);
}

// q / n through one float multiply, for 0 <= q, 1 <= n and q + n < 2^22:
// (q + 0.5) / n lies at least 0.5 / n from an integer and the rounded
// product (inv_n = 1/n rounded) is within (q + n) 2^-23 / n of it, so
// truncation gives the exact quotient.
__device__ __forceinline__ int small_div(int q, float inv_n) {
  return __float2int_rz((static_cast<float>(q) + 0.5f) * inv_n);
}

// Copy R contiguous rows of D floats into shared rows of DS floats, the
// 16-byte pieces (VEC) or words dealt over all threads in order.
template <bool VEC>
__device__ __forceinline__ void comm_stage_flat(float* dst, int DS,
                                                const float* src, int R, int D) {
  if constexpr (VEC) {
    const int D4 = D >> 2;
    const float inv = 1.0f / D4;
    for (int q = threadIdx.x; q < R * D4; q += blockDim.x) {
      const int r = small_div(q, inv), c4 = q - r * D4;
      cp_async16(dst + r * DS + 4 * c4, src + 4 * (int64_t)q);
    }
  } else {
    const float inv = 1.0f / D;
    for (int q = threadIdx.x; q < R * D; q += blockDim.x) {
      const int r = small_div(q, inv), c = q - r * D;
      cp_async4(dst + r * DS + c, src + q);
    }
  }
}

// Multi-episode form for large batches of short episodes (N <= 32, W_qkv in
// shared memory). A tile is E consecutive episodes (R = E * N <= RT rows,
// contiguous in x); blocks loop over tiles with stride gridDim.x, the weights
// staged once per block and the next tile's x rows copied in once the
// current tile's projection has consumed them. Per tile:
//   projection  thread (column c, row group g) forms q, k and v column c of
//               four rows at a time (12 accumulators): every staged W_qkv
//               piece feeds four rows, every x piece three outputs;
//   scores      one thread per (agent, key) pair of an episode;
//   selection   one thread per agent: the k best scores (lowest key index on
//               a tie), normalised weights and key indices;
//   aggregate   thread (message column c, row group g) over rows g, g + RG,
//               ...: V aggregate (top-k) or the online softmax (dense), GELU;
//   output      thread (output column c, row group g), four rows per step,
//               W_proj column c in registers (m <= 16) or read from a
//               transposed copy (consecutive threads, consecutive words).
// Row and column indices come from small_div (one float multiply) instead of
// integer division by the runtime N, m and in_dim.
// Every output is formed with the operations of comm_forward_kernel in the
// same order, so both forms give the same bits.
template <int MP>
__host__ __device__ constexpr int comm_tile_rows() {
  return 4 * (COMM_THREADS / MP) > 32 ? 4 * (COMM_THREADS / MP) : 32;
}

template <int MP, int KM, bool VEC>
__global__ void __launch_bounds__(COMM_THREADS, COMM_TILE_BPS)
    comm_tile_kernel(CommParams p, int E) {
  extern __shared__ __align__(16) float comm_sm[];
  constexpr int RG = COMM_THREADS / MP;  // row groups
  constexpr int RT = comm_tile_rows<MP>();
  constexpr int KS = KM > 0 ? KM : 1;
  const int N = p.N, D = p.in_dim, m = p.m, M3 = 3 * m;
  const int DS = comm_row_stride(D, VEC);
  float* sw = comm_sm;                    // [3m][DS]
  float* sx = sw + (size_t)M3 * DS;       // [RT][DS]
  float* sq = sx + (size_t)RT * DS;       // [RT][MP] each
  float* sk = sq + RT * MP;
  float* sv = sk + RT * MP;
  float* sg = sv + RT * MP;               // GELU(message) [RT][MP]
  float* swn = sg + RT * MP;              // normalised weights [RT][KS]
  int* sidx = reinterpret_cast<int*>(swn + RT * KS);  // key indices [RT][KS]
  float* ss = reinterpret_cast<float*>(sidx + RT * KS);  // scores [RT][N]
  float* spt = ss + RT * N;               // W_proj transposed [m][m]
  float* spb = spt + m * m;
  float* sbq = spb + m;
  const int ntile = (p.B + E - 1) / E;

  const float inv_n = 1.0f / N;
  auto stage_tile = [&](int t) {
    const int b0 = t * E;
    const int R = min(E, p.B - b0) * N;
    comm_stage_flat<VEC>(sx, DS, p.x + (int64_t)b0 * N * D, R, D);
  };

  comm_stage_flat<VEC>(sw, DS, p.wqkv, M3, D);
  const float inv_m = 1.0f / m;
  for (int e = threadIdx.x; e < m * m; e += COMM_THREADS) {
    const int oc = small_div(e, inv_m), t = e - oc * m;
    cp_async4(spt + t * m + oc, p.wproj + e);
  }
  for (int e = threadIdx.x; e < m; e += COMM_THREADS) cp_async4(spb + e, p.bproj + e);
  for (int e = threadIdx.x; e < M3; e += COMM_THREADS) cp_async4(sbq + e, p.bqkv + e);
  if (m < MP)  // padded message columns stay zero
    for (int e = threadIdx.x; e < 3 * RT * MP; e += COMM_THREADS) sq[e] = 0.f;
  if ((int)blockIdx.x < ntile) stage_tile(blockIdx.x);

  const int pc = threadIdx.x % MP, pg = threadIdx.x / MP;
  for (int tile = blockIdx.x; tile < ntile; tile += gridDim.x) {
    const int b0 = tile * E;
    const int R = min(E, p.B - b0) * N;
    cp_async_wait_all();  // this tile's x rows (and, first, the weights)
    __syncthreads();

    // ---- projection: four rows x (q, k, v) column pc per step -------------
    if (pc < m) {
      const float* w0 = sw + pc * DS;
      const float* w1 = sw + (pc + m) * DS;
      const float* w2 = sw + (pc + 2 * m) * DS;
      for (int r0 = 4 * pg; r0 < R; r0 += 4 * RG) {
        const float* x0 = sx + r0 * DS;
        float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f},
              a2[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (VEC) {
          for (int c = 0; c < D; c += 4) {
            const float4 u0 = *reinterpret_cast<const float4*>(w0 + c);
            const float4 u1 = *reinterpret_cast<const float4*>(w1 + c);
            const float4 u2 = *reinterpret_cast<const float4*>(w2 + c);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float4 xv = *reinterpret_cast<const float4*>(x0 + r * DS + c);
              a0[r] = fmaf(xv.x, u0.x, a0[r]);
              a0[r] = fmaf(xv.y, u0.y, a0[r]);
              a0[r] = fmaf(xv.z, u0.z, a0[r]);
              a0[r] = fmaf(xv.w, u0.w, a0[r]);
              a1[r] = fmaf(xv.x, u1.x, a1[r]);
              a1[r] = fmaf(xv.y, u1.y, a1[r]);
              a1[r] = fmaf(xv.z, u1.z, a1[r]);
              a1[r] = fmaf(xv.w, u1.w, a1[r]);
              a2[r] = fmaf(xv.x, u2.x, a2[r]);
              a2[r] = fmaf(xv.y, u2.y, a2[r]);
              a2[r] = fmaf(xv.z, u2.z, a2[r]);
              a2[r] = fmaf(xv.w, u2.w, a2[r]);
            }
          }
        } else {
          for (int c = 0; c < D; ++c) {
            const float u0 = w0[c], u1 = w1[c], u2 = w2[c];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float xv = x0[r * DS + c];
              a0[r] = fmaf(xv, u0, a0[r]);
              a1[r] = fmaf(xv, u1, a1[r]);
              a2[r] = fmaf(xv, u2, a2[r]);
            }
          }
        }
        const float bq0 = sbq[pc], bq1 = sbq[pc + m], bq2 = sbq[pc + 2 * m];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (r0 + r < R) {
            sq[(r0 + r) * MP + pc] = a0[r] + bq0;
            sk[(r0 + r) * MP + pc] = a1[r] + bq1;
            sv[(r0 + r) * MP + pc] = a2[r] + bq2;
          }
        }
      }
    }
    __syncthreads();  // q, k, v complete; the x tile is free
    if (tile + (int)gridDim.x < ntile) stage_tile(tile + gridDim.x);

    // ---- scores: one thread per (agent, key) pair --------------------------
    for (int it = threadIdx.x; it < R * N; it += COMM_THREADS) {
      const int r = small_div(it, inv_n), j = it - r * N;
      const float* qr = sq + r * MP;
      const float* kr = sk + (small_div(r, inv_n) * N + j) * MP;
      float s = 0.f;
#pragma unroll
      for (int t = 0; t < MP; t += 4) {
        const float4 a = *reinterpret_cast<const float4*>(qr + t);
        const float4 f = *reinterpret_cast<const float4*>(kr + t);
        s = fmaf(a.x, f.x, s);
        s = fmaf(a.y, f.y, s);
        s = fmaf(a.z, f.z, s);
        s = fmaf(a.w, f.w, s);
      }
      ss[it] = KM > 0 ? s : s * p.scale;
    }
    __syncthreads();

    // ---- selection: one thread per agent -----------------------------------
    if constexpr (KM > 0) {
      for (int r = threadIdx.x; r < R; r += COMM_THREADS) {
        const int i = r - small_div(r, inv_n) * N;
        const float* sr = ss + r * N;
        float bs[KM];
        int bi[KM];
#pragma unroll
        for (int s = 0; s < KM; ++s) {
          bs[s] = -INFINITY;
          bi[s] = -1;
        }
        for (int j = 0; j < N; ++j) {
          const float s = sr[j];
          if (j != i && s > bs[KM - 1]) buf_insert<KM, false>(bs, bi, s, j);
        }
        const int kk = p.topk;
        const float mx = bs[0] * p.scale;
        float den = 0.f, w[KM];
#pragma unroll
        for (int s = 0; s < KM; ++s) {
          w[s] = (s < kk && bi[s] >= 0) ? expf(bs[s] * p.scale - mx) : 0.f;
          den += w[s];
        }
#pragma unroll
        for (int s = 0; s < KM; ++s) {
          const bool on = w[s] > 0.f;
          swn[r * KS + s] = on ? w[s] / den : 0.f;
          sidx[r * KS + s] = on ? bi[s] : -1;
        }
      }
      __syncthreads();
    }

    // ---- aggregate and GELU: thread (column pc, row group pg) ---------------
    if (pc < m) {
      for (int r = pg; r < R; r += RG) {
        const int r0 = small_div(r, inv_n) * N;  // the episode's first row
        float msg = 0.f;
        if constexpr (KM > 0) {
#pragma unroll
          for (int s = 0; s < KM; ++s) {
            const int j = sidx[r * KS + s];
            if (j >= 0) msg = fmaf(swn[r * KS + s], sv[(r0 + j) * MP + pc], msg);
          }
        } else {
          const int i = r - r0;
          const float* sr = ss + r * N;
          float mref = -INFINITY, l = 0.f;
          for (int j = 0; j < N; ++j) {
            if (j == i) continue;
            const float s = sr[j];
            if (s > mref) {
              const float a = expf(mref - s);
              l *= a;
              msg *= a;
              mref = s;
            }
            const float e = expf(s - mref);
            l += e;
            msg = fmaf(e, sv[(r0 + j) * MP + pc], msg);
          }
          msg *= 1.0f / l;
        }
        sg[r * MP + pc] = gelu_erf(msg);
      }
    }
    __syncthreads();

    // ---- output projection: thread (column pc, row group pg), four rows ----
    // per step; W_proj column pc from registers (m <= 16) or shared memory
    if (pc < m) {
      float wc[MP <= 16 ? MP : 1];
      if constexpr (MP <= 16) {
#pragma unroll
        for (int t = 0; t < MP; ++t) wc[t] = t < m ? spt[t * m + pc] : 0.f;
      }
      const float bo = spb[pc];
      float* out = p.out + (int64_t)b0 * N * m;
      for (int r0 = 4 * pg; r0 < R; r0 += 4 * RG) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int t = 0; t < MP; t += 4) {
          float w4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if constexpr (MP <= 16) w4[u] = wc[t + u];
            else w4[u] = t + u < m ? spt[(t + u) * m + pc] : 0.f;
          }
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            const float4 gv = *reinterpret_cast<const float4*>(sg + (r0 + rr) * MP + t);
            if (t < m) acc[rr] = fmaf(gv.x, w4[0], acc[rr]);
            if (t + 1 < m) acc[rr] = fmaf(gv.y, w4[1], acc[rr]);
            if (t + 2 < m) acc[rr] = fmaf(gv.z, w4[2], acc[rr]);
            if (t + 3 < m) acc[rr] = fmaf(gv.w, w4[3], acc[rr]);
          }
        }
#pragma unroll
        for (int rr = 0; rr < 4; ++rr)
          if (r0 + rr < R) out[(r0 + rr) * m + pc] = acc[rr] + bo;
      }
    }
    // the next iteration's first barrier keeps sg and ss until every thread
    // is done with them
  }
  cp_async_wait_all();
}

// Dynamic shared memory of comm_tile_kernel (W_qkv included).
template <int MP, int KM>
static size_t comm_tile_smem_bytes(int N, int in_dim, int m, bool vec) {
  constexpr int RT = comm_tile_rows<MP>();
  const int KS = KM > 0 ? KM : 1;
  const int DS = comm_row_stride(in_dim, vec);
  return sizeof(float) * ((size_t)3 * m * DS + (size_t)RT * DS +
                          (size_t)4 * RT * MP + (size_t)2 * RT * KS +
                          (size_t)RT * N + (size_t)m * m + 4 * (size_t)m);
}

size_t comm_smem_bytes(int N, int in_dim, int m, int MP, bool vec) {
  return sizeof(float) * ((size_t)m * m + 4 * (size_t)m + (size_t)3 * N * MP +
                          (size_t)COMM_XTILE * comm_row_stride(in_dim, vec) +
                          COMM_THREADS);
}

bool comm_vec(const float* x, const float* wqkv, int in_dim) {
  return in_dim % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(wqkv) % 16 == 0;
}

// W_qkv joins the block's shared memory when the total stays within this
static constexpr size_t COMM_SMEM_WITH_W = 160 * 1024;

template <int MP, int KM, bool VEC>
static cudaError_t launch_comm_t(CommParams p, cudaStream_t s) {
  size_t sm = comm_smem_bytes(p.N, p.in_dim, p.m, MP, VEC);
  const size_t wb =
      sizeof(float) * (size_t)3 * p.m * comm_row_stride(p.in_dim, VEC);
  p.w_smem = sm + wb <= COMM_SMEM_WITH_W;
  if (p.w_smem) sm += wb;
  // Large batches of short episodes: the multi-episode tile form stages the
  // weights once per block, shares each W_qkv read among four rows and forms
  // each score once (B=4096, N=6: 41 us with one block per episode). Tiles
  // of about B / (4 * SMs) episodes, at most COMM_TILE_BPS blocks per SM.
  int dev = 0, nsm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  constexpr int RT = comm_tile_rows<MP>();
  const size_t tsm = comm_tile_smem_bytes<MP, KM>(p.N, p.in_dim, p.m, VEC);
  if (p.N <= RT && p.B >= nsm && tsm <= 220 * 1024) {
    const int bps = (int)std::min<size_t>(COMM_TILE_BPS, (220 * 1024) / tsm);
    const int E = std::max(1, std::min(RT / p.N, (p.B + 4 * nsm - 1) / (4 * nsm)));
    const int grid = std::min((p.B + E - 1) / E, bps * nsm);
    e = raise_smem_limit((const void*)comm_tile_kernel<MP, KM, VEC>, tsm);
    if (e != cudaSuccess) return e;
    comm_tile_kernel<MP, KM, VEC><<<grid, COMM_THREADS, tsm, s>>>(p, E);
    return cudaGetLastError();
  }
  e = raise_smem_limit(
      (const void*)comm_forward_kernel<MP, KM, VEC>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  comm_forward_kernel<MP, KM, VEC><<<p.B, COMM_THREADS, sm, s>>>(p);
  return cudaGetLastError();
}

template <int MP, int KM>
static cudaError_t launch_comm_v(const CommParams& p, cudaStream_t s) {
  return comm_vec(p.x, p.wqkv, p.in_dim) ? launch_comm_t<MP, KM, true>(p, s)
                                         : launch_comm_t<MP, KM, false>(p, s);
}

template <int MP>
static cudaError_t launch_comm_m(const CommParams& p, cudaStream_t s) {
  if (p.topk == 0) return launch_comm_v<MP, 0>(p, s);
  if (p.topk <= 1) return launch_comm_v<MP, 1>(p, s);
  if (p.topk <= 2) return launch_comm_v<MP, 2>(p, s);
  if (p.topk <= 4) return launch_comm_v<MP, 4>(p, s);
  return launch_comm_v<MP, 8>(p, s);
}

// m padded to 8, 16, 32 or 64 columns
int comm_padded_m(int m) { return m <= 8 ? 8 : m <= 16 ? 16 : m <= 32 ? 32 : 64; }

cudaError_t launch_comm_forward(const CommParams& p, cudaStream_t s) {
  switch (comm_padded_m(p.m)) {
    case 8: return launch_comm_m<8>(p, s);
    case 16: return launch_comm_m<16>(p, s);
    case 32: return launch_comm_m<32>(p, s);
    default: return launch_comm_m<64>(p, s);
  }
}

}  // namespace tarmac
