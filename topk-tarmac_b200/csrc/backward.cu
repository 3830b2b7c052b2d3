// backward.cu — gradients of the attention core (training path).
//
// The reference trains through its eager PyTorch path (src/agents/mappo.py:
// 192-231 topk_gather, 265-292 zorder_k, 361-373 dense) and autograd; its
// Triton kernels are forward-only (scripts/bench_attention_core.py:172-176).
// These kernels give the same gradients for the sm_100a forward kernels:
//
// Attention over a fixed peer set (top-k after selection, Morton window,
// given indices): with s_m = (q_i . k_{j_m}) * scale, w = softmax(s),
// out_i = sum_m w_m v_{j_m} and g = dL/dout,
//     ds_m = w_m (g_i . v_{j_m} - sum_m' w_m' g_i . v_{j_m'})
//     dq_i = scale * sum_m ds_m k_{j_m}
//     dk_j += scale * ds_m q_i,  dv_j += w_m g_i      for every j_m = j.
// The selection carries no gradient: torch.topk's backward scatters only into
// the selected entries, and the Morton selection depends on positions only.
//
// Dense masked-diagonal attention: P = softmax(Q K^T scale), out = P V,
// D_i = g_i . out_i,
//     dq_i = scale sum_j P_ij (g_i . v_j - D_i) k_j
//     dk_j = scale sum_i P_ij (g_i . v_j - D_i) q_i,   dv_j = sum_i P_ij g_i.
// Two kernels: one per query row (row log-sum-exp, D_i, dq_i), then one per
// key row (dk_j, dv_j) reading the first kernel's row statistics; P is
// recomputed, never stored. Deterministic (no atomics).
//
// All arithmetic is fp32 (bf16 inputs widened on load); gradients are
// written as fp32 [B, N, d], contiguous.
#include "backward.cuh"

namespace tarmac {

// CPL columns [c0, c0 + CPL) of a row as fp32, zero at and beyond d.
template <int CPL, typename T>
__device__ __forceinline__ void load_cols(float (&x)[CPL], const T* row, int c0,
                                          int d, bool vec) {
  if (vec) {
#pragma unroll
    for (int c = 0; c < CPL; c += 4) {
      if (c0 + c < d) {
        const float4 f = load4(row + c0 + c);
        x[c] = f.x; x[c + 1] = f.y; x[c + 2] = f.z; x[c + 3] = f.w;
      } else {
        x[c] = 0.f; x[c + 1] = 0.f; x[c + 2] = 0.f; x[c + 3] = 0.f;
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < CPL; ++c)
      x[c] = (c0 + c < d) ? to_f32<T>(row[c0 + c]) : 0.f;
  }
}

// Sum over the LPR lanes that share a row (aligned lane groups).
template <int LPR>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <int CPL>
__device__ __forceinline__ float dotc(const float (&a)[CPL], const float* b) {
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < CPL; ++c) s = fmaf(a[c], b[c], s);
  return s;
}

// ---------------------------------------------------------------------------
// gather attention: one group of DP/4 lanes per query row, 4 columns a lane
// ---------------------------------------------------------------------------

template <int DP, typename T, typename I>
__global__ void __launch_bounds__(128) gather_bwd_kernel(BwdParams p) {
  constexpr int LPR = DP / 4;
  constexpr int RPW = 32 / LPR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % LPR, rsub = lane / LPR;
  const int N = p.N, d = p.d;
  const int64_t rows = (int64_t)p.B * N;
  const int64_t grow = ((int64_t)blockIdx.x * 4 + warp) * RPW + rsub;
  const bool live = grow < rows;
  const int b = live ? (int)(grow / N) : 0;
  const int i = live ? (int)(grow - (int64_t)b * N) : 0;
  const int c0 = sub * 4;
  const bool vec = p.vec != 0;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.vb;
  float q4[4], g4[4];
  load_cols<4, T>(q4, static_cast<const T*>(p.q) + (int64_t)b * p.qb +
                          (int64_t)i * p.qn, c0, d, vec);
  load_cols<4, T>(g4, static_cast<const T*>(p.g) + (int64_t)b * p.gb +
                          (int64_t)i * p.gn, c0, d, vec);
  const I* ix = static_cast<const I*>(p.idx) + (live ? grow : 0) * p.kk;
  const float sc = p.scale;

  // peer m's index (clamped; `bad` records an index outside [0, N))
  bool bad = false;
  auto peer = [&](int m) {
    const int64_t j = live ? (int64_t)ix[m] : 0;
    const bool ok = j >= 0 && j < N;
    bad |= !ok;
    return ok ? (int)j : 0;
  };
  // pass A: row log-sum-exp of the kk scores
  float mx = -INFINITY, sum = 0.f;
  for (int m = 0; m < p.kk; ++m) {
    const int j = peer(m);
    float k4[4];
    load_cols<4, T>(k4, K + (int64_t)j * p.kn, c0, d, vec);
    const float s = group_sum<LPR>(dotc<4>(q4, k4)) * sc;
    if (s > mx) {
      sum = sum * expf(mx - s) + 1.f;
      mx = s;
    } else {
      sum += expf(s - mx);
    }
  }
  const float lse = mx + logf(sum);
  // pass B: D = sum_m w_m (g . v_{j_m})  (= g . out)
  float D = 0.f;
  for (int m = 0; m < p.kk; ++m) {
    const int j = peer(m);
    float k4[4], v4[4];
    load_cols<4, T>(k4, K + (int64_t)j * p.kn, c0, d, vec);
    load_cols<4, T>(v4, V + (int64_t)j * p.vn, c0, d, vec);
    const float s = group_sum<LPR>(dotc<4>(q4, k4)) * sc;
    D = fmaf(expf(s - lse), group_sum<LPR>(dotc<4>(g4, v4)), D);
  }
  // pass C: ds, dq, scatter into dk and dv
  float dq4[4] = {0.f, 0.f, 0.f, 0.f};
  const bool row_ok = live && !bad;
  float* dK = p.dk + (int64_t)b * N * d;
  float* dV = p.dv + (int64_t)b * N * d;
  // vector reductions need every row of dk and dv on a 16-byte boundary
  const bool vred = d % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(p.dk) | reinterpret_cast<uintptr_t>(p.dv)) & 15u) == 0;
  for (int m = 0; m < p.kk; ++m) {
    const int j = peer(m);
    float k4[4], v4[4];
    load_cols<4, T>(k4, K + (int64_t)j * p.kn, c0, d, vec);
    load_cols<4, T>(v4, V + (int64_t)j * p.vn, c0, d, vec);
    const float s = group_sum<LPR>(dotc<4>(q4, k4)) * sc;
    const float w = expf(s - lse);
    const float ds = w * (group_sum<LPR>(dotc<4>(g4, v4)) - D);
#pragma unroll
    for (int c = 0; c < 4; ++c) dq4[c] = fmaf(ds, k4[c], dq4[c]);
    if (row_ok) {
      float* dkr = dK + (int64_t)j * d + c0;
      float* dvr = dV + (int64_t)j * d + c0;
      if (vred) {
        // four columns per vector reduction (rows start on 16 bytes)
        if (c0 < d) {
          atomicAdd(reinterpret_cast<float4*>(dkr),
                    make_float4(sc * ds * q4[0], sc * ds * q4[1], sc * ds * q4[2],
                                sc * ds * q4[3]));
          atomicAdd(reinterpret_cast<float4*>(dvr),
                    make_float4(w * g4[0], w * g4[1], w * g4[2], w * g4[3]));
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c0 + c < d) {
            atomicAdd(dkr + c, sc * ds * q4[c]);
            atomicAdd(dvr + c, w * g4[c]);
          }
        }
      }
    }
  }
  if (!live) return;
  float* dqr = p.dq + grow * d + c0;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    if (c0 + c < d) dqr[c] = bad ? __int_as_float(0x7fc00000) : sc * dq4[c];
}

// ---------------------------------------------------------------------------
// dense attention: LPR lanes per row, CPL = DP / LPR columns a lane
// ---------------------------------------------------------------------------

constexpr int BWD_TILE = 32;  // streamed rows per shared-memory tile
constexpr float BWD_LOG2E = 1.4426950408889634f;
constexpr float BWD_RESCALE_LOG2 = 8.0f;  // see the log-sum-exp pass below

// 2^x by the hardware approximation (relative error about 2^-22; 2^-inf = 0)
__device__ __forceinline__ float bwd_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int DP>
__host__ __device__ constexpr int bwd_cpl() { return DP < 32 ? DP : 32; }

// Stage rows [r0, r0 + BWD_TILE) of a [*, d] matrix as fp32 [BWD_TILE][DP],
// zero beyond N and d (all threads of the block).
template <int DP, typename T>
__device__ __forceinline__ void stage_f32(float* dst, const T* base, int64_t rs,
                                          int r0, int N, int d) {
  for (int e = threadIdx.x; e < BWD_TILE * DP; e += blockDim.x) {
    const int r = e / DP, c = e - (e / DP) * DP;
    const int gr = r0 + r;
    dst[e] = (gr < N && c < d) ? to_f32<T>(base[(int64_t)gr * rs + c]) : 0.f;
  }
}

template <int DP, typename T>
__global__ void __launch_bounds__(128) dense_bwd_dq_kernel(BwdParams p) {
  constexpr int CPL = bwd_cpl<DP>();
  constexpr int LPR = DP / CPL;
  constexpr int RB = 128 / LPR;  // rows per block
  __shared__ __align__(16) float sk[BWD_TILE * DP];
  __shared__ __align__(16) float sv[BWD_TILE * DP];
  const int N = p.N, d = p.d;
  const int tiles_per_ep = cdiv(N, RB);
  const int b = blockIdx.x / tiles_per_ep;
  const int i0 = (blockIdx.x - b * tiles_per_ep) * RB;
  const int sub = threadIdx.x % LPR, r = threadIdx.x / LPR;
  const int i = i0 + r;
  const bool live = i < N;
  const int ii = live ? i : 0;
  const int c0 = sub * CPL;
  const bool vec = p.vec != 0;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.vb;
  float qr[CPL], gr[CPL], orow[CPL];
  load_cols<CPL, T>(qr, static_cast<const T*>(p.q) + (int64_t)b * p.qb +
                            (int64_t)ii * p.qn, c0, d, vec);
  load_cols<CPL, T>(gr, static_cast<const T*>(p.g) + (int64_t)b * p.gb +
                            (int64_t)ii * p.gn, c0, d, vec);
  load_cols<CPL, T>(orow, static_cast<const T*>(p.o) + (int64_t)b * p.ob +
                              (int64_t)ii * p.on, c0, d, vec);
  const float D = group_sum<LPR>(dotc<CPL>(gr, orow));
  const float sc = p.scale;
  const float c2 = sc * BWD_LOG2E;  // scores in base-2 exponent units

  // pass 1: row log-sum-exp (base 2) over the keys j != i. The reference
  // point moves only when a score exceeds it by more than 2^8, so each key
  // costs one exponential and the terms stay below 2^8 (no overflow).
  float mref = -INFINITY, sum = 0.f;
  for (int t0 = 0; t0 < N; t0 += BWD_TILE) {
    __syncthreads();
    stage_f32<DP, T>(sk, K, p.kn, t0, N, d);
    __syncthreads();
    const int nt = min(BWD_TILE, N - t0);
    for (int jj = 0; jj < nt; ++jj) {
      const float s = group_sum<LPR>(dotc<CPL>(qr, sk + jj * DP + c0)) * c2;
      if (t0 + jj != i) {  // no collective inside: lanes may diverge here
        if (s > mref + BWD_RESCALE_LOG2) {
          sum *= bwd_ex2(mref - s);
          mref = s;
        }
        sum += bwd_ex2(s - mref);
      }
    }
  }
  const float lse = mref + log2f(sum);
  // pass 2: dq
  float acc[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) acc[c] = 0.f;
  for (int t0 = 0; t0 < N; t0 += BWD_TILE) {
    __syncthreads();
    stage_f32<DP, T>(sk, K, p.kn, t0, N, d);
    stage_f32<DP, T>(sv, V, p.vn, t0, N, d);
    __syncthreads();
    const int nt = min(BWD_TILE, N - t0);
    for (int jj = 0; jj < nt; ++jj) {
      const float* kr = sk + jj * DP + c0;
      const float s = group_sum<LPR>(dotc<CPL>(qr, kr)) * c2;
      const float dp = group_sum<LPR>(dotc<CPL>(gr, sv + jj * DP + c0));
      const float pw = (t0 + jj == i) ? 0.f : bwd_ex2(s - lse);
      const float ds = pw * (dp - D);
#pragma unroll
      for (int c = 0; c < CPL; ++c) acc[c] = fmaf(ds, kr[c], acc[c]);
    }
  }
  if (!live) return;
  float* dqr = p.dq + ((int64_t)b * N + i) * d + c0;
#pragma unroll
  for (int c = 0; c < CPL; ++c)
    if (c0 + c < d) dqr[c] = sc * acc[c];
  if (sub == 0) {
    p.work[(int64_t)b * N + i] = lse;
    p.work[(int64_t)p.B * N + (int64_t)b * N + i] = D;
  }
}

template <int DP, typename T>
__global__ void __launch_bounds__(128) dense_bwd_dkdv_kernel(BwdParams p) {
  constexpr int CPL = bwd_cpl<DP>();
  constexpr int LPR = DP / CPL;
  constexpr int RB = 128 / LPR;
  __shared__ __align__(16) float sq[BWD_TILE * DP];
  __shared__ __align__(16) float sg[BWD_TILE * DP];
  __shared__ float slse[BWD_TILE], sD[BWD_TILE];
  const int N = p.N, d = p.d;
  const int tiles_per_ep = cdiv(N, RB);
  const int b = blockIdx.x / tiles_per_ep;
  const int j0 = (blockIdx.x - b * tiles_per_ep) * RB;
  const int sub = threadIdx.x % LPR, r = threadIdx.x / LPR;
  const int j = j0 + r;
  const bool live = j < N;
  const int jj = live ? j : 0;
  const int c0 = sub * CPL;
  const bool vec = p.vec != 0;
  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.qb;
  const T* G = static_cast<const T*>(p.g) + (int64_t)b * p.gb;
  const float* LSE = p.work + (int64_t)b * N;
  const float* DD = p.work + (int64_t)p.B * N + (int64_t)b * N;
  float kr[CPL], vr[CPL], dk[CPL], dv[CPL];
  load_cols<CPL, T>(kr, static_cast<const T*>(p.k) + (int64_t)b * p.kb +
                            (int64_t)jj * p.kn, c0, d, vec);
  load_cols<CPL, T>(vr, static_cast<const T*>(p.v) + (int64_t)b * p.vb +
                            (int64_t)jj * p.vn, c0, d, vec);
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    dk[c] = 0.f;
    dv[c] = 0.f;
  }
  const float sc = p.scale;
  const float c2 = sc * BWD_LOG2E;
  for (int t0 = 0; t0 < N; t0 += BWD_TILE) {
    __syncthreads();
    stage_f32<DP, T>(sq, Q, p.qn, t0, N, d);
    stage_f32<DP, T>(sg, G, p.gn, t0, N, d);
    if (threadIdx.x < BWD_TILE) {
      const int gi = t0 + threadIdx.x;
      slse[threadIdx.x] = gi < N ? LSE[gi] : 0.f;
      sD[threadIdx.x] = gi < N ? DD[gi] : 0.f;
    }
    __syncthreads();
    const int nt = min(BWD_TILE, N - t0);
    for (int q = 0; q < nt; ++q) {
      const float* qrow = sq + q * DP + c0;
      const float* grow = sg + q * DP + c0;
      const float s = group_sum<LPR>(dotc<CPL>(kr, qrow)) * c2;
      const float dp = group_sum<LPR>(dotc<CPL>(vr, grow));
      const float pw = (t0 + q == j) ? 0.f : bwd_ex2(s - slse[q]);
      const float ds = pw * (dp - sD[q]);
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        dv[c] = fmaf(pw, grow[c], dv[c]);
        dk[c] = fmaf(ds, qrow[c], dk[c]);
      }
    }
  }
  if (!live) return;
  float* dkr = p.dk + ((int64_t)b * N + j) * d + c0;
  float* dvr = p.dv + ((int64_t)b * N + j) * d + c0;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    if (c0 + c < d) {
      dkr[c] = sc * dk[c];
      dvr[c] = dv[c];
    }
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------

template <int DP, typename T>
static cudaError_t launch_gather_bwd_t(const BwdParams& p, cudaStream_t s) {
  constexpr int RPB = 4 * (32 / (DP / 4));  // rows per block
  const int64_t rows = (int64_t)p.B * p.N;
  const int64_t blocks = (rows + RPB - 1) / RPB;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  if (p.idx_i64)
    gather_bwd_kernel<DP, T, int64_t><<<(unsigned)blocks, 128, 0, s>>>(p);
  else
    gather_bwd_kernel<DP, T, int32_t><<<(unsigned)blocks, 128, 0, s>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_gather_bwd_dt(const BwdParams& p, cudaStream_t s) {
  if (p.d <= 4) return launch_gather_bwd_t<4, T>(p, s);
  if (p.d <= 8) return launch_gather_bwd_t<8, T>(p, s);
  if (p.d <= 16) return launch_gather_bwd_t<16, T>(p, s);
  if (p.d <= 32) return launch_gather_bwd_t<32, T>(p, s);
  if (p.d <= 64) return launch_gather_bwd_t<64, T>(p, s);
  return launch_gather_bwd_t<128, T>(p, s);
}

cudaError_t launch_gather_bwd(const BwdParams& p, int bf16, cudaStream_t s) {
  const size_t bytes = (size_t)p.B * p.N * p.d * sizeof(float);
  cudaError_t e = cudaMemsetAsync(p.dk, 0, bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p.dv, 0, bytes, s);
  if (e != cudaSuccess) return e;
  return bf16 ? launch_gather_bwd_dt<__nv_bfloat16>(p, s)
              : launch_gather_bwd_dt<float>(p, s);
}

template <int DP, typename T>
static cudaError_t launch_dense_bwd_t(const BwdParams& p, cudaStream_t s) {
  constexpr int RB = 128 / (DP / bwd_cpl<DP>());
  const int64_t blocks = (int64_t)p.B * cdiv(p.N, RB);
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  dense_bwd_dq_kernel<DP, T><<<(unsigned)blocks, 128, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dense_bwd_dkdv_kernel<DP, T><<<(unsigned)blocks, 128, 0, s>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_dense_bwd_dt(const BwdParams& p, cudaStream_t s) {
  if (p.d <= 8) return launch_dense_bwd_t<8, T>(p, s);
  if (p.d <= 16) return launch_dense_bwd_t<16, T>(p, s);
  if (p.d <= 32) return launch_dense_bwd_t<32, T>(p, s);
  if (p.d <= 64) return launch_dense_bwd_t<64, T>(p, s);
  return launch_dense_bwd_t<128, T>(p, s);
}

bool dense_bwd_tc_supported(const BwdParams& p, int bf16);
cudaError_t launch_dense_bwd_tc(const BwdParams& p, cudaStream_t s);

cudaError_t launch_dense_bwd(const BwdParams& p, int bf16, cudaStream_t s) {
  // fp32, d = 16, N >= 128: the tensor-core kernels (backward_tc.cu)
  if (dense_bwd_tc_supported(p, bf16)) return launch_dense_bwd_tc(p, s);
  return bf16 ? launch_dense_bwd_dt<__nv_bfloat16>(p, s)
              : launch_dense_bwd_dt<float>(p, s);
}

}  // namespace tarmac
