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
#include "comm.cuh"
#include "topk_chunk.cuh"

namespace tarmac {

constexpr int COMM_THREADS = 128;
constexpr int COMM_XTILE = 32;  // x rows staged per step



__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// Dynamic shared memory layout (floats): W_proj [m][m], b_proj [m], Q/K/V
// [N][MP] each (columns m..MP-1 zero), x tile [32][in_dim + 1], and, when
// p.w_smem, W_qkv [3m][in_dim + 1] (both pads put a warp's 32 reads on
// distinct banks). Without p.w_smem W_qkv is read from global memory
// through L1.
template <int MP, int KM>
__global__ void __launch_bounds__(COMM_THREADS) comm_forward_kernel(CommParams p) {
  extern __shared__ __align__(16) float comm_sm[];
  const int N = p.N, D = p.in_dim, m = p.m;
  const int DS = D + 1;
  float* spw = comm_sm;
  float* spb = spw + m * m;
  float* sq = spb + m;
  float* sk = sq + (size_t)N * MP;
  float* sv = sk + (size_t)N * MP;
  float* sx = sv + (size_t)N * MP;
  float* sw = sx + (size_t)COMM_XTILE * DS;
  const int b = blockIdx.x;
  const float* X = p.x + (int64_t)b * N * D;

  for (int e = threadIdx.x; e < m * m; e += blockDim.x) spw[e] = p.wproj[e];
  for (int e = threadIdx.x; e < m; e += blockDim.x) spb[e] = p.bproj[e];
  for (int e = threadIdx.x; e < 3 * N * MP; e += blockDim.x) sq[e] = 0.f;
  if (p.w_smem)
    for (int e = threadIdx.x; e < 3 * m * D; e += blockDim.x)
      sw[(e / D) * DS + e % D] = p.wqkv[e];

  // ---- phase 1: q, k, v rows of every agent --------------------------------
  // Threads take (row, output) pairs of the staged tile, consecutive threads
  // consecutive outputs of one row: the x row is a broadcast read, the
  // weight rows distinct banks.
  const int M3 = 3 * m;
  for (int r0 = 0; r0 < N; r0 += COMM_XTILE) {
    const int nr = min(COMM_XTILE, N - r0);
    __syncthreads();
    for (int e = threadIdx.x; e < nr * D; e += blockDim.x)
      sx[(e / D) * DS + e % D] = X[(int64_t)r0 * D + e];
    __syncthreads();
    for (int pr = threadIdx.x; pr < nr * M3; pr += blockDim.x) {
      const int rr = pr / M3, o = pr - rr * M3;
      const float* xr = sx + rr * DS;
      float acc = 0.f;
      if (p.w_smem) {
        const float* wr = sw + o * DS;
        for (int c = 0; c < D; ++c) acc = fmaf(xr[c], wr[c], acc);
      } else {
        const float* wr = p.wqkv + (int64_t)o * D;
        for (int c = 0; c < D; ++c) acc = fmaf(xr[c], __ldg(wr + c), acc);
      }
      acc += __ldg(p.bqkv + o);
      const int part = o / m, col = o - part * m;
      float* dst = part == 0 ? sq : (part == 1 ? sk : sv);
      dst[(r0 + rr) * MP + col] = acc;
    }
  }
  __syncthreads();

  // ---- phase 2: attention, GELU, projection per query agent ---------------
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

size_t comm_smem_bytes(int N, int in_dim, int m, int MP) {
  return sizeof(float) * ((size_t)m * m + m + (size_t)3 * N * MP +
                          (size_t)COMM_XTILE * (in_dim + 1));
}

// W_qkv joins the block's shared memory when the total stays within this
static constexpr size_t COMM_SMEM_WITH_W = 160 * 1024;

template <int MP, int KM>
static cudaError_t launch_comm_t(CommParams p, cudaStream_t s) {
  size_t sm = comm_smem_bytes(p.N, p.in_dim, p.m, MP);
  const size_t wb = sizeof(float) * (size_t)3 * p.m * (p.in_dim + 1);
  p.w_smem = sm + wb <= COMM_SMEM_WITH_W;
  if (p.w_smem) sm += wb;
  cudaError_t e = raise_smem_limit(
      (const void*)comm_forward_kernel<MP, KM>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  comm_forward_kernel<MP, KM><<<p.B, COMM_THREADS, sm, s>>>(p);
  return cudaGetLastError();
}

template <int MP>
static cudaError_t launch_comm_m(const CommParams& p, cudaStream_t s) {
  if (p.topk == 0) return launch_comm_t<MP, 0>(p, s);
  if (p.topk <= 1) return launch_comm_t<MP, 1>(p, s);
  if (p.topk <= 2) return launch_comm_t<MP, 2>(p, s);
  if (p.topk <= 4) return launch_comm_t<MP, 4>(p, s);
  return launch_comm_t<MP, 8>(p, s);
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
