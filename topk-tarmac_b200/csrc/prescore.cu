// prescore.cu — attention over a peer set fixed before any score exists.
//
// Restates _fused_prescore_kernel (src/kernels/fused_prescore_attention.py:
// 27-81): for each query row, walk its kk given peers in order, score each
// (q . k_j * scale), keep an online softmax (running max, normaliser,
// accumulator) and write only the result. The eager counterpart is
// prescore_attention (src/kernels/prescore_selection.py:184-195).
//
// Layout: d <= 16: one thread per query row (its softmax runs once). For
// N <= 512 with 16-byte rows, one block per episode stages the episode's K
// and V rows in shared memory and gathers the peers there; otherwise the
// peers' K and V rows are loaded from global memory two peers at a time
// before the scores.
// Wider rows: a group of L = DP/4 lanes, each owning 4 consecutive columns,
// so Q/O accesses are fully coalesced 16-byte vectors and each gathered K/V
// row is fetched as L contiguous 16-byte pieces; the partial dot products
// meet in log2(L) butterfly shuffles.
#include "prescore.cuh"

namespace tarmac {

template <int DP, typename T, typename I>
__global__ void __launch_bounds__(256) prescore_kernel(AttnParams p,
                                                       const I* __restrict__ idx,
                                                       int kk) {
  constexpr int L = DP / 4;
  constexpr int RPB = 256 / L;  // rows per block
  const int sub = threadIdx.x % L;
  const int64_t row = (int64_t)blockIdx.x * RPB + threadIdx.x / L;
  const int64_t rows = (int64_t)p.B * p.N;
  const bool live = row < rows;
  const int N = p.N;
  const int b = live ? (int)(row / N) : 0;
  const int i = live ? (int)(row - (int64_t)b * N) : 0;
  const I* ir = idx + (live ? row : 0) * kk;

  PrescoreRow<DP, T> pr;
  pr.init(p, b, i, sub, live);
  bool bad = false;
  // peers in groups of four: the group's indices, then its K and V rows, are
  // loaded together
  for (int j0 = 0; j0 < kk; j0 += 4) {
    const int cnt = min(4, kk - j0);
    int js[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int64_t pj = (live && m < cnt) ? (int64_t)ir[j0 + m] : 0;
      const bool ok = pj >= 0 && pj < N;
      bad |= !ok;
      js[m] = ok ? (int)pj : 0;
    }
    pr.template steps<4>(p, b, js, cnt, sub);
  }
  if (live) pr.finish(p, b, i, sub, bad);
}

// d <= DT (8 or 16): one query row per thread; the peers' indices, then
// their K and V rows, two peers at a time.
template <int DT, typename T, typename I>
__global__ void __launch_bounds__(256) prescore_thread_kernel(
    AttnParams p, const I* __restrict__ idx, int kk) {
  const int64_t row = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (row >= (int64_t)p.B * p.N) return;
  const int N = p.N;
  const int b = (int)(row / N);
  const int i = (int)(row - (int64_t)b * N);
  const T* Kb = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* Vb = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  PrescoreRowThread<DT, T> pr;
  pr.init(p, static_cast<const T*>(p.q) + (int64_t)b * p.st.qb +
                 (int64_t)i * p.st.qn,
          true);
  const I* ir = idx + row * kk;
  bool bad = false;
  for (int j0 = 0; j0 < kk; j0 += 2) {
    const int cnt = min(2, kk - j0);
    const T* kr[2];
    const T* vr[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int64_t pj = m < cnt ? (int64_t)ir[j0 + m] : 0;
      const bool ok = pj >= 0 && pj < N;
      bad |= !ok;
      const int64_t j = ok ? pj : 0;
      kr[m] = Kb + j * p.st.kn;
      vr[m] = Vb + j * p.st.vn;
    }
    pr.steps2(p, kr, vr, cnt);
  }
  pr.finish(p, static_cast<T*>(p.o) + (int64_t)b * p.st.ob +
                   (int64_t)i * p.st.on,
            bad);
}

// d <= DT (8 or 16), N <= 512, 16-byte rows: one block per episode with one
// query row per thread; the episode's K and V rows are first copied into
// shared memory (swizzled pieces) and the peers are gathered there, so the
// random row accesses cost shared-memory bank conflicts instead of one L1
// line lookup per lane.
template <int DT, typename T, typename I, int NT>
__global__ void __launch_bounds__(NT) prescore_episode_kernel(
    AttnParams p, const I* __restrict__ idx, int kk) {
  extern __shared__ __align__(16) unsigned char kv_smem[];
  constexpr int CPR = DT * (int)sizeof(T) / 16;
  const int N = p.N, b = blockIdx.x;
  const uint32_t sK = tc_smem_base(kv_smem);
  const uint32_t sV = sK + (uint32_t)N * CPR * 16u;
  stage_kv_episode<DT, T, NT>(p, b, sK, sV);
  cp_async_wait<0>();
  __syncthreads();
  const T* Qb = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  T* Ob = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;
  for (int i = threadIdx.x; i < N; i += NT) {
    PrescoreRowThread<DT, T> pr;
    pr.init(p, Qb + (int64_t)i * p.st.qn, true);
    const I* ir = idx + ((int64_t)b * N + i) * kk;
    bool bad = false;
    for (int j0 = 0; j0 < kk; j0 += 4) {
      const int cnt = min(4, kk - j0);
      int js[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int64_t pj = m < cnt ? (int64_t)ir[j0 + m] : 0;
        const bool ok = pj >= 0 && pj < N;
        bad |= !ok;
        js[m] = ok ? (int)pj : 0;
      }
#pragma unroll
      for (int m = 0; m < 4; ++m)
        if (m < cnt)
          pr.step_shared(p, sK, sV, js[m], [](int row, int c) {
            return kv_piece_off<DT, T>(row, c);
          });
    }
    pr.finish(p, Ob + (int64_t)i * p.st.on, bad);
  }
}

template <int DT, typename T, typename I, int NT>
static cudaError_t launch_prescore_episode(const AttnParams& p,
                                           const void* idx, int kk,
                                           cudaStream_t s) {
  const size_t sm = (size_t)2 * p.N * DT * sizeof(T);
  cudaError_t e = raise_smem_limit(
      (const void*)prescore_episode_kernel<DT, T, I, NT>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  prescore_episode_kernel<DT, T, I, NT><<<p.B, NT, sm, s>>>(
      p, static_cast<const I*>(idx), kk);
  return cudaGetLastError();
}

template <int DT, typename T, typename I>
static cudaError_t launch_prescore_thread(const AttnParams& p, const void* idx,
                                          int kk, cudaStream_t s) {
  if (kv_stageable<T>(p) && p.N <= 512) {
    if (p.N <= 128) return launch_prescore_episode<DT, T, I, 128>(p, idx, kk, s);
    if (p.N <= 256) return launch_prescore_episode<DT, T, I, 256>(p, idx, kk, s);
    return launch_prescore_episode<DT, T, I, 512>(p, idx, kk, s);
  }
  const int64_t rows = (int64_t)p.B * p.N;
  const int64_t blocks = (rows + 255) / 256;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  prescore_thread_kernel<DT, T, I><<<(unsigned)blocks, 256, 0, s>>>(
      p, static_cast<const I*>(idx), kk);
  return cudaGetLastError();
}

template <int DP, typename T, typename I>
static cudaError_t launch_prescore_t(const AttnParams& p, const void* idx,
                                     int kk, cudaStream_t s) {
  constexpr int RPB = 256 / (DP / 4);
  const int64_t rows = (int64_t)p.B * p.N;
  const int64_t blocks = (rows + RPB - 1) / RPB;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  prescore_kernel<DP, T, I><<<(unsigned)blocks, 256, 0, s>>>(
      p, static_cast<const I*>(idx), kk);
  return cudaGetLastError();
}

template <typename T, typename I>
static cudaError_t launch_prescore_ti(const AttnParams& p, const void* idx,
                                      int kk, cudaStream_t s) {
  if (p.d <= 8) return launch_prescore_thread<8, T, I>(p, idx, kk, s);
  if (p.d <= 16) return launch_prescore_thread<16, T, I>(p, idx, kk, s);
  if (p.d <= 32) return launch_prescore_t<32, T, I>(p, idx, kk, s);
  if (p.d <= 64) return launch_prescore_t<64, T, I>(p, idx, kk, s);
  return launch_prescore_t<128, T, I>(p, idx, kk, s);
}

cudaError_t launch_prescore(const AttnParams& p, int dtype, const void* idx,
                            bool idx_i64, int kk, cudaStream_t s) {
  if (dtype == TARMAC_BF16)
    return idx_i64 ? launch_prescore_ti<__nv_bfloat16, int64_t>(p, idx, kk, s)
                   : launch_prescore_ti<__nv_bfloat16, int32_t>(p, idx, kk, s);
  return idx_i64 ? launch_prescore_ti<float, int64_t>(p, idx, kk, s)
                 : launch_prescore_ti<float, int32_t>(p, idx, kk, s);
}

}  // namespace tarmac
