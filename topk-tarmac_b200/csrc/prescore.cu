// prescore.cu — attention over a peer set fixed before any score exists.
//
// Restates _fused_prescore_kernel (src/kernels/fused_prescore_attention.py:
// 27-81): for each query row, walk its kk given peers in order, score each
// (q . k_j * scale), keep an online softmax (running max, normaliser,
// accumulator) and write only the result. The eager counterpart is
// prescore_attention (src/kernels/prescore_selection.py:442-453).
//
// Layout: a row is handled by a group of L = DP/4 lanes, each owning 4
// consecutive columns, so Q/O accesses are fully coalesced 16-byte vectors and
// each gathered K/V row is fetched as L contiguous 16-byte pieces. The
// partial dot products meet in log2(L) butterfly shuffles.
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
#pragma unroll 4
  for (int j = 0; j < kk; ++j) {
    const int64_t pj = live ? (int64_t)ir[j] : 0;
    const bool ok = pj >= 0 && pj < N;
    bad |= !ok;
    pr.step(p, b, ok ? (int)pj : 0, sub);
  }
  if (live) pr.finish(p, b, i, sub, bad);
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
  if (p.d <= 8) return launch_prescore_t<8, T, I>(p, idx, kk, s);
  if (p.d <= 16) return launch_prescore_t<16, T, I>(p, idx, kk, s);
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
