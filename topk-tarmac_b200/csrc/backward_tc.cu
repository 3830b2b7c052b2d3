// backward_tc.cu — gradients of dense masked-diagonal attention on the
// tensor cores, for fp32 inputs with d = 16 (the message width of the
// reference's comm module) and at least 128 agents: the same gradients as
// the FFMA kernels of backward.cu (the reference trains its eager dense path,
// src/agents/mappo.py:361-373, through autograd), with every product
// formed as the six bf16 plane products of the exact three-plane split of
// its fp32 operands (tc_common.cuh:split3_bf16x2), small terms first, as
// the forward kernels do (dense_tc.cu).
//
// With s_ij = q_i . k_j, P_ij = 2^(s_ij c2 - lse2_i) (c2 = scale log2 e,
// lse2 the row log-sum-exp in base 2), dP_ij = g_i . v_j, D_i = g_i . out_i
// and dS_ij = P_ij (dP_ij - D_i):
//   dq_i = scale sum_j dS_ij k_j,  dk_j = scale sum_i dS_ij q_i,
//   dv_j = sum_i P_ij g_i.
// Two kernels, one block of 8 warps per 128 rows: thread t of warp w owns
// row 32 (w mod 4) + t (its TMEM lane) and columns [32 (w / 4), + 32) of
// each 64-wide tile; the first 128 threads stage the tiles, one thread
// issues the products:
// * dq: per 128 queries, a first pass over 64-key tiles forms S = Q K^T and
//   the row log-sum-exp; the second forms S and dP = dO V^T (TMEM columns
//   [0, 64) and [64, 128)), dS as three bf16 planes into shared memory
//   (the K-major A operand), and dQ += dS K (K staged MN-major) into TMEM
//   columns [128, 144). It writes lse2 and D for the second kernel.
// * dk/dv: per 128 keys and 64-query tile, S^T = K Q^T and dP^T = V dO^T,
//   then P^T (planes) for dV += P^T dO and dS^T for dK += dS^T Q (Q and dO
//   staged MN-major), accumulators in TMEM columns [128, 160).
// Deterministic (no atomics). Every wait on a product is a bounded mbarrier
// poll; a wait that runs out makes the block write NaN rows.
#include "backward.cuh"
#include "tc_common.cuh"

namespace tarmac {

constexpr int BTC_THREADS = 256;  // two threads per row, 32 columns of a tile each
constexpr int BTC_TILE = 64;   // keys (dq kernel) or queries (dk/dv kernel) per tile
constexpr int BTC_DP = 16;     // head width
constexpr float BTC_LOG2E = 1.4426950408889634f;
constexpr float BTC_RESCALE_LOG2 = 8.0f;
// plane products, small terms first: m.m, l.h, h.l, m.h, h.m, h.h
// (0 = hi, 1 = mid, 2 = lo; first = A, second = B)
__device__ constexpr int BTC_PA[6] = {1, 2, 0, 1, 0, 0};
__device__ constexpr int BTC_PB[6] = {1, 0, 2, 0, 1, 0};

namespace btc {

constexpr int KCH = BTC_DP / 8;               // 16-byte chunks per 16-column row
constexpr int RB = 128 * BTC_DP * 2;          // one plane of a 128-row tile
constexpr int TB = BTC_TILE * BTC_DP * 2;     // one plane of a 64-row tile
constexpr int WB = 128 * BTC_TILE * 2;        // one plane of a 128 x 64 weight tile
constexpr int WCH = BTC_TILE / 8;             // 16-byte chunks per weight row
constexpr uint32_t TMEM_COLS = 256;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// D[tmem] = or += A(128 x 16, K-major planes at a) . B(64 x 16, K-major
// planes at b)^T: one K step of six plane products
__device__ __forceinline__ void mma_rows_x_tile(uint32_t dt, uint32_t a, uint32_t b) {
  const uint32_t idesc = tc::idesc_bf16(128, BTC_TILE, false, false);
#pragma unroll
  for (int t = 0; t < 6; ++t)
    tc::mma_bf16(dt, tc::smem_desc(a + BTC_PA[t] * RB, 128, KCH * 128),
                 tc::smem_desc(b + BTC_PB[t] * TB, 128, KCH * 128), idesc, t > 0);
}

// D[tmem] (+)= W(128 x 64, K-major planes at w) . X(64 x 16, MN-major planes
// at x): four K steps of six plane products
__device__ __forceinline__ void mma_weights_x_tile(uint32_t dt, uint32_t w, uint32_t x,
                                                   bool accumulate) {
  const uint32_t idesc = tc::idesc_bf16(128, BTC_DP, false, true);
#pragma unroll
  for (int ks = 0; ks < BTC_TILE / 16; ++ks)
#pragma unroll
    for (int t = 0; t < 6; ++t)
      tc::mma_bf16(dt, tc::smem_desc(w + BTC_PA[t] * WB + ks * 256, 128, WCH * 128),
                   tc::smem_desc(x + BTC_PB[t] * TB + ks * 256, 128, BTC_TILE * 16),
                   idesc, accumulate || ks > 0 || t > 0);
}

// 32 fp32 values (columns 32 h .. 32 h + 31 of this thread's weight row) as
// three exact bf16 planes into the K-major weight tile (row base wrow)
__device__ __forceinline__ void store_weights32(unsigned char* wrow, int h,
                                                const float (&x)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hi[4], mi[4], lo[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      tc::split3_bf16x2(x[8 * c + 2 * u], x[8 * c + 2 * u + 1], hi[u], mi[u], lo[u]);
    unsigned char* dst = wrow + (4 * h + c) * 128;
    *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(dst + WB) = make_uint4(mi[0], mi[1], mi[2], mi[3]);
    *reinterpret_cast<uint4*>(dst + 2 * WB) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// Scores of columns [c0, c0 + 32) of row r (one of the warp's rows
// [r0, r0 + 32)) set to -inf where they must not count: the diagonal,
// columns past N, and every column of a padding row (r >= N). Warp-uniform
// test: only tiles that hold the warp's diagonal or padding are touched.
__device__ __forceinline__ void mask_edge(float (&s)[32], int c0, int r0, int r, int N) {
  if (c0 + 32 > N || r0 + 32 > N || (c0 < r0 + 32 && r0 < c0 + 32)) {
#pragma unroll
    for (int t = 0; t < 32; ++t)
      if (c0 + t >= N || c0 + t == r || r >= N) s[t] = -INFINITY;
  }
}

__device__ __forceinline__ void sync_smem_for_mma() {
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

}  // namespace btc

__global__ void __launch_bounds__(BTC_THREADS, 2) dense_bwd_tc_dq_kernel(BwdParams p) {
  using namespace btc;
  extern __shared__ __align__(16) unsigned char btc_smem[];
  unsigned char* sQ = btc_smem;          // Q rows, 3 planes
  unsigned char* sG = sQ + 3 * RB;       // dO rows, 3 planes
  unsigned char* sK = sG + 3 * RB;       // K tile, K-major
  unsigned char* sV = sK + 3 * TB;       // V tile, K-major
  unsigned char* sKm = sV + 3 * TB;      // K tile, MN-major
  unsigned char* sW = sKm + 3 * TB;      // dS, 3 planes
  __shared__ __align__(8) uint64_t mbar;
  __shared__ uint32_t tmem_sh;

  const int N = p.N, d = p.d;
  const int qblocks = cdiv(N, 128);
  const int b = blockIdx.x / qblocks;
  const int q0 = (blockIdx.x - b * qblocks) * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = threadIdx.x >> 7, wq = warp & 3;
  const bool stager = threadIdx.x < 128;
  const int row = wq * 32 + lane, i = q0 + row;
  const float* Q = static_cast<const float*>(p.q) + (int64_t)b * p.qb;
  const float* K = static_cast<const float*>(p.k) + (int64_t)b * p.kb;
  const float* V = static_cast<const float*>(p.v) + (int64_t)b * p.vb;
  const float* G = static_cast<const float*>(p.g) + (int64_t)b * p.gb;
  const float* O = static_cast<const float*>(p.o) + (int64_t)b * p.ob;
  __shared__ float red_m[2][128], red_s[2][128];
  const uint32_t qa = tc::smem_addr(sQ), ga = tc::smem_addr(sG), ka = tc::smem_addr(sK),
                 va = tc::smem_addr(sV), kma = tc::smem_addr(sKm), wa = tc::smem_addr(sW);

  float D = 0.f;
  if (i < N)
    for (int c = 0; c < d; ++c)
      D = fmaf(G[(int64_t)i * p.gn + c], O[(int64_t)i * p.on + c], D);
  if (stager) {
    tc::SplitTile<BTC_DP, 128, false> t;
    t.load(Q + (int64_t)q0 * p.qn, p.qn, N - q0, d);
    t.store(qa, RB);
    t.load(G + (int64_t)q0 * p.gn, p.gn, N - q0, d);
    t.store(ga, RB);
  }
  if (warp == 0) tc::tmem_alloc(&tmem_sh, TMEM_COLS);
  if (threadIdx.x == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init_fence();
  }
  sync_smem_for_mma();
  const uint32_t tmem = tmem_sh;
  const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
  const uint32_t t_s = tmem, t_dp = tmem + 64, t_dq = tmem + 128;
  const int cb = 32 * half;  // this thread's first column of a tile
  uint32_t phase = 0;
  bool ok = true;
  auto wait_products = [&]() {
    ok &= tc::mbar_wait(&mbar, phase & 1);
    ++phase;
    tc::fence_after_sync();
  };
  const float c2 = p.scale * BTC_LOG2E;
  const int tiles = cdiv(N, BTC_TILE);
  unsigned char* wrow = sW + (row >> 3) * WCH * 128 + (row & 7) * 16;

  // The next tile's rows are loaded into registers while the current one
  // is in the products and the exponentials (first 128 threads).
  tc::SplitTile<BTC_DP, BTC_TILE, false> kt, vt;
  tc::SplitTile<BTC_DP, BTC_TILE, true> kmt;

  // pass 1: row log-sum-exp (base 2) over the keys j != i, each thread over
  // its 32 columns of every tile; the reference point moves only when a
  // score exceeds it by more than 2^8
  // the reference starts finite, so a masked score (-inf) adds 2^-inf = 0
  float mref = -1e30f, sum = 0.f;
  if (stager) kt.load(K, p.kn, N, d);
  for (int j = 0; j < tiles; ++j) {
    const int k0 = j * BTC_TILE;
    if (stager) {
      kt.store(ka, TB);
      if (j + 1 < tiles)
        kt.load(K + (int64_t)(k0 + BTC_TILE) * p.kn, p.kn, N - k0 - BTC_TILE, d);
    }
    sync_smem_for_mma();
    if (threadIdx.x == 0) {
      mma_rows_x_tile(t_s, qa, ka);
      tc::mma_commit(&mbar);
    }
    wait_products();
    {
      float s[32];
      tc::tmem_ld32(t_s + lane_off + cb, s);
      mask_edge(s, k0 + cb, q0 + wq * 32, i, N);
      // the reference moves at most once a tile, to the tile's maximum
      float mt = s[0];
#pragma unroll
      for (int t = 1; t + 1 < 32; t += 2) mt = max3f(mt, s[t], s[t + 1]);
      mt = fmaxf(mt, s[31]) * c2;
      if (mt > mref + BTC_RESCALE_LOG2) {
        sum *= btc::ex2(mref - mt);
        mref = mt;
      }
#pragma unroll
      for (int t = 0; t < 32; ++t) sum += btc::ex2(fmaf(s[t], c2, -mref));
    }
    tc::fence_before_sync();
    __syncthreads();  // S read by every thread before the next product
  }
  // the two halves of the row combine their partial sums
  red_m[half][row] = mref;
  red_s[half][row] = sum;
  __syncthreads();
  float lse2;
  {
    const float mo = red_m[half ^ 1][row], so = red_s[half ^ 1][row];
    const float m = fmaxf(mref, mo);
    lse2 = m + log2f(sum * btc::ex2(mref - m) + so * btc::ex2(mo - m));
    if (i >= N) lse2 = 0.f;  // a padding row: every score is masked below
  }

  // pass 2: dS and dQ
  if (stager) {
    kt.load(K, p.kn, N, d);
    vt.load(V, p.vn, N, d);
  }
  for (int j = 0; j < tiles; ++j) {
    const int k0 = j * BTC_TILE;
    if (stager) {
      kt.store(ka, TB);
      kmt.x[0][0] = kt.x[0][0];  // the same rows, MN-major for dQ += dS K
      kmt.x[0][1] = kt.x[0][1];
      kmt.store(kma, TB);
      vt.store(va, TB);
      if (j + 1 < tiles) {
        kt.load(K + (int64_t)(k0 + BTC_TILE) * p.kn, p.kn, N - k0 - BTC_TILE, d);
        vt.load(V + (int64_t)(k0 + BTC_TILE) * p.vn, p.vn, N - k0 - BTC_TILE, d);
      }
    }
    sync_smem_for_mma();
    if (threadIdx.x == 0) {
      mma_rows_x_tile(t_s, qa, ka);
      mma_rows_x_tile(t_dp, ga, va);
      tc::mma_commit(&mbar);
    }
    wait_products();
    {
      float s[32], dp[32];
      tc::tmem_ld32(t_s + lane_off + cb, s);
      tc::tmem_ld32(t_dp + lane_off + cb, dp);
      mask_edge(s, k0 + cb, q0 + wq * 32, i, N);
#pragma unroll
      for (int t = 0; t < 32; ++t) s[t] = btc::ex2(fmaf(s[t], c2, -lse2)) * (dp[t] - D);
      store_weights32(wrow, half, s);
    }
    sync_smem_for_mma();
    if (threadIdx.x == 0) {
      mma_weights_x_tile(t_dq, wa, kma, j > 0);
      tc::mma_commit(&mbar);
    }
    wait_products();  // dS and the K tiles are free again
  }

  float dq[BTC_DP];
#pragma unroll
  for (int c = 0; c < BTC_DP; c += 8) {
    float o8[8];
    tc::tmem_ld8(t_dq + lane_off + c, o8);
#pragma unroll
    for (int u = 0; u < 8; ++u) dq[c + u] = o8[u];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
  if (i >= N || half != 0) return;
  float* dqr = p.dq + ((int64_t)b * N + i) * d;
#pragma unroll
  for (int c = 0; c < BTC_DP; ++c)
    if (c < d) dqr[c] = ok ? p.scale * dq[c] : __int_as_float(0x7fc00000);
  p.work[(int64_t)b * N + i] = ok ? lse2 : __int_as_float(0x7fc00000);
  p.work[(int64_t)p.B * N + (int64_t)b * N + i] = D;
}

__global__ void __launch_bounds__(BTC_THREADS, 2) dense_bwd_tc_dkdv_kernel(BwdParams p) {
  using namespace btc;
  extern __shared__ __align__(16) unsigned char btc_smem[];
  unsigned char* sK = btc_smem;          // K rows, 3 planes (A of S^T)
  unsigned char* sV = sK + 3 * RB;       // V rows (A of dP^T)
  unsigned char* sQ = sV + 3 * RB;       // Q tile, K-major (B of S^T)
  unsigned char* sG = sQ + 3 * TB;       // dO tile, K-major (B of dP^T)
  unsigned char* sQm = sG + 3 * TB;      // Q tile, MN-major (B of dK)
  unsigned char* sGm = sQm + 3 * TB;     // dO tile, MN-major (B of dV)
  unsigned char* sW = sGm + 3 * TB;      // P^T, then dS^T, 3 planes
  __shared__ float slse[BTC_TILE], sD[BTC_TILE];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ uint32_t tmem_sh;

  const int N = p.N, d = p.d;
  const int kblocks = cdiv(N, 128);
  const int b = blockIdx.x / kblocks;
  const int j0 = (blockIdx.x - b * kblocks) * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = threadIdx.x >> 7, wq = warp & 3;
  const bool stager = threadIdx.x < 128;
  const int row = wq * 32 + lane, jr = j0 + row;
  const float* Q = static_cast<const float*>(p.q) + (int64_t)b * p.qb;
  const float* K = static_cast<const float*>(p.k) + (int64_t)b * p.kb;
  const float* V = static_cast<const float*>(p.v) + (int64_t)b * p.vb;
  const float* G = static_cast<const float*>(p.g) + (int64_t)b * p.gb;
  const float* LSE = p.work + (int64_t)b * N;
  const float* DD = p.work + (int64_t)p.B * N + (int64_t)b * N;
  const uint32_t ka = tc::smem_addr(sK), va = tc::smem_addr(sV), qa = tc::smem_addr(sQ),
                 ga = tc::smem_addr(sG), qma = tc::smem_addr(sQm), gma = tc::smem_addr(sGm),
                 wa = tc::smem_addr(sW);
  if (stager) {
    tc::SplitTile<BTC_DP, 128, false> t;
    t.load(K + (int64_t)j0 * p.kn, p.kn, N - j0, d);
    t.store(ka, RB);
    t.load(V + (int64_t)j0 * p.vn, p.vn, N - j0, d);
    t.store(va, RB);
  }
  if (warp == 0) tc::tmem_alloc(&tmem_sh, TMEM_COLS);
  if (threadIdx.x == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init_fence();
  }
  sync_smem_for_mma();
  const uint32_t tmem = tmem_sh;
  const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
  const uint32_t t_s = tmem, t_dp = tmem + 64, t_dk = tmem + 128, t_dv = tmem + 144;
  const int cb = 32 * half;  // this thread's first column of a tile
  uint32_t phase = 0;
  bool ok = true;
  auto wait_products = [&]() {
    ok &= tc::mbar_wait(&mbar, phase & 1);
    ++phase;
    tc::fence_after_sync();
  };
  const float c2 = p.scale * BTC_LOG2E;
  const int tiles = cdiv(N, BTC_TILE);
  unsigned char* wrow = sW + (row >> 3) * WCH * 128 + (row & 7) * 16;

  // the next query tile's rows load into registers during this one
  tc::SplitTile<BTC_DP, BTC_TILE, false> qt, gt;
  tc::SplitTile<BTC_DP, BTC_TILE, true> mt;
  if (stager) {
    qt.load(Q, p.qn, N, d);
    gt.load(G, p.gn, N, d);
  }
  for (int it = 0; it < tiles; ++it) {
    const int i0 = it * BTC_TILE;
    if (stager) {
      qt.store(qa, TB);
      mt.x[0][0] = qt.x[0][0];
      mt.x[0][1] = qt.x[0][1];
      mt.store(qma, TB);
      gt.store(ga, TB);
      mt.x[0][0] = gt.x[0][0];
      mt.x[0][1] = gt.x[0][1];
      mt.store(gma, TB);
      if (it + 1 < tiles) {
        qt.load(Q + (int64_t)(i0 + BTC_TILE) * p.qn, p.qn, N - i0 - BTC_TILE, d);
        gt.load(G + (int64_t)(i0 + BTC_TILE) * p.gn, p.gn, N - i0 - BTC_TILE, d);
      }
    }
    if (threadIdx.x < BTC_TILE) {
      const int gi = i0 + threadIdx.x;
      slse[threadIdx.x] = gi < N ? LSE[gi] : 0.f;
      sD[threadIdx.x] = gi < N ? DD[gi] : 0.f;
    }
    sync_smem_for_mma();
    if (threadIdx.x == 0) {
      mma_rows_x_tile(t_s, ka, qa);
      mma_rows_x_tile(t_dp, va, ga);
      tc::mma_commit(&mbar);
    }
    wait_products();
    // P^T for dV; the weights stay in registers for dS^T
    float pw[32];
    tc::tmem_ld32(t_s + lane_off + cb, pw);
    mask_edge(pw, i0 + cb, j0 + wq * 32, jr, N);
#pragma unroll
    for (int t = 0; t < 32; ++t) pw[t] = btc::ex2(fmaf(pw[t], c2, -slse[cb + t]));
    store_weights32(wrow, half, pw);
    sync_smem_for_mma();
    if (threadIdx.x == 0) {
      mma_weights_x_tile(t_dv, wa, gma, it > 0);
      tc::mma_commit(&mbar);
    }
    wait_products();  // P^T read: the weight tile takes dS^T next
    // dS^T for dK
    {
      float dp[32];
      tc::tmem_ld32(t_dp + lane_off + cb, dp);
#pragma unroll
      for (int t = 0; t < 32; ++t) pw[t] *= dp[t] - sD[cb + t];
      store_weights32(wrow, half, pw);
    }
    sync_smem_for_mma();
    if (threadIdx.x == 0) {
      mma_weights_x_tile(t_dk, wa, qma, it > 0);
      tc::mma_commit(&mbar);
    }
    wait_products();  // every tile of this round is free again
  }

  // the first half of the threads reads dK, the second dV
  float acc[BTC_DP];
  const uint32_t t_acc = half == 0 ? t_dk : t_dv;
#pragma unroll
  for (int c = 0; c < BTC_DP; c += 8) {
    float o8[8];
    tc::tmem_ld8(t_acc + lane_off + c, o8);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc[c + u] = o8[u];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
  if (jr >= N) return;
  float* dst = (half == 0 ? p.dk : p.dv) + ((int64_t)b * N + jr) * d;
  const float f = half == 0 ? p.scale : 1.0f;
  const float nan = __int_as_float(0x7fc00000);
#pragma unroll
  for (int c = 0; c < BTC_DP; ++c)
    if (c < d) dst[c] = ok ? f * acc[c] : nan;
}

// fp32, d = 16, 16-byte aligned q/k/v/dO rows, at least 128 agents (below
// that, and at d = 8, the FFMA kernels were faster)
bool dense_bwd_tc_supported(const BwdParams& p, int bf16) {
  const auto a16 = [](const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; };
  return !bf16 && p.N >= 128 && p.d == 16 && a16(p.q) && a16(p.k) &&
         a16(p.v) && a16(p.g) && p.qn % 4 == 0 && p.kn % 4 == 0 && p.vn % 4 == 0 &&
         p.gn % 4 == 0 && p.qb % 4 == 0 && p.kb % 4 == 0 && p.vb % 4 == 0 &&
         p.gb % 4 == 0;
}

cudaError_t launch_dense_bwd_tc(const BwdParams& p, cudaStream_t s) {
  using namespace btc;
  constexpr size_t dq_smem = 2 * 3 * RB + 3 * 3 * TB + 3 * WB;
  constexpr size_t dkdv_smem = 2 * 3 * RB + 4 * 3 * TB + 3 * WB;
  cudaError_t e = raise_smem_limit((const void*)dense_bwd_tc_dq_kernel, dq_smem);
  if (e == cudaSuccess)
    e = raise_smem_limit((const void*)dense_bwd_tc_dkdv_kernel, dkdv_smem);
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.B * cdiv(p.N, 128);
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  dense_bwd_tc_dq_kernel<<<(unsigned)blocks, BTC_THREADS, dq_smem, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dense_bwd_tc_dkdv_kernel<<<(unsigned)blocks, BTC_THREADS, dkdv_smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace tarmac
