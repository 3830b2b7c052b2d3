// dense_tc.cu — dense masked-diagonal attention on the fifth-generation
// tensor cores (tcgen05, TMEM accumulators), for bf16 and fp32 inputs.
//
// Same function as dense.cu and the reference's _flash_dense_kernel
// (src/kernels/fused_dense_attention.py:38-99): softmax(q k^T * scale) v with
// the diagonal excluded, an online softmax, no score matrix in global memory.
// * bf16: bf16 x bf16 products accumulate in fp32 (the reference's bf16
//   path); the softmax weights enter the second product as bf16, as the
//   reference's `tl.dot(p.to(v.dtype), v)` does.
// * fp32 (d <= 16): Q, K and V are split exactly into three bf16 planes
//   (tc_common.cuh:split3_bf16x2), and so are the softmax weights P; each
//   product is the six-plane-product sum (small terms first), an
//   fp32-accurate result. K and V tiles go through registers (loaded at the
//   top of a tile, split into their ring slots once those are free).
//
// One block (4 warps) owns 128 queries of one episode; thread t of warp w
// owns query row 32*w + t, its TMEM lane. Per tile of 64 keys:
// * S = Q K^T (M = 128, N = 64) into TMEM columns [0, 64), issued by one
//   thread as soon as the tile's K is staged.
// * Each thread reads its 64 scores, masks the diagonal and the padding,
//   and updates a base-2 online softmax whose reference maximum moves only
//   when a score exceeds it by more than 2^8 (the stale maximum bounds every
//   weight by 2^8; the final division cancels the reference point). When it
//   moves, the thread rescales its row of the output accumulator in TMEM.
//   The weights go to shared memory as bf16 in the K-major A-operand layout.
// * O += P V (M = 128, N = d, K = 64) into TMEM columns [64, 64 + d), with
//   V staged MN-major (its rows are the contraction dimension).
// K and V tiles stream through two-slot rings with 16-byte cp.async; the
// next tile loads while the current one is in the softmax. The next tile's
// Q K^T is issued ahead of the current tile's P V, so the softmax waits only
// for its scores, and P V runs under the next softmax's exponentials. The weights
// come from ex2.approx (relative error ~2^-22, far below their bf16
// rounding).
#include "tc_common.cuh"

namespace tarmac {

constexpr int DTC_THREADS = 128;
constexpr int DTC_KEYS = 64;  // keys per tile
constexpr float DTC_LOG2E = 1.4426950408889634f;
constexpr float DTC_RESCALE_LOG2 = 8.0f;

template <int DP>
__host__ __device__ constexpr int dtc_tmem_cols() {
  return DTC_KEYS + DP <= 128 ? 128 : 256;
}

// bytes of shared memory: Q, two-slot K and V rings and the weights P, each
// in PL bf16 planes (1, or 3 for fp32)
template <int DP>
__host__ __device__ constexpr size_t dtc_smem_bytes(int PL) {
  return (size_t)PL * ((size_t)128 * DP * 2            // Q
                       + (size_t)2 * DTC_KEYS * DP * 2 // K ring
                       + (size_t)2 * DTC_KEYS * DP * 2 // V ring
                       + (size_t)128 * DTC_KEYS * 2);  // P
}

// plane products of a split operand pair, small terms first: m.m, l.h, h.l,
// m.h, h.m, h.h (plane 0 = hi, 1 = mid, 2 = lo; first = A, second = B)
__device__ constexpr int DTC_PA[6] = {1, 2, 0, 1, 0, 0};
__device__ constexpr int DTC_PB[6] = {1, 0, 2, 0, 1, 0};

template <typename T, int DP>
__global__ void __launch_bounds__(DTC_THREADS,
                                  sizeof(T) == 4 ? 2 : (DP >= 128 ? 2 : 3))
    dense_tc_kernel(AttnParams p, int vec16) {
  constexpr bool F32 = sizeof(T) == 4;
  constexpr int PL = F32 ? 3 : 1;            // bf16 planes per operand
  constexpr int KCH = DP / 8;               // 16-byte chunks per Q/K row
  constexpr int QB = 128 * DP * 2;          // bytes of one Q plane
  constexpr int KB = DTC_KEYS * DP * 2;     // bytes of one K or V tile plane
  constexpr int PB = 128 * DTC_KEYS * 2;    // bytes of one P plane
  constexpr int PCH = DTC_KEYS / 8;         // 16-byte chunks per P row
  static_assert(!F32 || DP == 16, "fp32 path: d <= 16");
  extern __shared__ __align__(16) unsigned char dtc_smem[];
  unsigned char* sQ = dtc_smem;             // PL planes
  unsigned char* sK = sQ + PL * QB;         // 2 slots x PL planes
  unsigned char* sV = sK + 2 * PL * KB;     // 2 slots x PL planes
  unsigned char* sP = sV + 2 * PL * KB;     // PL planes of 128 x 64, K-major
  __shared__ __align__(8) uint64_t mbar_s, mbar_pv;
  __shared__ uint32_t tmem_sh;

  const int N = p.N, d = p.d;
  const int qblocks = cdiv(N, 128);
  const int b = blockIdx.x / qblocks;
  const int q0 = (blockIdx.x - b * qblocks) * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = warp * 32 + lane;
  const int i = q0 + row;
  const bool vec = p.vec != 0;
  const bool v16 = vec16 != 0;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  const uint32_t qa = tc::smem_addr(sQ), ka = tc::smem_addr(sK),
                 va = tc::smem_addr(sV), pa = tc::smem_addr(sP);
  // bf16: K (or V) rows [r0, r0 + 64) into ring slot sl by cp.async
  auto stage_k = [&](int sl, int r0) {
    if constexpr (!F32) {
      if (v16)
        tc::stage_fast<DP, DTC_KEYS, false>(ka + sl * KB,
                                            K + (int64_t)r0 * p.st.kn, p.st.kn,
                                            N - r0, d);
      else
        tc::stage_kmajor<DP>(sK + sl * KB, K, p.st.kn, r0, DTC_KEYS, N, d,
                             false);
    }
  };
  auto stage_v = [&](int sl, int r0) {
    if constexpr (!F32) {
      if (v16)
        tc::stage_fast<DP, DTC_KEYS, true>(va + sl * KB,
                                           V + (int64_t)r0 * p.st.vn, p.st.vn,
                                           N - r0, d);
      else
        tc::stage_mnmajor<DP>(sV + sl * KB, V, p.st.vn, r0, DTC_KEYS, N, d,
                              false);
    }
  };
  // fp32: the next K and V tiles in registers (loaded at the top of a tile,
  // split into their ring slots once those are free)
  tc::SplitTile<DP, DTC_KEYS, false> kpre;
  tc::SplitTile<DP, DTC_KEYS, true> vpre;
  const float* Kf = reinterpret_cast<const float*>(K);
  const float* Vf = reinterpret_cast<const float*>(V);
  if constexpr (F32) {
    tc::SplitTile<DP, 128, false> qt;
    qt.load(reinterpret_cast<const float*>(Q) + (int64_t)q0 * p.st.qn, p.st.qn,
            N - q0, d);
    kpre.load(Kf, p.st.kn, N, d);
    vpre.load(Vf, p.st.vn, N, d);
    qt.store(qa, QB);
    kpre.store(ka, KB);
    vpre.store(va, KB);
  } else {
    if (v16)
      tc::stage_fast<DP, 128, false>(qa, Q + (int64_t)q0 * p.st.qn, p.st.qn,
                                     N - q0, d);
    else
      tc::stage_kmajor<DP>(sQ, Q, p.st.qn, q0, 128, N, d, false);
    stage_k(0, 0);
    stage_v(0, 0);
  }
  if (warp == 0) tc::tmem_alloc(&tmem_sh, dtc_tmem_cols<DP>());
  if (threadIdx.x == 0) {
    tc::mbar_init(&mbar_s, 1);
    tc::mbar_init(&mbar_pv, 1);
    tc::mbar_init_fence();
  }
  cp_async_wait_all();
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_sh;
  const uint32_t t_s = tmem, t_o = tmem + DTC_KEYS;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t idesc_s = tc::idesc_bf16(128, DTC_KEYS, false, false);
  const uint32_t idesc_o = tc::idesc_bf16(128, DP, false, true);

  auto issue_s = [&](int slot) {
    const uint32_t kt = ka + slot * (PL * KB);
#pragma unroll
    for (int ks = 0; ks < DP / 16; ++ks) {
#pragma unroll
      for (int t = 0; t < (F32 ? 6 : 1); ++t) {
        const int a = F32 ? DTC_PA[t] : 0, bpl = F32 ? DTC_PB[t] : 0;
        tc::mma_bf16(t_s,
                     tc::smem_desc(qa + a * QB + ks * 256, 128, KCH * 128),
                     tc::smem_desc(kt + bpl * KB + ks * 256, 128, KCH * 128),
                     idesc_s, ks > 0 || t > 0);
      }
    }
    tc::mma_commit(&mbar_s);
  };
  if (threadIdx.x == 0) issue_s(0);

  const float c2 = p.qscale * p.post_scale * DTC_LOG2E;
  float mref = -1e30f;         // reference maximum in exponent units
  float mth = -INFINITY;       // raw score above which the reference moves
  float l = 0.f;
  bool ok = true;
  const int tiles = cdiv(N, DTC_KEYS);
  unsigned char* prow = sP + (row >> 3) * PCH * 128 + (row & 7) * 16;

  // Per tile j: S_j was issued ahead of P V_{j-1}, so its wait does not
  // include that product; P V_{j-1} is awaited only once the weights are in
  // registers, just before P, the accumulator and V's ring slot are reused.
  for (int j = 0; j < tiles; ++j) {
    const int k0 = j * DTC_KEYS;
    const bool more = j + 1 < tiles;
    ok &= tc::mbar_wait(&mbar_s, (uint32_t)(j & 1));
    tc::fence_after_sync();
    // K slot (j + 1) & 1 last held tile j - 1, whose Q K^T has completed
    if constexpr (F32) {
      if (more) {
        kpre.load(Kf + (int64_t)(k0 + DTC_KEYS) * p.st.kn, p.st.kn,
                  N - k0 - DTC_KEYS, d);
        vpre.load(Vf + (int64_t)(k0 + DTC_KEYS) * p.st.vn, p.st.vn,
                  N - k0 - DTC_KEYS, d);
      }
    } else {
      if (more) {
        stage_k((j + 1) & 1, k0 + DTC_KEYS);
        cp_async_commit();
      }
    }
    float s[DTC_KEYS];
    {
      float h[32];
      tc::tmem_ld32(t_s + lane_off, h);
#pragma unroll
      for (int t = 0; t < 32; ++t) s[t] = h[t];
      tc::tmem_ld32(t_s + lane_off + 32, h);
#pragma unroll
      for (int t = 0; t < 32; ++t) s[32 + t] = h[t];
    }
    // warp-uniform: the tile holds padding or this warp's diagonal
    if (k0 + DTC_KEYS > N || (k0 < q0 + warp * 32 + 32 && q0 + warp * 32 < k0 + DTC_KEYS)) {
#pragma unroll
      for (int t = 0; t < DTC_KEYS; ++t)
        if (k0 + t >= N || k0 + t == i) s[t] = -INFINITY;
    }
    float mt = s[0];
#pragma unroll
    for (int t = 1; t + 1 < DTC_KEYS; t += 2) mt = max3f(mt, s[t], s[t + 1]);
    mt = fmaxf(mt, s[DTC_KEYS - 1]);
    const bool move = mt > mth;
    float alpha = 1.0f;
    if (move) {
      const float mn = mt * c2;
      alpha = tc::ex2_approx(mref - mn);
      l *= alpha;
      mref = mn;
      mth = mt + DTC_RESCALE_LOG2 / c2;
    }
#pragma unroll
    for (int t = 0; t < DTC_KEYS; ++t) {
      s[t] = tc::ex2_approx(fmaf(s[t], c2, -mref));
      l += s[t];
    }

    // P V_{j-1} complete: P, the accumulator and V slot (j + 1) & 1 are free
    if (j >= 1) {
      ok &= tc::mbar_wait(&mbar_pv, (uint32_t)((j - 1) & 1));
      tc::fence_after_sync();
    }
    if constexpr (F32) {
      // K slot (j + 1) & 1 is free (Q K^T_{j-1} done), V slot (j + 1) & 1
      // too (P V_{j-1} done)
      if (more) {
        kpre.store(ka + ((j + 1) & 1) * (PL * KB), KB);
        vpre.store(va + ((j + 1) & 1) * (PL * KB), KB);
      }
    } else {
      if (more) {
        stage_v((j + 1) & 1, k0 + DTC_KEYS);
        cp_async_commit();
      }
    }
    // TMEM loads and stores are warp-collective: the whole warp rescales
    // when any lane moved its reference (the others multiply by 1)
    if (j > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll
      for (int c = 0; c < DP; c += 8) {
        float o8[8];
        tc::tmem_ld8(t_o + lane_off + c, o8);
#pragma unroll
        for (int u = 0; u < 8; ++u) o8[u] *= alpha;
        tc::tmem_st8(t_o + lane_off + c, o8);
      }
    }
    if constexpr (F32) {
      // weights in [0, 2^8]: three exact bf16 planes
#pragma unroll
      for (int c = 0; c < PCH; ++c) {
        uint32_t h[4], m[4], l[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          tc::split3_bf16x2(s[8 * c + 2 * u], s[8 * c + 2 * u + 1], h[u], m[u],
                            l[u]);
        *reinterpret_cast<uint4*>(prow + c * 128) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(prow + PB + c * 128) = make_uint4(m[0], m[1], m[2], m[3]);
        *reinterpret_cast<uint4*>(prow + 2 * PB + c * 128) = make_uint4(l[0], l[1], l[2], l[3]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < PCH; ++c) {
        uint4 w;
        w.x = tc::pack_bf16x2(s[8 * c], s[8 * c + 1]);
        w.y = tc::pack_bf16x2(s[8 * c + 2], s[8 * c + 3]);
        w.z = tc::pack_bf16x2(s[8 * c + 4], s[8 * c + 5]);
        w.w = tc::pack_bf16x2(s[8 * c + 6], s[8 * c + 7]);
        *reinterpret_cast<uint4*>(prow + c * 128) = w;
      }
      // this thread's K_{j+1} and V_j have landed (V_{j+1} may be in flight)
      if (more)
        cp_async_wait<1>();
      else
        cp_async_wait<0>();
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (threadIdx.x == 0) {
      if (more) issue_s((j + 1) & 1);
      const uint32_t vt = va + (j & 1) * (PL * KB);
#pragma unroll
      for (int ks = 0; ks < DTC_KEYS / 16; ++ks) {
#pragma unroll
        for (int t = 0; t < (F32 ? 6 : 1); ++t) {
          const int a = F32 ? DTC_PA[t] : 0, bpl = F32 ? DTC_PB[t] : 0;
          tc::mma_bf16(t_o,
                       tc::smem_desc(pa + a * PB + ks * 256, 128, PCH * 128),
                       tc::smem_desc(vt + bpl * KB + ks * 256, 128,
                                     DTC_KEYS * 16),
                       idesc_o, j > 0 || ks > 0 || t > 0);
        }
      }
      tc::mma_commit(&mbar_pv);
    }
  }
  ok &= tc::mbar_wait(&mbar_pv, (uint32_t)((tiles - 1) & 1));
  tc::fence_after_sync();

  float o[DP];
#pragma unroll
  for (int c = 0; c < DP; c += 8) {
    float o8[8];
    tc::tmem_ld8(t_o + lane_off + c, o8);
#pragma unroll
    for (int u = 0; u < 8; ++u) o[c + u] = o8[u];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, dtc_tmem_cols<DP>());
  if (i >= N) return;
  const float inv = 1.0f / l;
#pragma unroll
  for (int c = 0; c < DP; ++c)
    o[c] = ok ? o[c] * inv : __int_as_float(0x7fc00000);
  store_row<DP, T>(O + (int64_t)i * p.st.on, o, d, vec);
}

template <typename T, int DP>
static cudaError_t launch_dtc(const AttnParams& p, int vec16, cudaStream_t s) {
  const size_t sm = dtc_smem_bytes<DP>(sizeof(T) == 4 ? 3 : 1);
  cudaError_t e = raise_smem_limit(
      (const void*)dense_tc_kernel<T, DP>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.B * cdiv(p.N, 128);
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  dense_tc_kernel<T, DP><<<(unsigned)blocks, DTC_THREADS, sm, s>>>(p, vec16);
  return cudaGetLastError();
}

// bf16, N >= 128: is the tensor-core dense path available?
// bf16 episodes from 65 agents: below 128 one part-filled 128-row tile
// still beats the FFMA kernel (B=1024, d=16: N=65 16.3 vs 24.7 us).
bool dense_tc_supported(const AttnParams& p) {
  return p.N >= 65 && p.d <= 128;
}

cudaError_t launch_dense_tc(const AttnParams& p, cudaStream_t s) {
  using B16 = __nv_bfloat16;
  const uintptr_t qa = reinterpret_cast<uintptr_t>(p.q);
  const uintptr_t ka = reinterpret_cast<uintptr_t>(p.k);
  const uintptr_t va = reinterpret_cast<uintptr_t>(p.v);
  const int vec16 = (p.d % 8 == 0) && (qa % 16 == 0) && (ka % 16 == 0) &&
                    (va % 16 == 0) && (p.st.qn % 8 == 0) &&
                    (p.st.kn % 8 == 0) && (p.st.vn % 8 == 0) &&
                    (p.st.qb % 8 == 0) && (p.st.kb % 8 == 0) &&
                    (p.st.vb % 8 == 0);
  if (p.d <= 16) return launch_dtc<B16, 16>(p, vec16, s);
  if (p.d <= 32) return launch_dtc<B16, 32>(p, vec16, s);
  if (p.d <= 64) return launch_dtc<B16, 64>(p, vec16, s);
  return launch_dtc<B16, 128>(p, vec16, s);
}

// fp32, N >= 128, d a multiple of 8 up to 16, 16-byte aligned Q/K/V rows
// (loaded as 16-byte pieces and split into bf16 planes): is the split
// tensor-core dense path available?
// fp32 episodes from 96 agents: below that the FFMA kernel is faster than
// one part-filled tile of six plane products (B=1024, d=16: N=88 29.5 vs
// 31.3 us; N=104 37.9 vs 31.5 us).
bool dense_tc_f32_supported(const AttnParams& p) {
  if (p.N < 96 || p.d > 16 || p.d % 8 != 0) return false;
  const auto a16 = [](const void* x) {
    return reinterpret_cast<uintptr_t>(x) % 16 == 0;
  };
  const Strides& t = p.st;
  return a16(p.q) && a16(p.k) && a16(p.v) && t.qn % 4 == 0 && t.kn % 4 == 0 &&
         t.vn % 4 == 0 && t.qb % 4 == 0 && t.kb % 4 == 0 && t.vb % 4 == 0;
}

cudaError_t launch_dense_tc_f32(const AttnParams& p, cudaStream_t s) {
  return launch_dtc<float, 16>(p, 1, s);
}

}  // namespace tarmac
