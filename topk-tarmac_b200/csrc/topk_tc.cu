// topk_tc.cu — fused top-k attention with the score matrix formed on the
// fifth-generation tensor cores (tcgen05, TMEM accumulators), for bf16 and
// fp32 inputs.
//
// Same function as the other fused top-k kernels (reference:
// src/kernels/fused_topk_attention.py:211-289, 405-504 and
// src/kernels/streaming_topk_attention.py:66-179): scores q.k with the
// diagonal excluded, the k best kept under the lowest- or highest-index tie
// rule, softmax over them, weighted sum of their V rows.
// * bf16 inputs: bf16 x bf16 products accumulate in fp32, the reference's
//   "bf16 with fp32 accumulation".
// * fp32 inputs: every Q and K row is split exactly into three bf16 planes
//   (hi + mid + lo, tc_common.cuh:split3_bf16x2) and six plane products
//   accumulate in fp32 per score, which reproduces the fp32 dot product to
//   within about 2^-23 * sum_c |q_c k_c| plus the fp32 accumulation
//   rounding — the size of an fp32 FFMA dot product's own rounding error,
//   and well inside the fp32 parity tolerance.
//
// One block (4 warps) owns 128 queries of one episode; thread t of warp w
// owns query row 32*w + t, which is also its tensor-memory (TMEM) lane.
// * Q (128 x d) is staged once in shared memory as bf16 in the K-major
//   core-matrix layout (tc_common.cuh); K streams through a ring of key
//   tiles, ahead of the scan: 16-byte cp.async for bf16, and for fp32 a
//   register prefetch issued before the scan of a round and split into the
//   three planes after it.
// * Per round one thread issues tcgen05.mma (M = 128, K = 16 per
//   instruction) for the round's score tile into TMEM and commits it to an
//   mbarrier: 128-key rounds in one buffer for d <= 16; otherwise 64-key
//   rounds in two buffers, round r + 1's product issued before round r is
//   scanned so the tensor core works under the scan. A block holds 128 TMEM
//   columns; up to four blocks share an SM's TMEM.
// * Pass 1 (per round): every thread reads its row's scores (tcgen05.ld, 32
//   columns at a time), forms the maximum of each chunk of CH keys and keeps
//   the KC >= k best chunks (the k best scores lie in them). A chunk that
//   enters the list has its CH scores saved to the row's shared-memory slot
//   of the chunk it evicts. Masked keys (the diagonal, the padding beyond N)
//   read as NaN, which no comparison accepts.
// * Pass 2 (after the last round): every thread rescans only its KC saved
//   chunks, in increasing key order, and keeps the exact k best under the
//   tie rule.
// * Softmax over the k retained scores; the V gather-aggregate and the
//   output store run row-cooperatively (16-byte coalesced pieces) when the
//   rows allow 16-byte access.
#include "tc_common.cuh"
#include "topk_chunk.cuh"

namespace tarmac {

constexpr int TC_THREADS = 128;
constexpr int TC_MIN_SMEM = 50 << 10; // caps residency at 4 blocks per SM
constexpr int TC_STAGE16 = 1;         // flags: 16-byte Q/K staging copies
constexpr int TC_COOP_VO = 2;         // flags: row-cooperative V/O moves

// Rounds: 128 keys in one TMEM buffer for d <= 16 (fewer rounds, so fewer
// block barriers; the other blocks on the SM run while one waits for its
// product — for fp32 this measured faster than 64-key rounds in two buffers
// despite the six plane products); 64 keys in two buffers (the next round's
// product computing under the current scan) for d > 16, where each product
// is larger. The K ring holds one tile more than the buffers. Both keep the
// block at 128 TMEM columns.
__host__ __device__ constexpr int tc_round(int DP) { return DP <= 16 ? 128 : 64; }
__host__ __device__ constexpr int tc_bufs(int DP) { return DP <= 16 ? 1 : 2; }
// bf16 planes per operand: one, or hi / mid / lo for fp32
__host__ __device__ constexpr int tc_planes(bool f32) { return f32 ? 3 : 1; }

// keys per chunk: 8 for every list size. Shorter chunks cost more list
// updates but make pass 2 and the saved-score slots smaller; with the list
// update branch-free (no warp vote), 8 measured fastest at every k and both
// dtypes (32, 16 and 4 were slower).
__host__ __device__ constexpr int tc_chunk(int, bool) { return 8; }

// A chunk-list entry packs the chunk id and the byte offset of the
// shared-memory slot holding its saved scores as (id << 8) | (slot * CH * 4);
// an empty entry has id -1, so it is negative and sorts last as an unsigned
// value. The slot offset is one mask away from the store address.

// Insert chunk maximum cm with entry ce into the descending list (mv, me) of
// KC chunks under the streaming tie rule, branch-free; a chunk that does not
// beat the last entry leaves the list unchanged.
template <int KC, bool TIE_HIGH>
__device__ __forceinline__ void chunk_insert(float (&mv)[KC], int (&me)[KC],
                                             float cm, int ce) {
#pragma unroll
  for (int p = KC - 1; p >= 1; --p) {
    const bool here = beats<TIE_HIGH>(cm, mv[p]);
    const bool above = beats<TIE_HIGH>(cm, mv[p - 1]);
    mv[p] = above ? mv[p - 1] : (here ? cm : mv[p]);
    me[p] = above ? me[p - 1] : (here ? ce : me[p]);
  }
  const bool top = beats<TIE_HIGH>(cm, mv[0]);
  mv[0] = top ? cm : mv[0];
  me[0] = top ? ce : me[0];
}

template <typename T, int DP, int KC, bool TIE_HIGH>
__global__ void __launch_bounds__(TC_THREADS, DP >= 128 ? 2 : 4)
    topk_tc_kernel(AttnParams p, int flags) {
  constexpr bool F32 = sizeof(T) == 4;
  constexpr int KCH = DP / 8;  // 16-byte chunks per bf16 row
  constexpr int RK = tc_round(DP);
  constexpr int NB = tc_bufs(DP);  // TMEM score buffers
  constexpr int TC_SLOTS = NB + 1;      // K ring depth
  constexpr int PL = tc_planes(F32);
  constexpr int QPLANE = 128 * DP * 2;  // bytes of one Q plane
  constexpr int KPLANE = RK * DP * 2;   // bytes of one K plane of a tile
  constexpr int TILE_BYTES = PL * KPLANE;
  constexpr int CH = tc_chunk(KC, F32);
  static_assert(CH == 8, "list entries pack the chunk id as (first key) << 5");
  constexpr int G = CH / 4;    // float4 groups per chunk
  constexpr int RG = KC * G;   // float4 groups per row's slots
  extern __shared__ __align__(16) unsigned char tc_smem[];
  unsigned char* sQ = tc_smem;               // PL planes of 128 x DP bf16
  unsigned char* sK = sQ + PL * QPLANE;      // TC_SLOTS x PL x RK x DP bf16
  // saved chunks: row r's KC slots at sv + r * (RG + 1); the one-float4 pad
  // puts the 8 lanes of a 128-byte wavefront on 8 distinct bank groups
  float4* sv = reinterpret_cast<float4*>(sK + TC_SLOTS * TILE_BYTES);
  __shared__ __align__(8) uint64_t mbar[2];
  __shared__ uint32_t tmem_sh;

  const int N = p.N, d = p.d;
  const int qblocks = cdiv(N, 128);
  const int b = blockIdx.x / qblocks;
  const int q0 = (blockIdx.x - b * qblocks) * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = warp * 32 + lane;  // TMEM lane
  const int i = q0 + row;            // query index
  const bool vec16 = (flags & TC_STAGE16) != 0;

  const T* Q = static_cast<const T*>(p.q) + (int64_t)b * p.st.qb;
  const T* K = static_cast<const T*>(p.k) + (int64_t)b * p.st.kb;
  const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
  T* O = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;

  const int rounds = cdiv(N, RK);
  // K rows [r0, r0 + RK) into ring slot sl (bf16: cp.async or element copies)
  auto stage_k = [&](int sl, int r0) {
    if constexpr (!F32) {
      if (vec16)
        tc::stage_fast<DP, RK, false>(tc::smem_addr(sK) + sl * TILE_BYTES,
                                      K + (int64_t)r0 * p.st.kn, p.st.kn,
                                      N - r0, d);
      else
        tc::stage_kmajor<DP>(sK + sl * TILE_BYTES, K, p.st.kn, r0, RK, N, d,
                             false);
    }
  };
  // fp32: the next K tile in registers, loaded before a round's scan and
  // split into its ring slot after it
  tc::SplitTile<DP, RK> kpre;
  if constexpr (F32) {
    const float* Qf = reinterpret_cast<const float*>(Q);
    const float* Kf = reinterpret_cast<const float*>(K);
    tc::SplitTile<DP, 128> qt;
    qt.load(Qf + (int64_t)q0 * p.st.qn, p.st.qn, N - q0, d);
    kpre.load(Kf, p.st.kn, N, d);
    qt.store(tc::smem_addr(sQ), QPLANE);
    kpre.store(tc::smem_addr(sK), KPLANE);
    if (NB == 2 && rounds > 1) {
      kpre.load(Kf + (int64_t)RK * p.st.kn, p.st.kn, N - RK, d);
      kpre.store(tc::smem_addr(sK) + TILE_BYTES, KPLANE);
    }
  } else {
    if (vec16)
      tc::stage_fast<DP, 128, false>(tc::smem_addr(sQ),
                                     Q + (int64_t)q0 * p.st.qn, p.st.qn,
                                     N - q0, d);
    else
      tc::stage_kmajor<DP>(sQ, Q, p.st.qn, q0, 128, N, d, false);
    stage_k(0, 0);
    if (NB == 2 && rounds > 1) stage_k(1, RK);
  }
  if (warp == 0) tc::tmem_alloc(&tmem_sh, NB * RK);
  if (threadIdx.x == 0) {
    tc::mbar_init(&mbar[0], 1);
    tc::mbar_init(&mbar[1], 1);
    tc::mbar_init_fence();
  }

  // chunk list; padding rows (i >= N) start full of +inf and admit nothing
  float mv[KC];
  int me[KC];
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    mv[m] = i < N ? -INFINITY : INFINITY;
    me[m] = (int)(0xffffff00u | (uint32_t)(m * CH * 4));  // empty, slot m
  }
  const uint32_t my_slots = tc::smem_addr(sv) + (uint32_t)(row * (RG + 1)) * 16u;

  const uint32_t qa = tc::smem_addr(sQ), ka = tc::smem_addr(sK);
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const float qnan = __int_as_float(0x7fc00000);
  bool ok = true;
  uint32_t tmem = 0;
  // one thread: scores of round r (K in slot r % TC_SLOTS) into TMEM buffer
  // r % NB, committed to that buffer's mbarrier
  auto issue = [&](int r) {
    const int nt = min(RK, cdiv(N - r * RK, 32) * 32);
    const uint32_t kt = ka + (uint32_t)((r % TC_SLOTS) * TILE_BYTES);
    const uint32_t idesc = tc::idesc_bf16(128, nt, false, false);
#pragma unroll
    for (int ks = 0; ks < DP / 16; ++ks) {
      if constexpr (F32) {
        // plane products, small terms first: m.m, l.h, h.l, m.h, h.m, h.h
        // (plane 0 = hi, 1 = mid, 2 = lo; A = Q, B = K)
        constexpr int PA[6] = {1, 2, 0, 1, 0, 0};
        constexpr int PB[6] = {1, 0, 2, 0, 1, 0};
#pragma unroll
        for (int t = 0; t < 6; ++t)
          tc::mma_bf16(tmem + (r % NB) * RK,
                       tc::smem_desc(qa + PA[t] * QPLANE + ks * 256, 128,
                                     KCH * 128),
                       tc::smem_desc(kt + PB[t] * KPLANE + ks * 256, 128,
                                     KCH * 128),
                       idesc, ks > 0 || t > 0);
      } else {
        tc::mma_bf16(tmem + (r % NB) * RK,
                     tc::smem_desc(qa + ks * 256, 128, KCH * 128),
                     tc::smem_desc(kt + ks * 256, 128, KCH * 128), idesc,
                     ks > 0);
      }
    }
    tc::mma_commit(&mbar[r % NB]);
  };

  for (int r = 0; r < rounds; ++r) {
    // This thread's copies of K tile r + NB - 1 (and Q at r = 0) have
    // landed; after the barrier they are visible to the tensor core, and
    // every lane has finished reading round r - 1's TMEM buffer.
    cp_async_wait_all();
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (r == 0) {
      tmem = tmem_sh;
      if (threadIdx.x == 0) issue(0);
    }
    if (threadIdx.x == 0) {
      if (NB == 2 && r + 1 < rounds) issue(r + 1);  // computes under the scan
      if (NB == 1 && r > 0) issue(r);
    }
    // slot (r + NB) % TC_SLOTS last held tile r - 1, whose product completed
    if constexpr (F32) {
      if (r + NB < rounds)
        kpre.load(reinterpret_cast<const float*>(K) +
                      (int64_t)(r + NB) * RK * p.st.kn,
                  p.st.kn, N - (r + NB) * RK, d);
    } else {
      if (r + NB < rounds) stage_k((r + NB) % TC_SLOTS, (r + NB) * RK);
    }
    ok &= tc::mbar_wait(&mbar[r % NB], (uint32_t)((r / NB) & 1));
    tc::fence_after_sync();

    const int k0 = r * RK;
    const int nt = min(RK, cdiv(N - k0, 32) * 32);
    const uint32_t tb = tmem + (r % NB) * RK + lane_off;
    for (int c = 0; c < nt / 32; ++c) {
      float v[32];
      tc::tmem_ld32(tb + c * 32, v);
      const int j0 = k0 + c * 32;
      // warp-uniform: these columns hold the warp's diagonal or the padding
      if (j0 + 32 > N || j0 == q0 + warp * 32) {
#pragma unroll
        for (int t = 0; t < 32; ++t)
          if (j0 + t >= N || j0 + t == i) v[t] = qnan;
      }
#pragma unroll
      for (int u = 0; u < 32 / CH; ++u) {
        const float cm = chunk_max<CH>(v + u * CH);
        // A chunk entering the list takes the slot of the entry it evicts.
        // Almost every chunk admits some lane of the warp, so the list
        // update runs for every chunk without a vote or a branch; only the
        // saved-score stores are conditional.
        const bool enter = beats<TIE_HIGH>(cm, mv[KC - 1]);
        const uint32_t soff = (uint32_t)me[KC - 1] & 0xffu;
        if (enter) {
          const uint32_t dst = my_slots + soff;
#pragma unroll
          for (int g = 0; g < G; ++g)
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst + 16u * g),
                         "f"(v[u * CH + 4 * g]), "f"(v[u * CH + 4 * g + 1]),
                         "f"(v[u * CH + 4 * g + 2]), "f"(v[u * CH + 4 * g + 3])
                         : "memory");
        }
        // chunk id (j0 + u CH) / CH in bits 8.., the slot offset below
        chunk_insert<KC, TIE_HIGH>(mv, me, cm,
                                   (int)(((uint32_t)(j0 + u * CH) << 5) | soff));
      }
    }
    if constexpr (F32) {
      if (r + NB < rounds)
        kpre.store(ka + (uint32_t)(((r + NB) % TC_SLOTS) * TILE_BYTES), KPLANE);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, NB * RK);

  // ---- pass 2: exact k best among the saved chunks ------------------------
  // The saved chunks, visited in increasing key order, are a stream holding
  // the k best scores of the row; the streaming insert keeps them under the
  // tie rule. Entries sort by chunk id (their high bits); empty entries
  // (negative) sort last as unsigned values and are skipped.
#pragma unroll
  for (int a = 0; a < KC; ++a)
#pragma unroll
    for (int m = 0; m + 1 < KC - a; ++m) {
      const unsigned x = (unsigned)me[m], y = (unsigned)me[m + 1];
      const bool sw = x > y;
      me[m] = sw ? (int)y : (int)x;
      me[m + 1] = sw ? (int)x : (int)y;
    }
  float bs[KC];
  int bi[KC];
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    bs[m] = -INFINITY;
    bi[m] = -1;
  }
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    if (me[m] < 0) break;
    const int jb = (me[m] >> 8) * CH;
    const uint32_t src = my_slots + ((uint32_t)me[m] & 0xffu);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float4 f;
      asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                   : "r"(src + 16u * g)
                   : "memory");
      buf_insert<KC, TIE_HIGH>(bs, bi, f.x, jb + 4 * g);
      buf_insert<KC, TIE_HIGH>(bs, bi, f.y, jb + 4 * g + 1);
      buf_insert<KC, TIE_HIGH>(bs, bi, f.z, jb + 4 * g + 2);
      buf_insert<KC, TIE_HIGH>(bs, bi, f.w, jb + 4 * g + 3);
    }
  }

  // ---- softmax over the k retained scores, V gather-aggregate, store ------
  const int kk = p.topk;
  const float sc = p.qscale * p.post_scale;
  const float mx = bs[0] * sc;
  float den = 0.f;
  float e[KC];
  bool empty = !ok;
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    e[m] = (m < kk) ? expf(bs[m] * sc - mx) : 0.f;
    den += e[m];
    empty |= (m < kk) && (bi[m] < 0);
  }
  if (i < N && p.idx_out != nullptr) {
    int32_t* io = p.idx_out + ((int64_t)b * N + i) * kk;
#pragma unroll
    for (int m = 0; m < KC; ++m)
      if (m < kk) io[m] = empty ? -1 : bi[m];
  }
  if (flags & TC_COOP_VO) {
    float w[KC];
#pragma unroll
    for (int m = 0; m < KC; ++m) w[m] = (m < kk) ? e[m] / den : 0.f;
    tc::coop_gather_store<T, DP, KC>(V, p.st.vn, O, p.st.on, q0 + warp * 32,
                                     N, d, kk, bi, w, empty);
    return;
  }
  if (i >= N) return;
  const bool vec = p.vec != 0;
  float acc[DP];
#pragma unroll
  for (int c = 0; c < DP; ++c) acc[c] = 0.f;
#pragma unroll
  for (int m = 0; m < KC; ++m) {
    if (m < kk && !empty) {
      const float w = e[m] / den;
      const T* vr = V + (int64_t)bi[m] * p.st.vn;
#pragma unroll
      for (int c = 0; c < DP; c += 4) {
        if (c < d) {
          float4 f;
          if (vec) {
            f = load4(vr + c);
          } else {
            f.x = to_f32<T>(vr[c]);
            f.y = (c + 1 < d) ? to_f32<T>(vr[c + 1]) : 0.f;
            f.z = (c + 2 < d) ? to_f32<T>(vr[c + 2]) : 0.f;
            f.w = (c + 3 < d) ? to_f32<T>(vr[c + 3]) : 0.f;
          }
          acc[c] = fmaf(w, f.x, acc[c]);
          acc[c + 1] = fmaf(w, f.y, acc[c + 1]);
          acc[c + 2] = fmaf(w, f.z, acc[c + 2]);
          acc[c + 3] = fmaf(w, f.w, acc[c + 3]);
        }
      }
    }
  }
  if (empty) {
#pragma unroll
    for (int c = 0; c < DP; ++c) acc[c] = qnan;
  }
  store_row<DP, T>(O + (int64_t)i * p.st.on, acc, d, vec);
}

template <typename T, int DP, int KC, bool TIE_HIGH>
static cudaError_t launch_tc_t(const AttnParams& p, int flags, cudaStream_t s) {
  constexpr bool F32 = sizeof(T) == 4;
  const size_t need =
      (size_t)tc_planes(F32) *
          (128 + (tc_bufs(DP) + 1) * tc_round(DP)) * DP * 2 +
      (size_t)128 * (KC * tc_chunk(KC, F32) + 4) * 4;
  const size_t sm = need > (size_t)TC_MIN_SMEM ? need : (size_t)TC_MIN_SMEM;
  cudaError_t e = raise_smem_limit(
      (const void*)topk_tc_kernel<T, DP, KC, TIE_HIGH>, (size_t)(sm));
  if (e != cudaSuccess) return e;
  const int64_t blocks = (int64_t)p.B * cdiv(p.N, 128);
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  topk_tc_kernel<T, DP, KC, TIE_HIGH>
      <<<(unsigned)blocks, TC_THREADS, sm, s>>>(p, flags);
  return cudaGetLastError();
}

template <typename T, int DP, bool TIE_HIGH>
static cudaError_t launch_tc_kc(const AttnParams& p, int flags, cudaStream_t s) {
  switch (chunk_slots(p.topk)) {
    case 1: return launch_tc_t<T, DP, 1, TIE_HIGH>(p, flags, s);
    case 2: return launch_tc_t<T, DP, 2, TIE_HIGH>(p, flags, s);
    case 4: return launch_tc_t<T, DP, 4, TIE_HIGH>(p, flags, s);
    default: return launch_tc_t<T, DP, 8, TIE_HIGH>(p, flags, s);
  }
}

static bool a16(const void* x) {
  return reinterpret_cast<uintptr_t>(x) % 16 == 0;
}

// bf16, N >= 128, k <= 8: is the tensor-core top-k path available?
// Episodes of 128 agents or more; below, from 65 agents for k <= 4 and from
// 96 for k <= 8, where one part-filled 128-row tile measured faster than
// the short-episode kernel (B=1024, d=16: N=96 k=2 15.2 vs 20.4 us fp32).
// Both bounds leave more 8-key chunks per episode (at least 9) than the
// chunk list holds.
static bool tc_episode_ok(const AttnParams& p) {
  return p.N >= 128 || (p.N >= 65 && (p.topk <= 4 || p.N >= 96));
}

bool topk_tc_supported(const AttnParams& p) {
  return tc_episode_ok(p) && p.d <= 128 && p.topk <= 8;
}

cudaError_t launch_topk_tc(const AttnParams& p, bool tie_high, cudaStream_t s) {
  using B16 = __nv_bfloat16;
  const bool d8 = p.d % 8 == 0;
  // 16-byte staging copies of Q and K; 16-byte row moves of V and O
  const bool qk = d8 && a16(p.q) && a16(p.k) && p.st.qn % 8 == 0 &&
                  p.st.kn % 8 == 0 && p.st.qb % 8 == 0 && p.st.kb % 8 == 0;
  const bool vo = d8 && a16(p.v) && a16(p.o) && p.st.vn % 8 == 0 &&
                  p.st.on % 8 == 0 && p.st.vb % 8 == 0 && p.st.ob % 8 == 0;
  const int flags = (qk ? TC_STAGE16 : 0) | (vo ? TC_COOP_VO : 0);
  const int dp = p.d <= 16 ? 16 : p.d <= 32 ? 32 : p.d <= 64 ? 64 : 128;
  switch (dp) {
    case 16: return tie_high ? launch_tc_kc<B16, 16, true>(p, flags, s) : launch_tc_kc<B16, 16, false>(p, flags, s);
    case 32: return tie_high ? launch_tc_kc<B16, 32, true>(p, flags, s) : launch_tc_kc<B16, 32, false>(p, flags, s);
    case 64: return tie_high ? launch_tc_kc<B16, 64, true>(p, flags, s) : launch_tc_kc<B16, 64, false>(p, flags, s);
    default: return tie_high ? launch_tc_kc<B16, 128, true>(p, flags, s) : launch_tc_kc<B16, 128, false>(p, flags, s);
  }
}

// fp32, N >= 128, d a multiple of 8 up to 16, k <= 8, 16-byte aligned rows
// (Q and K rows are loaded as 16-byte pieces and split into bf16 planes; V
// and O rows move as 16-byte pieces): is the split tensor-core path
// available?
bool topk_tc_f32_supported(const AttnParams& p) {
  if (!tc_episode_ok(p) || p.d > 16 || p.d % 8 != 0 || p.topk > 8) return false;
  const Strides& t = p.st;
  return a16(p.q) && a16(p.k) && a16(p.v) && a16(p.o) && t.qn % 4 == 0 &&
         t.kn % 4 == 0 && t.vn % 4 == 0 && t.on % 4 == 0 && t.qb % 4 == 0 &&
         t.kb % 4 == 0 && t.vb % 4 == 0 && t.ob % 4 == 0;
}

cudaError_t launch_topk_tc_f32(const AttnParams& p, bool tie_high,
                               cudaStream_t s) {
  const int flags = TC_STAGE16 | TC_COOP_VO;
  return tie_high ? launch_tc_kc<float, 16, true>(p, flags, s)
                  : launch_tc_kc<float, 16, false>(p, flags, s);
}

}  // namespace tarmac
