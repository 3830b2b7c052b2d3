// topk_ws.cu — fused top-k attention on the tensor cores, warp-specialized
// and persistent: one block per SM loops over whole episodes (N <= 512).
//
// Same function as topk_tc.cu (reference: src/kernels/fused_topk_attention.py
// :211-289, 405-504 and src/kernels/streaming_topk_attention.py:66-179):
// scores q.k with the diagonal excluded, the k best under the lowest- or
// highest-index tie rule, softmax over them, weighted sum of their V rows.
// The scores are formed exactly as there (bf16 products; fp32 as six exact
// bf16 plane products, smallest first), so both kernels return the same bits.
//
// Roles of the 20 warps:
// * warps 0..15 — four consumer warpgroups. Group g owns query rows
//   [128 g, 128 g + 128) of the current episode, TMEM lanes 0..127 of the
//   128-column TMEM quarter g. Per 128-key tile they read their scores,
//   release the quarter, and run the chunk-maximum selection of topk_tc.cu;
//   after the last tile, pass 2, the softmax and the V aggregation.
// * warps 16, 17 — K producers: each 128-key K tile of the episode is staged
//   once into a two-slot ring read by all four groups' products (fp32: copied
//   with cp.async into a raw ring and split into three bf16 planes; bf16:
//   copied straight into the K-major layout). They also stage the episode's
//   V rows into shared memory when they fit, and prefetch the next episode's
//   K and V rows into L2.
// * warp 18 — Q producer: the next episode's Q tiles go into the second of
//   two Q buffers while the current episode runs.
// * warp 19 — one thread issues the tcgen05 products (M = 128, N = 128,
//   K = 16 per instruction) and commits them to mbarriers.
// Every wait is a bounded mbarrier poll; a wait that runs out raises a
// shared abort flag that the other roles poll, so every role ends, frees
// nothing it does not own, and the block frees its TMEM; rows of an aborted
// episode are not written.
#include "topk_chunk.cuh"
#include "ws_common.cuh"

namespace tarmac {

constexpr int WS_CONSUMERS = 512;        // warps 0..15
constexpr int WS_KPROD = 64;             // warps 16, 17
constexpr int WS_QPROD = 32;             // warp 18
constexpr int WS_KWARP0 = WS_CONSUMERS / 32;
constexpr int WS_QWARP = WS_KWARP0 + WS_KPROD / 32;
constexpr int WS_MMA_WARP = WS_QWARP + 1;
constexpr int WS_THREADS = (WS_MMA_WARP + 1) * 32;
constexpr int WS_NS = 3;                 // K ring slots
constexpr int WS_RK = 128;               // keys per K tile
constexpr int WS_NQ = 4;                 // query tiles per episode (max)
constexpr int WS_MAX_N = WS_NQ * 128;
constexpr int WS_NR = 4;                 // fp32 raw slots per producer ring
constexpr int WS_RAWB = 64 * 16 * 4;     // one raw slot: 64 fp32 rows of 16
constexpr size_t WS_SMEM_LIMIT = 227 * 1024;  // the per-block maximum (232,448 bytes)

namespace ws {

// fp32 (16 columns): the pieces e = tid + NT u of a 64-row item (128 pieces
// of 8 values) into a raw slot (piece e at byte 32 e); rows >= nvalid and
// columns >= d are zero-filled.
template <int NT>
__device__ __forceinline__ void copy_raw(uint32_t raw, const float* src,
                                         int64_t rs, int nvalid, int d,
                                         int tid) {
#pragma unroll
  for (int u = 0; u < 128 / NT; ++u) {
    const int e = tid + NT * u;
    int r, c;
    piece_rc<2>(e, r, c);
    const bool ok = r < nvalid && c * 8 < d;
    const float* g = ok ? src + (int64_t)r * rs + c * 8 : src;
    cp16(raw + (uint32_t)e * 32u, g, ok);
    cp16(raw + (uint32_t)e * 32u + 16u, g + 4, ok);
  }
}

// fp32: split the pieces this thread copied into a raw slot into three bf16
// planes at base (plane stride `plane` bytes), piece e at byte 16 e.
template <int NT>
__device__ __forceinline__ void split_raw(uint32_t base, uint32_t plane,
                                          uint32_t raw, int tid) {
  constexpr int U = 128 / NT;
  float4 x[U][2];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t a = raw + (uint32_t)(tid + NT * u) * 32u;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(x[u][0].x), "=f"(x[u][0].y), "=f"(x[u][0].z), "=f"(x[u][0].w)
                 : "r"(a));
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(x[u][1].x), "=f"(x[u][1].y), "=f"(x[u][1].z), "=f"(x[u][1].w)
                 : "r"(a + 16u));
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t dst = base + (uint32_t)(tid + NT * u) * 16u;
    uint32_t h[4], m[4], l[4];
    tc::split3_bf16x2(x[u][0].x, x[u][0].y, h[0], m[0], l[0]);
    tc::split3_bf16x2(x[u][0].z, x[u][0].w, h[1], m[1], l[1]);
    tc::split3_bf16x2(x[u][1].x, x[u][1].y, h[2], m[2], l[2]);
    tc::split3_bf16x2(x[u][1].z, x[u][1].w, h[3], m[3], l[3]);
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst),
                 "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
                 : "memory");
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst + plane),
                 "r"(m[0]), "r"(m[1]), "r"(m[2]), "r"(m[3])
                 : "memory");
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst + 2 * plane),
                 "r"(l[0]), "r"(l[1]), "r"(l[2]), "r"(l[3])
                 : "memory");
  }
}

// descending chunk-list insert, branch-free (the list of topk_tc.cu)
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

}  // namespace ws

struct WsShared {
  uint64_t kfull[WS_NS], kempty[WS_NS];
  uint64_t qfull[2][WS_NQ], qempty[2][WS_NQ];
  uint64_t tfull[WS_NQ], tempty[WS_NQ];
  uint64_t vfull, vempty;
  uint32_t tmem;
  int abort_flag;
};

// Shared memory: two Q buffers (the next episode's Q is staged while the
// current one runs), a two-slot ring of 128-key K tiles, fp32 raw rings (K
// producers, Q producer), the consumers' saved chunks, and the episode's V
// rows when they fit (VST).
template <typename T, int DP, int KC, int CH>
struct WsPlan {
  static constexpr bool F32 = sizeof(T) == 4;
  static constexpr int PL = F32 ? 3 : 1;       // bf16 planes per operand
  static constexpr int KCH = DP / 8;           // 16-byte chunks per bf16 row
  static constexpr int QPLANE = 128 * DP * 2;
  static constexpr int KPLANE = WS_RK * DP * 2;
  static constexpr int QTILE = PL * QPLANE;
  static constexpr int KTILE = PL * KPLANE;
  static constexpr int KBYTES = WS_NS * KTILE;
  static constexpr int RAWBYTES = F32 ? 2 * WS_NR * WS_RAWB : 0;
  static constexpr int SVBYTES = WS_MAX_N * (KC * CH + 4) * 4;
  static constexpr int VROW = DP * (int)sizeof(T);
  // staged V rows: 16-byte piece c of row r sits at piece c ^ vswz(r) of the
  // row, so the pieces that the epilogue's 32 lanes read from 32 random rows
  // spread over all eight 16-byte bank groups (unswizzled, piece c of every
  // 64-byte row falls in one of two)
  static constexpr int VPPR = VROW / 16;                 // pieces per row
  static constexpr int VRPB = VPPR < 8 ? 8 / VPPR : 1;   // rows per 128 bytes
  __device__ static __forceinline__ int vswz(int r) { return (r / VRPB) & (VPPR - 1); }
  static constexpr int VALL = WS_MAX_N * VROW;
  static constexpr int REST = KBYTES + RAWBYTES + SVBYTES;
  static constexpr int LIM = (int)WS_SMEM_LIMIT;
  // preference: Q double buffered (the next episode's Q is ready when the
  // current one ends; with one buffer the products wait for it at every
  // episode boundary: bf16 d = 64 measured 549 against 319 us), then, for
  // bf16, V staged (the epilogue reads shared memory instead of gathering
  // from L2: d = 32 265 against 269 us). fp32 gathers from L2: its raw rings
  // and split stores already load the shared-memory pipe, which the tensor
  // core's operand reads take first (C2 k = 2 84.8 against 87.4 us).
  static constexpr int NQB = (REST + 2 * WS_NQ * QTILE <= LIM) ? 2 : 1;
  static constexpr bool VST = !F32 && REST + NQB * WS_NQ * QTILE + VALL <= LIM;
  static constexpr int QBYTES = NQB * WS_NQ * QTILE;
  static constexpr int VBYTES = VST ? VALL : 0;
  static constexpr int TOTAL = QBYTES + REST + VBYTES;
  static constexpr bool FITS = TOTAL <= LIM;
  static constexpr uint32_t KFULL = F32 ? 4 : 2;   // producer arrivals per K tile
  static constexpr uint32_t QFULL = F32 ? 2 : 1;   // per Q tile
};

template <typename T, int DP, int KC, int CH, bool TIE_HIGH>
__global__ void __launch_bounds__(WS_THREADS, 1)
    topk_ws_kernel(AttnParams p) {
  using Plan = WsPlan<T, DP, KC, CH>;
  constexpr bool F32 = Plan::F32;
  constexpr int KCH = Plan::KCH;
  constexpr int QPLANE = Plan::QPLANE, KPLANE = Plan::KPLANE;
  constexpr int QTILE = Plan::QTILE, KTILE = Plan::KTILE;
  constexpr int G = CH / 4, RG = KC * G;
  static_assert(CH == 8 || CH == 16, "8- or 16-key chunks");
  // a list entry packs (first key of the chunk) << 5 | slot byte offset;
  // the offset stays below CH * 32
  constexpr uint32_t SMASK = (uint32_t)CH * 32u - 1u;
  extern __shared__ __align__(128) unsigned char ws_smem[];
  __shared__ WsShared sh;
  unsigned char* sQ = ws_smem;
  unsigned char* sK = sQ + Plan::QBYTES;
  unsigned char* sRaw = sK + Plan::KBYTES;  // fp32: K ring, then Q ring
  T* sV = reinterpret_cast<T*>(sRaw + Plan::RAWBYTES);
  float4* sv = reinterpret_cast<float4*>(sRaw + Plan::RAWBYTES + Plan::VBYTES);
  volatile int* abort_flag = &sh.abort_flag;

  const int N = p.N, d = p.d;
  const int nqt = cdiv(N, 128), nkt = cdiv(N, WS_RK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nep = (int)blockIdx.x < p.B
                      ? (p.B - 1 - (int)blockIdx.x) / (int)gridDim.x + 1
                      : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS_NS; ++s) {
      tc::mbar_init(&sh.kfull[s], Plan::KFULL);
      tc::mbar_init(&sh.kempty[s], 1);
    }
    for (int g = 0; g < WS_NQ; ++g) {
      for (int qb = 0; qb < 2; ++qb) {
        tc::mbar_init(&sh.qfull[qb][g], Plan::QFULL);
        tc::mbar_init(&sh.qempty[qb][g], 1);
      }
      tc::mbar_init(&sh.tfull[g], 1);
      tc::mbar_init(&sh.tempty[g], 4);
    }
    tc::mbar_init(&sh.vfull, WS_KPROD);
    tc::mbar_init(&sh.vempty, 4 * nqt);
    sh.abort_flag = 0;
    tc::mbar_init_fence();
  }
  if (warp == WS_MMA_WARP) tc::tmem_alloc(&sh.tmem, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sh.tmem;
  const uint32_t qa = tc::smem_addr(sQ), ka = tc::smem_addr(sK);
  constexpr int L = WS_NR - 1;  // fp32 raw-ring lookahead (items)

  if (warp >= WS_KWARP0 && warp < WS_QWARP) {
    // ---------------- K / V producers ----------------
    const int tid = threadIdx.x - WS_CONSUMERS;
    const T* Kall = static_cast<const T*>(p.k);
    auto kptr = [&](int it, int r0) {
      return Kall + (int64_t)(blockIdx.x + it * gridDim.x) * p.st.kb +
             (int64_t)r0 * p.st.kn;
    };
    auto prefetch = [&](int it) {
      const T* kb = kptr(it, 0);
      const T* vb = static_cast<const T*>(p.v) +
                    (int64_t)(blockIdx.x + it * gridDim.x) * p.st.vb;
      for (int r = tid; r < N; r += WS_KPROD) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + (int64_t)r * p.st.kn));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + (int64_t)r * p.st.vn));
      }
    };
    // the episode's V rows into sV, tracked by vfull (one arrival per thread
    // once all of its copies have landed)
    auto stage_v = [&](int it) -> bool {
      if (!ws::wait(&sh.vempty, (uint32_t)((it & 1) ^ 1), abort_flag)) return false;
      const T* V = static_cast<const T*>(p.v) +
                   (int64_t)(blockIdx.x + it * gridDim.x) * p.st.vb;
      constexpr int PPR = DP * (int)sizeof(T) / 16;  // 16-byte pieces per row
      constexpr int EPP = 16 / (int)sizeof(T);       // elements per piece
      const uint32_t va = tc::smem_addr(sV);
      for (int e = tid; e < N * PPR; e += WS_KPROD) {
        const int r = e / PPR, c = e - (e / PPR) * PPR;
        const bool ok = c * EPP < d;
        ws::cp16(va + (uint32_t)(r * PPR + (c ^ Plan::vswz(r))) * 16u,
                 ok ? V + (int64_t)r * p.st.vn + c * EPP : V, ok);
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(
                       tc::smem_addr(&sh.vfull))
                   : "memory");
      return true;
    };
    if (nep > 0) prefetch(0);
    if constexpr (F32) {
      // 2 nkt 64-row half tiles per episode through the raw ring, L items
      // ahead; each thread splits the pieces it copied itself
      const uint32_t raw0 = tc::smem_addr(sRaw);
      const int ipe = 2 * nkt, total = nep * ipe;
      auto issue = [&](int n) {
        if (n < total) {
          const int it = n / ipe, w = n - (n / ipe) * ipe;
          ws::copy_raw<WS_KPROD>(raw0 + (uint32_t)((n % WS_NR) * WS_RAWB),
                                 reinterpret_cast<const float*>(kptr(it, 64 * w)),
                                 p.st.kn, N - 64 * w, d, tid);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
      for (int n = 0; n < L; ++n) issue(n);
      for (int n = 0; n < total; ++n) {
        issue(n + L);
        asm volatile("cp.async.wait_group %0;" ::"n"(L) : "memory");
        const int it = n / ipe, w = n - (n / ipe) * ipe;
        if (w == 0 && it + 1 < nep) prefetch(it + 1);
        const uint32_t kc = (uint32_t)(it * nkt + (w >> 1));
        const int s = kc % WS_NS;
        if ((w & 1) == 0 &&
            !ws::wait(&sh.kempty[s], ((kc / WS_NS) & 1) ^ 1, abort_flag)) break;
        ws::split_raw<WS_KPROD>(ka + (uint32_t)(s * KTILE + (w & 1) * 2048), KPLANE,
                                raw0 + (uint32_t)((n % WS_NR) * WS_RAWB), tid);
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.kfull[s]);
        if (Plan::VST && w == ipe - 1 && !stage_v(it)) break;
      }
    } else {
      // K tiles straight into the ring, one tile in flight ahead: tile n's
      // copies are issued before the producers wait for tile n - 1's to land
      // and announce it (the rows were prefetched into L2 an episode earlier)
      const int total = nep * nkt;
      for (int n = 0; n <= total; ++n) {
        if (n < total) {
          const int it = n / nkt, j = n - it * nkt;
          if (j == 0 && it + 1 < nep) prefetch(it + 1);
          const int s = n % WS_NS;
          if (!ws::wait(&sh.kempty[s], ((n / WS_NS) & 1) ^ 1, abort_flag)) break;
          ws::copy_tile_bf16<DP, WS_RK, WS_KPROD>(
              ka + (uint32_t)(s * KTILE),
              reinterpret_cast<const __nv_bfloat16*>(kptr(it, WS_RK * j)), p.st.kn,
              N - WS_RK * j, d, tid);
          asm volatile("cp.async.commit_group;" ::: "memory");
          asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
          asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        if (n > 0) {
          const int pn = n - 1, pit = pn / nkt;
          tc::fence_async_smem();
          __syncwarp();
          if (lane == 0) ws::arrive(&sh.kfull[pn % WS_NS]);
          if (Plan::VST && pn - pit * nkt == nkt - 1 && !stage_v(pit)) break;
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == WS_QWARP) {
    // ---------------- Q producer ----------------
    // Episode it's Q tiles go into buffer it & 1 once the products of
    // episode it - 2 that read it are done.
    const T* Qall = static_cast<const T*>(p.q);
    auto qptr = [&](int it, int r0) {
      return Qall + (int64_t)(blockIdx.x + it * gridDim.x) * p.st.qb +
             (int64_t)r0 * p.st.qn;
    };
    if constexpr (F32) {
      const uint32_t raw0 = tc::smem_addr(sRaw) + (uint32_t)(WS_NR * WS_RAWB);
      const int ipe = 2 * nqt, total = nep * ipe;
      auto issue = [&](int n) {
        if (n < total) {
          const int it = n / ipe, w = n - (n / ipe) * ipe;
          ws::copy_raw<WS_QPROD>(raw0 + (uint32_t)((n % WS_NR) * WS_RAWB),
                                 reinterpret_cast<const float*>(qptr(it, 64 * w)),
                                 p.st.qn, N - 64 * w, d, lane);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
      for (int n = 0; n < L; ++n) issue(n);
      for (int n = 0; n < total; ++n) {
        issue(n + L);
        asm volatile("cp.async.wait_group %0;" ::"n"(L) : "memory");
        const int it = n / ipe, w = n - (n / ipe) * ipe;
        const int g = w >> 1, qb = it % Plan::NQB;
        const uint32_t use = (uint32_t)(it / Plan::NQB);
        if ((w & 1) == 0 && !ws::wait(&sh.qempty[qb][g], (use & 1) ^ 1, abort_flag)) break;
        ws::split_raw<WS_QPROD>(
            qa + (uint32_t)(qb * WS_NQ * QTILE + g * QTILE + (w & 1) * 2048), QPLANE,
            raw0 + (uint32_t)((n % WS_NR) * WS_RAWB), lane);
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.qfull[qb][g]);
      }
    } else {
      bool live = true;
      for (int it = 0; it < nep && live; ++it) {
        const int qb = it % Plan::NQB;
        const uint32_t use = (uint32_t)(it / Plan::NQB);
        for (int g = 0; g < nqt; ++g) {
          if (!ws::wait(&sh.qempty[qb][g], (use & 1) ^ 1, abort_flag)) {
            live = false;
            break;
          }
          ws::copy_tile_bf16<DP, 128, WS_QPROD>(
              qa + (uint32_t)(qb * WS_NQ * QTILE + g * QTILE),
              reinterpret_cast<const __nv_bfloat16*>(qptr(it, 128 * g)), p.st.qn,
              N - 128 * g, d, lane);
          asm volatile("cp.async.commit_group;" ::: "memory");
          asm volatile("cp.async.wait_group 0;" ::: "memory");
          tc::fence_async_smem();
          __syncwarp();
          if (lane == 0) ws::arrive(&sh.qfull[qb][g]);
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == WS_MMA_WARP) {
    // ---------------- MMA issuer ----------------
    // Event-driven: each group's product for tile j is issued as soon as the
    // group has read tile j - 1 and K_j has landed, so a slow group holds up
    // no other; a K slot is released once every group's product of its tile
    // has been issued. The per-group state is unrolled into registers.
    // Descriptors are formed once; plane, K-step and tile offsets are added
    // to the 14-bit address field (addresses stay below 256 KB: no carry).
    if (lane == 0) {
      uint32_t kcount = 0;
      const uint32_t idesc = tc::idesc_bf16(128, WS_RK, false, false);
      const uint64_t dq0 = tc::smem_desc(qa, 128, KCH * 128);
      const uint64_t dk0 = tc::smem_desc(ka, 128, KCH * 128);
      int it = 0;
      for (; it < nep; ++it) {
        const int qb = it % Plan::NQB;
        const uint32_t use = (uint32_t)(it / Plan::NQB);
        for (int g = 0; g < nqt; ++g)
          if (!ws::wait(&sh.qfull[qb][g], use & 1, abort_flag)) goto mma_done;
        int nx[WS_NQ] = {0, 0, 0, 0};   // next tile of each group
        uint32_t issued = 0;            // per slot (8 bits): groups issued
        int finished = 0;
        uint32_t idle = 0;
        while (finished < nqt) {
          bool progress = false;
#pragma unroll
          for (int g = 0; g < WS_NQ; ++g) {
            if (g >= nqt || nx[g] == nkt) continue;
            // the TMEM quarter's uses so far: one per tile of earlier episodes
            const uint32_t tu = (uint32_t)(kcount + nx[g]);
            const uint32_t kj = kcount + (uint32_t)nx[g];
            const int s = kj % WS_NS;
            if (!ws::test(&sh.tempty[g], (tu & 1) ^ 1) ||
                !ws::test(&sh.kfull[s], (kj / WS_NS) & 1))
              continue;
            tc::fence_after_sync();
            const uint64_t dk = dk0 + (uint64_t)((s * KTILE) >> 4);
            const uint64_t dq = dq0 + (uint64_t)((qb * WS_NQ * QTILE + g * QTILE) >> 4);
            const uint32_t td = tmem + g * 128;
#pragma unroll
            for (int ks = 0; ks < DP / 16; ++ks) {
              const uint64_t a = dq + (uint64_t)(ks * 16), b = dk + (uint64_t)(ks * 16);
              if constexpr (F32) {
                // plane products, small terms first: m.m, l.h, h.l, m.h, h.m, h.h
                tc::mma_bf16(td, a + (QPLANE >> 4), b + (KPLANE >> 4), idesc, ks > 0);
                tc::mma_bf16(td, a + (2 * QPLANE >> 4), b, idesc, true);
                tc::mma_bf16(td, a, b + (2 * KPLANE >> 4), idesc, true);
                tc::mma_bf16(td, a + (QPLANE >> 4), b, idesc, true);
                tc::mma_bf16(td, a, b + (KPLANE >> 4), idesc, true);
                tc::mma_bf16(td, a, b, idesc, true);
              } else {
                tc::mma_bf16(td, a, b, idesc, ks > 0);
              }
            }
            tc::mma_commit(&sh.tfull[g]);
            issued += 1u << (8 * s);
            if (((issued >> (8 * s)) & 0xffu) == (uint32_t)nqt) {
              issued &= ~(0xffu << (8 * s));
              tc::mma_commit(&sh.kempty[s]);
            }
            if (++nx[g] == nkt) ++finished;
            progress = true;
          }
          if (progress) {
            idle = 0;
          } else if (++idle > WS_WAIT_LIMIT || *abort_flag) {
            *abort_flag = 1;
            goto mma_done;
          }
        }
        kcount += (uint32_t)nkt;
        for (int g = 0; g < nqt; ++g) tc::mma_commit(&sh.qempty[qb][g]);
      }
      // drain: the last episode's products and commits have landed before
      // the block may exit
      if (it > 0) {
        const int qb = (it - 1) % Plan::NQB;
        const uint32_t use = (uint32_t)((it - 1) / Plan::NQB);
        for (int g = 0; g < nqt; ++g)
          if (!ws::wait(&sh.qempty[qb][g], use & 1, abort_flag)) break;
      }
    mma_done:;
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int g = warp >> 2, wq = warp & 3;
    const int row = wq * 32 + lane;  // TMEM lane
    // this row's KC saved-chunk slots (CH scores each) in shared memory; a
    // list entry carries its slot's byte offset (slot * CH * 4) in the low
    // bits, so one mask gives the store address
    const uint32_t my_slots =
        tc::smem_addr(sv) + (uint32_t)((g * 128 + row) * (RG + 1)) * 16u;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const float qnan = __int_as_float(0x7fc00000);
    const float sc = p.qscale * p.post_scale;
    const int kk = p.topk;
    uint32_t cu = 0;
    bool ok = true;
    for (int it = 0; it < nep && ok; ++it) {
      if (g >= nqt) continue;
      const int b = blockIdx.x + it * gridDim.x;
      const int q0 = 128 * g, i = q0 + row;
      // chunk list; padding rows (i >= N) start full of +inf and admit nothing
      float mv[KC];
      int me[KC];
#pragma unroll
      for (int m = 0; m < KC; ++m) {
        mv[m] = i < N ? -INFINITY : INFINITY;
        me[m] = (int)(~SMASK | (uint32_t)(m * CH * 4));  // empty, slot m
      }
      for (int j = 0; j < nkt; ++j) {
        if (!ws::wait(&sh.tfull[g], cu & 1, abort_flag)) {
          ok = false;
          break;
        }
        ++cu;
        tc::fence_after_sync();
        const uint32_t tb = tmem + g * 128 + lane_off;
#pragma unroll 1
        for (int c = 0; c < WS_RK / 32; ++c) {
          float v[32];
          tc::tmem_ld32(tb + c * 32, v);
          if (c == WS_RK / 32 - 1) {
            // the tile is read: release the TMEM quarter to the next product
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) ws::arrive(&sh.tempty[g]);
          }
          const int j0 = WS_RK * j + 32 * c;
          // warp-uniform: these columns hold the warp's diagonal or padding
          if (j0 + 32 > N || j0 == q0 + wq * 32) {
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (j0 + t >= N || j0 + t == i) v[t] = qnan;
          }
#pragma unroll
          for (int u = 0; u < 32 / CH; ++u) {
            const float cm = chunk_max<CH>(v + u * CH);
            // a chunk entering the list takes the slot of the entry it evicts
            const bool enter = beats<TIE_HIGH>(cm, mv[KC - 1]);
            const uint32_t soff = (uint32_t)me[KC - 1] & SMASK;
            if (enter) {
              const uint32_t dst = my_slots + soff;
#pragma unroll
              for (int gg = 0; gg < G; ++gg)
                asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(
                                 dst + 16u * gg),
                             "f"(v[u * CH + 4 * gg]), "f"(v[u * CH + 4 * gg + 1]),
                             "f"(v[u * CH + 4 * gg + 2]), "f"(v[u * CH + 4 * gg + 3])
                             : "memory");
            }
            // the chunk's first key in bits 5.., the slot offset below
            ws::chunk_insert<KC, TIE_HIGH>(
                mv, me, cm, (int)(((uint32_t)(j0 + u * CH) << 5) | soff));
          }
        }
      }
      if (!ok) break;
      // ---- pass 2: exact k best among the saved chunks, in key order ----
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
        const int jb = (me[m] >> 5) & ~(CH - 1);
        const uint32_t src = my_slots + ((uint32_t)me[m] & SMASK);
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
          float4 f;
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                       : "r"(src + 16u * gg)
                       : "memory");
          buf_insert<KC, TIE_HIGH>(bs, bi, f.x, jb + 4 * gg);
          buf_insert<KC, TIE_HIGH>(bs, bi, f.y, jb + 4 * gg + 1);
          buf_insert<KC, TIE_HIGH>(bs, bi, f.z, jb + 4 * gg + 2);
          buf_insert<KC, TIE_HIGH>(bs, bi, f.w, jb + 4 * gg + 3);
        }
      }
      // ---- softmax over the k retained scores ----
      const float mx = bs[0] * sc;
      float den = 0.f;
      float e[KC];
      bool empty = false;
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
      T* Ob = static_cast<T*>(p.o) + (int64_t)b * p.st.ob;
      if constexpr (Plan::VST) {
        // the episode's V rows sit in sV (staged by the K producers)
        if (!ws::wait(&sh.vfull, (uint32_t)(it & 1), abort_flag)) {
          ok = false;
          break;
        }
        constexpr int EPV = 16 / (int)sizeof(T);
        float wm[KC];
#pragma unroll
        for (int m = 0; m < KC; ++m) wm[m] = (m < kk && !empty) ? e[m] / den : 0.f;
        T* O = Ob + (int64_t)i * p.st.on;
        // one 16-byte piece of the output row at a time: EPV accumulators
#pragma unroll
        for (int c = 0; c < DP / EPV; ++c) {
          float acc[EPV];
#pragma unroll
          for (int u = 0; u < EPV; ++u) acc[u] = 0.f;
#pragma unroll
          for (int m = 0; m < KC; ++m) {
            if (m < kk && !empty) {
              const uint4 raw =
                  reinterpret_cast<const uint4*>(sV + bi[m] * DP)[c ^ Plan::vswz(bi[m])];
              const uint32_t h[4] = {raw.x, raw.y, raw.z, raw.w};
              float f[EPV];
              if constexpr (F32) {
#pragma unroll
                for (int u = 0; u < 4; ++u) f[u] = __uint_as_float(h[u]);
              } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const float2 t2 = __bfloat1622float2(
                      *reinterpret_cast<const __nv_bfloat162*>(&h[u]));
                  f[2 * u] = t2.x;
                  f[2 * u + 1] = t2.y;
                }
              }
#pragma unroll
              for (int u = 0; u < EPV; ++u) acc[u] = fmaf(wm[m], f[u], acc[u]);
            }
          }
          if (i < N && c * EPV < d) {
            uint4 out;
            if constexpr (F32) {
              out = empty ? make_uint4(0x7fc00000u, 0x7fc00000u, 0x7fc00000u, 0x7fc00000u)
                          : make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]),
                                       __float_as_uint(acc[2]), __float_as_uint(acc[3]));
            } else {
              out = empty ? make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u)
                          : make_uint4(tc::pack_bf16x2(acc[0], acc[1]),
                                       tc::pack_bf16x2(acc[2], acc[3]),
                                       tc::pack_bf16x2(acc[4], acc[5]),
                                       tc::pack_bf16x2(acc[6], acc[7]));
            }
            *reinterpret_cast<uint4*>(O + c * EPV) = out;
          }
        }
        // sV is read: release it to the next episode's staging
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.vempty);
      } else {
        float w[KC];
#pragma unroll
        for (int m = 0; m < KC; ++m) w[m] = (m < kk) ? e[m] / den : 0.f;
        const T* V = static_cast<const T*>(p.v) + (int64_t)b * p.st.vb;
        // at most 8 loads in flight per lane: this kernel has 96 registers
        tc::coop_gather_store<T, DP, KC, 8>(V, p.st.vn, Ob, p.st.on, q0 + wq * 32, N,
                                            d, kk, bi, w, empty);
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == WS_MMA_WARP) tc::tmem_dealloc(tmem, 512);
}

template <typename T, int DP, int KC, bool TIE_HIGH>
static cudaError_t launch_ws_t(const AttnParams& p, cudaStream_t s) {
#ifdef WS_FORCE_CH
  constexpr int CH = WS_FORCE_CH;
#else
  constexpr int CH = 8;
#endif
  using Plan = WsPlan<T, DP, KC, CH>;
  if constexpr (!Plan::FITS) {
    return cudaErrorInvalidConfiguration;
  } else {
    const void* fn = (const void*)topk_ws_kernel<T, DP, KC, CH, TIE_HIGH>;
    cudaError_t e = raise_smem_limit(fn, (size_t)Plan::TOTAL);
    if (e != cudaSuccess) return e;
    int dev = 0, nsm = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const int grid = p.B < nsm ? p.B : nsm;
    if (grid <= 0) return cudaSuccess;
    topk_ws_kernel<T, DP, KC, CH, TIE_HIGH><<<grid, WS_THREADS, Plan::TOTAL, s>>>(p);
    return cudaGetLastError();
  }
}

template <typename T, int DP, bool TIE_HIGH>
static cudaError_t launch_ws_kc(const AttnParams& p, cudaStream_t s) {
  switch (chunk_slots(p.topk)) {
    case 1: return launch_ws_t<T, DP, 1, TIE_HIGH>(p, s);
    case 2: return launch_ws_t<T, DP, 2, TIE_HIGH>(p, s);
    default: return launch_ws_t<T, DP, 4, TIE_HIGH>(p, s);
  }
}

static bool ws_a16(const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; }

// The persistent kernel serves episodes of up to 512 agents whose three or
// four query tiles share each staged K tile: from 320 agents for bf16 and
// 352 for fp32 (N = 384, B = 4096, k = 2: fp32 210 against 234 us, bf16 d = 32
// 187 against 242; at N = 272 the per-block kernel is ahead, at N = 320 to
// 352 they meet). Measured against the per-block kernel on the same
// episodes (N = 512, the same bits):
// * fp32: d a multiple of 8 up to 16, k <= 2, batches of at least two
//   episodes per SM (k = 2: B = 256 31.0 against 31.1 us, B = 296 31.1
//   against 34.7, B = 1024 84 against 98.5; k = 1 at B = 256 27.5 against
//   28.9 for the per-block kernel; at k = 4 the per-block kernel is faster);
// * bf16: d a multiple of 8 from 24 to 64, k <= 4 where the shared-memory
//   plan fits, batches of at least one episode per SM (k = 2, B = 148: d = 32
//   17.2 against 20.8 us, d = 64 24.9 against 26.9; B = 4096: 265 against
//   373 and 364 against 518); at d <= 16 the per-block kernel is as fast.
constexpr int WS_MIN_B_F32 = 2 * 148;
constexpr int WS_MIN_B_BF16 = 148;
bool topk_ws_supported(const AttnParams& p, int dtype) {
  const int min_b = dtype == TARMAC_BF16 ? WS_MIN_B_BF16 : WS_MIN_B_F32;
  const int min_n = dtype == TARMAC_BF16 ? 320 : 352;
  if (p.B < min_b || p.N < min_n || p.N > WS_MAX_N || p.topk < 1 || p.d % 8 != 0)
    return false;
  const Strides& t = p.st;
  const int64_t al = dtype == TARMAC_BF16 ? 8 : 4;  // elements per 16 bytes
  if (!(ws_a16(p.q) && ws_a16(p.k) && ws_a16(p.v) && ws_a16(p.o))) return false;
  if (t.qn % al || t.kn % al || t.vn % al || t.on % al || t.qb % al ||
      t.kb % al || t.vb % al || t.ob % al)
    return false;
  if (dtype == TARMAC_F32) return p.d <= 16 && p.topk <= 2;
  if (p.d <= 16 || p.d > 64 || p.topk > 4) return false;
  if (p.d > 32 && p.topk > 2) return false;  // DP = 64, KC = 4 does not fit
  return true;
}

cudaError_t launch_topk_ws(const AttnParams& p, int dtype, bool tie_high,
                           cudaStream_t s) {
  using B16 = __nv_bfloat16;
  if (dtype == TARMAC_F32)
    return tie_high ? launch_ws_kc<float, 16, true>(p, s)
                    : launch_ws_kc<float, 16, false>(p, s);
  const int dp = p.d <= 16 ? 16 : p.d <= 32 ? 32 : 64;
  switch (dp) {
    case 16: return tie_high ? launch_ws_kc<B16, 16, true>(p, s) : launch_ws_kc<B16, 16, false>(p, s);
    case 32: return tie_high ? launch_ws_kc<B16, 32, true>(p, s) : launch_ws_kc<B16, 32, false>(p, s);
    default: return tie_high ? launch_ws_kc<B16, 64, true>(p, s) : launch_ws_kc<B16, 64, false>(p, s);
  }
}

}  // namespace tarmac
