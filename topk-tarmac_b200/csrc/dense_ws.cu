// dense_ws.cu — dense masked-diagonal attention on the tensor cores for bf16
// inputs, warp-specialized and persistent: one block per SM loops over whole
// episodes of 320 to 512 agents.
//
// Same function and the same arithmetic as dense_tc.cu (reference:
// src/kernels/fused_dense_attention.py:38-99): per 64-key tile, S = Q K^T
// (bf16 products, fp32 accumulation in TMEM), a base-2 online softmax whose
// reference maximum moves only when a score exceeds it by more than 2^8, the
// weights rounded to bf16 and O += P V in TMEM; the tiles, the order of every
// product and the weights are those of dense_tc.cu, so both kernels return
// the same bits.
//
// Roles of the 20 warps:
// * warps 0..15 — four consumer groups; group g owns query tile g (rows
//   [128 g, 128 g + 128)) and TMEM columns [128 g, 128 g + 128): S in the
//   first 64, the output accumulator O in the next d and, for d <= 32, P
//   (bf16 pairs) in the last 32. Per tile it reads S, releases it at once
//   (the next tile's Q K^T runs under the softmax), computes the weights,
//   waits for the previous P V, rescales O when its reference moved, writes
//   P (to TMEM for d <= 32, else to its shared-memory tile) and announces it.
// * warps 16, 17 — K/V producers: each 64-key K tile (K-major) and V tile
//   (MN-major, its rows are the contraction dimension) is staged once per
//   episode into a ring (2 to 8 slots) read by all four groups; they also prefetch the
//   next episode's K and V rows into L2.
// * warp 18 — Q producer (two Q buffers: the next episode's Q is staged
//   while the current one runs).
// * warp 19 — one thread issues the products, event-driven: a group's S_j
//   as soon as the group has read S_{j-1} and K_j has landed, its P V_j as
//   soon as P_j is written, so a slow group holds up no other; the state of
//   the four groups is unrolled into registers (kept in local memory, the
//   issue loop was the bottleneck: d = 64 1297 against 748 us).
// Every wait is a bounded mbarrier poll; a wait that runs out raises a
// shared abort flag that the other roles poll, so every role ends and the
// block frees its TMEM; rows of an aborted episode are written as NaN.
#include "ws_common.cuh"

namespace tarmac {

constexpr int DWS_CONSUMERS = 512;
constexpr int DWS_KVPROD = 64;
constexpr int DWS_KVWARP0 = DWS_CONSUMERS / 32;
constexpr int DWS_QWARP = DWS_KVWARP0 + DWS_KVPROD / 32;
constexpr int DWS_MMA_WARP = DWS_QWARP + 1;
constexpr int DWS_THREADS = (DWS_MMA_WARP + 1) * 32;
constexpr int DWS_KEYS = 64;           // keys per tile
constexpr int DWS_NQ = 4;              // query tiles per episode (max)
constexpr int DWS_MAX_N = DWS_NQ * 128;
constexpr int DWS_MIN_B = 4 * 148;     // at least four episodes per SM
constexpr int DWS_SMEM_LIMIT = 227 * 1024;  // the per-block maximum (232,448 bytes)
constexpr float DWS_LOG2E = 1.4426950408889634f;
constexpr float DWS_RESCALE_LOG2 = 8.0f;

constexpr int DWS_MAX_NS = 8;         // K/V ring slots (max)

struct DwsShared {
  uint64_t kvfull[DWS_MAX_NS], kvempty[DWS_MAX_NS];
  uint64_t qfull[2][DWS_NQ], qempty[2][DWS_NQ];
  uint64_t sfull[DWS_NQ], sempty[DWS_NQ];
  uint64_t pfull[DWS_NQ], pvdone[DWS_NQ];
  uint32_t tmem;
  int abort_flag;
};

template <int DP>
struct DwsPlan {
  static constexpr int QTILE = 128 * DP * 2;
  static constexpr int KVTILE = DWS_KEYS * DP * 2;       // one K or V tile
  // d <= 32: P in tensor memory beside S and O (64 + 32 + 32 columns), the
  // A operand of P V; that takes P's stores and half of P V's operand reads
  // off the shared-memory pipe (B = 4096, N = 512, d = 32: 547 against 571 us)
  static constexpr bool PT = DP <= 32;
  static constexpr int PTILE = 128 * DWS_KEYS * 2;       // one group's P
  static constexpr int PBYTES = PT ? 0 : DWS_NQ * PTILE;
  // two Q buffers first, then as many K/V ring slots (2..8) as fit
  static constexpr int NQB = (2 * DWS_NQ * QTILE + 2 * 2 * KVTILE + PBYTES <=
                              DWS_SMEM_LIMIT) ? 2 : 1;
  static constexpr int QBYTES = NQB * DWS_NQ * QTILE;
  static constexpr int FREE = DWS_SMEM_LIMIT - QBYTES - PBYTES;
  static constexpr int NS0 = FREE / (2 * KVTILE);
  static constexpr int NS = NS0 > DWS_MAX_NS ? DWS_MAX_NS : NS0;
  static constexpr int KVBYTES = NS * 2 * KVTILE;
  static constexpr int TOTAL = QBYTES + KVBYTES + PBYTES;
};

namespace ws {
// rows [0, R) of a bf16 [*, d] matrix (row stride rs, d % 8 == 0) as the
// MN-major B operand of a product contracting over those rows: piece
// (row r, 8-column chunk c) at byte ((r / 8) + c * (R / 8)) * 128 + (r % 8) * 16.
template <int DP, int R, int NT>
__device__ __forceinline__ void copy_tile_mn_bf16(uint32_t base,
                                                  const __nv_bfloat16* src,
                                                  int64_t rs, int nvalid, int d,
                                                  int tid) {
  constexpr int KCH = DP / 8;
#pragma unroll 4
  for (int e = tid; e < R * KCH; e += NT) {
    const int r = e / KCH, c = e - (e / KCH) * KCH;
    const bool ok = r < nvalid && c * 8 < d;
    cp16(base + (uint32_t)(((r >> 3) + c * (R >> 3)) * 128 + (r & 7) * 16),
         ok ? src + (int64_t)r * rs + c * 8 : src, ok);
  }
}
// 32 consecutive 32-bit columns into this thread's TMEM lane (warp-collective);
// complete when the call returns
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
               "tcgen05.wait::st.sync.aligned;" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], issued by one thread (A K-major in TMEM:
// lane m, column k / 2, the lower k in the low half)
__device__ __forceinline__ void mma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a,
                                            uint64_t bdesc, uint32_t idesc,
                                            bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate));
}
}  // namespace ws

template <int DP>
__global__ void __launch_bounds__(DWS_THREADS, 1) dense_ws_kernel(AttnParams p) {
  using Plan = DwsPlan<DP>;
  using B16 = __nv_bfloat16;
  constexpr int NS = Plan::NS;
  constexpr int KCH = DP / 8;
  constexpr int QTILE = Plan::QTILE, KVTILE = Plan::KVTILE, PTILE = Plan::PTILE;
  constexpr int PCH = DWS_KEYS / 8;  // 16-byte chunks per P row
  extern __shared__ __align__(128) unsigned char dws_smem[];
  __shared__ DwsShared sh;
  unsigned char* sQ = dws_smem;
  unsigned char* sKV = sQ + Plan::QBYTES;  // slot s: K tile, then V tile
  unsigned char* sP = sKV + Plan::KVBYTES;
  volatile int* abort_flag = &sh.abort_flag;

  const int N = p.N, d = p.d;
  const int nqt = cdiv(N, 128), nt = cdiv(N, DWS_KEYS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nep = (int)blockIdx.x < p.B
                      ? (p.B - 1 - (int)blockIdx.x) / (int)gridDim.x + 1
                      : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(&sh.kvfull[s], DWS_KVPROD / 32);
      tc::mbar_init(&sh.kvempty[s], 1);
    }
    for (int g = 0; g < DWS_NQ; ++g) {
      for (int qb = 0; qb < 2; ++qb) {
        tc::mbar_init(&sh.qfull[qb][g], 1);
        tc::mbar_init(&sh.qempty[qb][g], 1);
      }
      tc::mbar_init(&sh.sfull[g], 1);
      tc::mbar_init(&sh.sempty[g], 4);
      tc::mbar_init(&sh.pfull[g], 4);
      tc::mbar_init(&sh.pvdone[g], 1);
    }
    sh.abort_flag = 0;
    tc::mbar_init_fence();
  }
  if (warp == DWS_MMA_WARP) tc::tmem_alloc(&sh.tmem, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sh.tmem;
  const uint32_t qa = tc::smem_addr(sQ), kva = tc::smem_addr(sKV), pa = tc::smem_addr(sP);

  if (warp >= DWS_KVWARP0 && warp < DWS_QWARP) {
    // ---------------- K / V producers ----------------
    const int tid = threadIdx.x - DWS_CONSUMERS;
    auto ep = [&](int it) { return (int)blockIdx.x + it * (int)gridDim.x; };
    auto prefetch = [&](int it) {
      const B16* kb = static_cast<const B16*>(p.k) + (int64_t)ep(it) * p.st.kb;
      const B16* vb = static_cast<const B16*>(p.v) + (int64_t)ep(it) * p.st.vb;
      for (int r = tid; r < N; r += DWS_KVPROD) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + (int64_t)r * p.st.kn));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + (int64_t)r * p.st.vn));
      }
    };
    if (nep > 0) prefetch(0);
    uint32_t kc = 0;
    bool live = true;
    for (int it = 0; it < nep && live; ++it) {
      if (it + 1 < nep) prefetch(it + 1);
      const B16* K = static_cast<const B16*>(p.k) + (int64_t)ep(it) * p.st.kb;
      const B16* V = static_cast<const B16*>(p.v) + (int64_t)ep(it) * p.st.vb;
      for (int j = 0; j < nt; ++j, ++kc) {
        const int s = kc % NS;
        if (!ws::wait(&sh.kvempty[s], ((kc / NS) & 1) ^ 1, abort_flag)) {
          live = false;
          break;
        }
        const uint32_t slot = kva + (uint32_t)(s * 2 * KVTILE);
        ws::copy_tile_bf16<DP, DWS_KEYS, DWS_KVPROD>(
            slot, K + (int64_t)(DWS_KEYS * j) * p.st.kn, p.st.kn, N - DWS_KEYS * j, d, tid);
        ws::copy_tile_mn_bf16<DP, DWS_KEYS, DWS_KVPROD>(
            slot + KVTILE, V + (int64_t)(DWS_KEYS * j) * p.st.vn, p.st.vn,
            N - DWS_KEYS * j, d, tid);
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.kvfull[s]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == DWS_QWARP) {
    // ---------------- Q producer ----------------
    bool live = true;
    for (int it = 0; it < nep && live; ++it) {
      const int qb = it % Plan::NQB;
      const uint32_t use = (uint32_t)(it / Plan::NQB);
      const B16* Q = static_cast<const B16*>(p.q) +
                     (int64_t)(blockIdx.x + it * gridDim.x) * p.st.qb;
      for (int g = 0; g < nqt; ++g) {
        if (!ws::wait(&sh.qempty[qb][g], (use & 1) ^ 1, abort_flag)) {
          live = false;
          break;
        }
        ws::copy_tile_bf16<DP, 128, 32>(qa + (uint32_t)(qb * DWS_NQ * QTILE + g * QTILE),
                                        Q + (int64_t)(128 * g) * p.st.qn, p.st.qn,
                                        N - 128 * g, d, lane);
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.qfull[qb][g]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == DWS_MMA_WARP) {
    // ---------------- MMA issuer ----------------
    // Event-driven: each group advances on its own as soon as its inputs are
    // ready (S_j once the group has read S_{j-1} and K_j has landed; P V_j
    // once its P_j is written), so a slow group holds up no other. A K/V
    // slot is released when every group's P V of its tile has been issued.
    // Descriptors are formed once and offset (addresses below 256 KB).
    if (lane == 0) {
      const uint32_t idesc_s = tc::idesc_bf16(128, DWS_KEYS, false, false);
      const uint32_t idesc_o = tc::idesc_bf16(128, DP, false, true);
      const uint64_t dq0 = tc::smem_desc(qa, 128, KCH * 128);
      const uint64_t dk0 = tc::smem_desc(kva, 128, KCH * 128);
      const uint64_t dv0 = tc::smem_desc(kva + KVTILE, 128, DWS_KEYS * 16);
      const uint64_t dp0 = tc::smem_desc(pa, 128, PCH * 128);
      uint32_t kc = 0;
      uint32_t su[DWS_NQ] = {0, 0, 0, 0}, pu[DWS_NQ] = {0, 0, 0, 0};
      int it = 0;
      for (; it < nep; ++it) {
        const int qb = it % Plan::NQB;
        const uint32_t use = (uint32_t)(it / Plan::NQB);
        for (int g = 0; g < nqt; ++g)
          if (!ws::wait(&sh.qfull[qb][g], use & 1, abort_flag)) goto mma_done;
        int ns[DWS_NQ] = {0, 0, 0, 0}, np[DWS_NQ] = {0, 0, 0, 0};
        // per ring slot (8 bits each): groups whose P V of the slot's tile
        // has been issued
        uint64_t pvcnt = 0;
        int finished = 0;
        uint32_t idle = 0;
        while (finished < nqt) {
          bool progress = false;
          // unrolled over the four groups so the per-group state stays in
          // registers
#pragma unroll
          for (int g = 0; g < DWS_NQ; ++g) {
            if (g >= nqt || np[g] == nt) continue;
            // S_{ns} (the group has read S_{ns - 1})
            if (ns[g] < nt) {
              const uint32_t kj = kc + (uint32_t)ns[g];
              const int s = kj % NS;
              if (ws::test(&sh.sempty[g], (su[g] & 1) ^ 1) &&
                  ws::test(&sh.kvfull[s], (kj / NS) & 1)) {
                tc::fence_after_sync();
                const uint64_t dq = dq0 + (uint64_t)((qb * DWS_NQ * QTILE + g * QTILE) >> 4);
                const uint64_t dk = dk0 + (uint64_t)((s * 2 * KVTILE) >> 4);
#pragma unroll
                for (int ks = 0; ks < DP / 16; ++ks)
                  tc::mma_bf16(tmem + g * 128, dq + (uint64_t)(ks * 16),
                               dk + (uint64_t)(ks * 16), idesc_s, ks > 0);
                tc::mma_commit(&sh.sfull[g]);
                ++su[g];
                ++ns[g];
                progress = true;
              }
            }
            // P V_{np}
            if (np[g] < ns[g] && ws::test(&sh.pfull[g], pu[g] & 1)) {
              ++pu[g];
              tc::fence_after_sync();
              const uint32_t kj = kc + (uint32_t)np[g];
              const int s = kj % NS;
              const uint64_t dv = dv0 + (uint64_t)((s * 2 * KVTILE) >> 4);
              if constexpr (Plan::PT) {
#pragma unroll
                for (int ks = 0; ks < DWS_KEYS / 16; ++ks)
                  ws::mma_bf16_ts(tmem + g * 128 + DWS_KEYS, tmem + g * 128 + DWS_KEYS + 32 + ks * 8,
                                  dv + (uint64_t)(ks * 16), idesc_o, np[g] > 0 || ks > 0);
              } else {
                const uint64_t dp = dp0 + (uint64_t)((g * PTILE) >> 4);
#pragma unroll
                for (int ks = 0; ks < DWS_KEYS / 16; ++ks)
                  tc::mma_bf16(tmem + g * 128 + DWS_KEYS, dp + (uint64_t)(ks * 16),
                               dv + (uint64_t)(ks * 16), idesc_o, np[g] > 0 || ks > 0);
              }
              tc::mma_commit(&sh.pvdone[g]);
              pvcnt += 1ull << (8 * s);
              if (((pvcnt >> (8 * s)) & 0xffu) == (uint64_t)nqt) {
                pvcnt &= ~(0xffull << (8 * s));
                tc::mma_commit(&sh.kvempty[s]);
              }
              if (++np[g] == nt) ++finished;
              progress = true;
            }
          }
          if (progress) {
            idle = 0;
          } else if (++idle > WS_WAIT_LIMIT || *abort_flag) {
            *abort_flag = 1;
            goto mma_done;
          }
        }
        kc += (uint32_t)nt;
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
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t t_s = tmem + g * 128, t_o = tmem + g * 128 + DWS_KEYS;
    unsigned char* prow = sP + g * PTILE + (row >> 3) * PCH * 128 + (row & 7) * 16;
    const float c2 = p.qscale * p.post_scale * DWS_LOG2E;
    uint32_t cs = 0, cpv = 0;
    bool ok = true;
    for (int it = 0; it < nep && ok; ++it) {
      if (g >= nqt) continue;
      const int b = blockIdx.x + it * gridDim.x;
      const int q0 = 128 * g, i = q0 + row;
      float mref = -1e30f;    // reference maximum in exponent units
      float mth = -INFINITY;  // raw score above which the reference moves
      float l = 0.f;
      for (int j = 0; j < nt; ++j) {
        const int k0 = j * DWS_KEYS;
        if (!ws::wait(&sh.sfull[g], cs & 1, abort_flag)) {
          ok = false;
          break;
        }
        ++cs;
        tc::fence_after_sync();
        float s[DWS_KEYS];
        {
          float h[32];
          tc::tmem_ld32(t_s + lane_off, h);
#pragma unroll
          for (int t = 0; t < 32; ++t) s[t] = h[t];
          tc::tmem_ld32(t_s + lane_off + 32, h);
#pragma unroll
          for (int t = 0; t < 32; ++t) s[32 + t] = h[t];
        }
        // S is read: the next tile's Q K^T may run under this softmax
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.sempty[g]);
        // warp-uniform: the tile holds padding or this warp's diagonal
        if (k0 + DWS_KEYS > N ||
            (k0 < q0 + wq * 32 + 32 && q0 + wq * 32 < k0 + DWS_KEYS)) {
#pragma unroll
          for (int t = 0; t < DWS_KEYS; ++t)
            if (k0 + t >= N || k0 + t == i) s[t] = -INFINITY;
        }
        float mt = s[0];
#pragma unroll
        for (int t = 1; t + 1 < DWS_KEYS; t += 2) mt = max3f(mt, s[t], s[t + 1]);
        mt = fmaxf(mt, s[DWS_KEYS - 1]);
        const bool move = mt > mth;
        float alpha = 1.0f;
        if (move) {
          const float mn = mt * c2;
          alpha = tc::ex2_approx(mref - mn);
          l *= alpha;
          mref = mn;
          mth = mt + DWS_RESCALE_LOG2 / c2;
        }
#pragma unroll
        for (int t = 0; t < DWS_KEYS; ++t) {
          s[t] = tc::ex2_approx(fmaf(s[t], c2, -mref));
          l += s[t];
        }
        // P V_{j-1} complete: P and the accumulator are free
        if (j >= 1) {
          if (!ws::wait(&sh.pvdone[g], cpv & 1, abort_flag)) {
            ok = false;
            break;
          }
          ++cpv;
          tc::fence_after_sync();
        }
        // TMEM loads and stores are warp-collective: the whole warp
        // rescales when any lane moved its reference (the others by 1)
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
        if constexpr (Plan::PT) {
          uint32_t pw[DWS_KEYS / 2];
#pragma unroll
          for (int t = 0; t < DWS_KEYS / 2; ++t) pw[t] = tc::pack_bf16x2(s[2 * t], s[2 * t + 1]);
          ws::tmem_st32(t_o + 32 + lane_off, pw);
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
          tc::fence_async_smem();
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) ws::arrive(&sh.pfull[g]);
      }
      if (!ok) break;
      // the last P V of the episode, then the output row
      if (!ws::wait(&sh.pvdone[g], cpv & 1, abort_flag)) {
        ok = false;
        break;
      }
      ++cpv;
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
      if (i < N) {
        const float inv = 1.0f / l;
        B16* O = static_cast<B16*>(p.o) + (int64_t)b * p.st.ob + (int64_t)i * p.st.on;
#pragma unroll
        for (int c = 0; c < DP / 8; ++c) {
          if (8 * c >= d) continue;
          uint4 w;
          w.x = tc::pack_bf16x2(o[8 * c] * inv, o[8 * c + 1] * inv);
          w.y = tc::pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          w.z = tc::pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          w.w = tc::pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(O + 8 * c) = w;
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == DWS_MMA_WARP) tc::tmem_dealloc(tmem, 512);
}

template <int DP>
static cudaError_t launch_dws_t(const AttnParams& p, cudaStream_t s) {
  using Plan = DwsPlan<DP>;
  static_assert(Plan::TOTAL <= DWS_SMEM_LIMIT, "shared-memory plan");
  const void* fn = (const void*)dense_ws_kernel<DP>;
  cudaError_t e = raise_smem_limit(fn, (size_t)Plan::TOTAL);
  if (e != cudaSuccess) return e;
  int dev = 0, nsm = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int grid = p.B < nsm ? p.B : nsm;
  if (grid <= 0) return cudaSuccess;
  dense_ws_kernel<DP><<<grid, DWS_THREADS, Plan::TOTAL, s>>>(p);
  return cudaGetLastError();
}

static bool dws_a16(const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; }

// bf16, batches of at least four episodes per SM, 320-512 agents (three or
// four query tiles share each staged K and V tile; N = 320, B = 4096: d = 64
// 410 against 473 us, d = 32 297 against 327; at N = 256 the two are even),
// d a multiple of 8 from 24 to 64, 16-byte aligned rows. B = 4096, N = 512: d = 64 748 against 891 us,
// d = 32 571 against 625 us; at d = 16 the per-block kernel is faster (518
// against 551 us). With fewer episodes per SM it wins only when the batch
// fills the SMs evenly (d = 64: B = 148 39.2 against 43.4 us, B = 444 94.7
// against 105.6) and ties or loses otherwise (B = 256 66.5 against 67.6,
// B = 512 120.3 against 121.3; d = 32, B = 512: 90.6 against 86.7), where the
// per-block kernel's 128-query blocks balance better.
bool dense_ws_supported(const AttnParams& p) {
  if (p.B < DWS_MIN_B || p.N < 320 || p.N > DWS_MAX_N || p.d % 8 != 0 || p.d <= 16 ||
      p.d > 64)
    return false;
  const Strides& t = p.st;
  return dws_a16(p.q) && dws_a16(p.k) && dws_a16(p.v) && dws_a16(p.o) &&
         t.qn % 8 == 0 && t.kn % 8 == 0 && t.vn % 8 == 0 && t.on % 8 == 0 &&
         t.qb % 8 == 0 && t.kb % 8 == 0 && t.vb % 8 == 0 && t.ob % 8 == 0;
}

cudaError_t launch_dense_ws(const AttnParams& p, cudaStream_t s) {
  return p.d <= 32 ? launch_dws_t<32>(p, s) : launch_dws_t<64>(p, s);
}

}  // namespace tarmac
