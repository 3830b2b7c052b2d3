// tc_common.cuh — fifth-generation tensor core (tcgen05) helpers for sm_100a.
//
// Operand layout: bf16 tiles in shared memory in the no-swizzle, K-major
// core-matrix layout. A core matrix is 8 rows x 16 bytes (8 bf16 along K),
// stored contiguously (128 B). For a [rows x DP] tile with KC = DP/8 16-byte
// chunks per row, element (r, k) sits at byte
//     ((r / 8) * KC + k / 8) * 128 + (r % 8) * 16 + (k % 8) * 2,
// so the descriptor's leading-dimension byte offset (next K chunk) is 128 and
// its stride-dimension byte offset (next 8 rows) is KC * 128. One MMA
// instruction consumes K = 16 (two chunks); K step s starts 2*s*128 bytes in.
//
// For an operand whose contiguous dimension is M/N (MN-major, e.g. V as the B
// operand of P.V, contiguous along d): element (k, n) sits at byte
//     ((k / 8) + (n / 8) * (KROWS / 8)) * 128 + (k % 8) * 16 + (n % 8) * 2,
// i.e. core matrices of 8 K-rows x 8 N-values; leading-dimension offset
// (next 8 K rows) 128 B, stride-dimension offset (next 8 N values)
// KROWS/8 * 128 B.
//
// Accumulators live in tensor memory (TMEM): an M=128 tile puts row m in TMEM
// lane m and column n in TMEM column base+n; warp w of the block reads lanes
// 32*(w%4) .. 32*(w%4)+31.
#pragma once

#include "common.cuh"

namespace tarmac {
namespace tc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// shared-memory matrix descriptor, no swizzle
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo,
                                              uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;                // base offset 0, absolute LBO mode, SWIZZLE_NONE
}

// instruction descriptor: bf16 x bf16 -> fp32, M x N, A/B majorness
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn,
                                                  bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A * B, issued by one thread
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc,
                                         uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate));
}

// arrive on an mbarrier when all MMAs issued so far by this thread complete
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_addr(mbar))
      : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(mbar)),
               "r"(count));
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Wait for the mbarrier phase `parity` to complete, polling at most
// `limit` times. Returns false if the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity,
                                          uint32_t limit = (1u << 24)) {
  const uint32_t a = smem_addr(mbar);
  for (uint32_t it = 0; it < limit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], "
        "%2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// TMEM allocation by one full warp; the base address is written to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_addr(dst)),
      "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile(
      "tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base),
      "r"(ncols));
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-collective).
// The load and its wait sit in one asm statement, so no use of the outputs
// can be scheduled ahead of the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
        "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// 8 consecutive fp32 columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[j]);
}

// 8 consecutive fp32 columns into this thread's TMEM lane (warp-collective);
// the store is complete (visible to later tcgen05 operations of this thread
// after a fence) when the call returns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
      "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
      : "memory");
}

// two fp32 values as a bf16 pair (round to nearest even), a in the low half
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// byte offset of row r, 16-byte chunk c in a K-major core-matrix tile with
// KC chunks per row
__device__ __forceinline__ uint32_t kmajor_off(int r, int c, int KC) {
  return (uint32_t)(((r >> 3) * KC + c) * 128 + (r & 7) * 16);
}

// Stage rows [r0, r0 + nrows) of a [*, d] bf16 matrix (row stride rs
// elements) into a K-major core-matrix tile of DP columns, zero-filling rows
// >= rlimit and columns >= d. 16-byte cp.async when `vec` (d % 8 == 0 and
// 16-byte aligned rows); element copies otherwise. All threads take part;
// the caller waits with cp_async_wait_all().
template <int DP>
__device__ __forceinline__ void stage_kmajor(unsigned char* tile,
                                             const __nv_bfloat16* src,
                                             int64_t rs, int r0, int nrows,
                                             int rlimit, int d, bool vec) {
  constexpr int KC = DP / 8;
  const uint32_t base = smem_addr(tile);
  for (int e = threadIdx.x; e < nrows * KC; e += blockDim.x) {
    const int r = e / KC, c = e - (e / KC) * KC;
    const uint32_t off = kmajor_off(r, c, KC);
    const int gr = r0 + r;
    const int c0 = c * 8;
    if (gr < rlimit && c0 < d) {
      const __nv_bfloat16* g = src + (int64_t)gr * rs + c0;
      if (vec) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(base + off),
                     "l"(g)
                     : "memory");
      } else {
        __nv_bfloat16 t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          t[u] = (c0 + u < d) ? g[u] : __float2bfloat16_rn(0.f);
        *reinterpret_cast<uint4*>(tile + off) = *reinterpret_cast<uint4*>(t);
      }
    } else {
      *reinterpret_cast<uint4*>(tile + off) = make_uint4(0, 0, 0, 0);
    }
  }
}


// Stage rows [r0, r0 + nrows) of a [*, d] bf16 matrix (row stride rs) as the
// MN-major B operand of a product that contracts over those rows: element
// (row k, column n) goes to byte ((k / 8) + (n / 8) * (nrows / 8)) * 128 +
// (k % 8) * 16 + (n % 8) * 2 (leading-dimension offset 128 B along k,
// stride-dimension offset nrows * 16 B along n). Rows >= rlimit and columns
// >= d are zero. nrows is a multiple of 8.
template <int DP>
__device__ __forceinline__ void stage_mnmajor(unsigned char* tile,
                                              const __nv_bfloat16* src,
                                              int64_t rs, int r0, int nrows,
                                              int rlimit, int d, bool vec) {
  constexpr int KC = DP / 8;
  const uint32_t base = smem_addr(tile);
  for (int e = threadIdx.x; e < nrows * KC; e += blockDim.x) {
    const int r = e / KC, c = e - (e / KC) * KC;
    const uint32_t off =
        (uint32_t)(((r >> 3) + c * (nrows >> 3)) * 128 + (r & 7) * 16);
    const int gr = r0 + r;
    const int c0 = c * 8;
    if (gr < rlimit && c0 < d) {
      const __nv_bfloat16* g = src + (int64_t)gr * rs + c0;
      if (vec) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(base + off),
                     "l"(g)
                     : "memory");
      } else {
        __nv_bfloat16 t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          t[u] = (c0 + u < d) ? g[u] : __float2bfloat16_rn(0.f);
        *reinterpret_cast<uint4*>(tile + off) = *reinterpret_cast<uint4*>(t);
      }
    } else {
      *reinterpret_cast<uint4*>(tile + off) = make_uint4(0, 0, 0, 0);
    }
  }
}


// Stage a full-width tile of R rows (rows r0_tile .. r0_tile + R - 1, of
// which the first `nvalid` exist) of a [*, d] bf16 matrix with 16-byte
// cp.async, for 128 threads, d % 8 == 0 and 16-byte aligned rows. Items are
// taken in the K-major core-matrix order (item e = 16-byte chunk at byte
// e * 16 of the K-major tile), so the 8 lanes of every shared-memory
// wavefront write 128 contiguous bytes and each warp reads whole 32-byte
// sectors of 8 or 16 rows. MN selects the MN-major destination layout of
// stage_mnmajor (same items, other placement). Missing rows and columns
// beyond d are written as zeros.
template <int DP, int R, bool MN>
__device__ __forceinline__ void stage_fast(uint32_t base,
                                           const __nv_bfloat16* src,
                                           int64_t rs, int nvalid, int d) {
  constexpr int KC = DP / 8;        // chunks per row
  constexpr int S = 128 / KC;       // rows between a thread's items
  constexpr int U = R * KC / 128;   // items per thread
  static_assert(U >= 1 && S % 8 == 0, "tile shape");
  const int tid = threadIdx.x;
  const int c = (tid >> 3) % KC;
  const int r0 = ((tid >> 3) / KC) * 8 + (tid & 7);
  const uint32_t off0 =
      MN ? (uint32_t)(((r0 >> 3) + c * (R / 8)) * 128 + (r0 & 7) * 16)
         : (uint32_t)(tid * 16);
  constexpr uint32_t dOff = MN ? (uint32_t)(S / 8) * 128 : 2048u;
  const bool col_ok = c * 8 < d;
  const __nv_bfloat16* g = src + (int64_t)r0 * rs + c * 8;
  const int64_t gstep = (int64_t)S * rs;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t dst = base + off0 + u * dOff;
    if (col_ok && r0 + u * S < nvalid) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
                   "l"(g + u * gstep)
                   : "memory");
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst),
                   "r"(0u)
                   : "memory");
    }
  }
}

// 2^x on the special-function unit (ex2.approx.ftz.f32: relative error
// about 2^-22, subnormal results flushed to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// Row-cooperative gather-aggregate-store over the 32 query rows of a warp.
// Lane t owns row row0 + t: its KC candidate indices idx (used for m < kk),
// their normalised weights w and a NaN-row flag. DP/EPV lanes share a row
// (EPV = elements per 16 bytes: 8 bf16 or 4 fp32) and each moves 16 bytes of
// every gathered V row and of the output row, so one warp instruction touches
// 32/(DP/EPV) whole rows rather than 32 scattered pieces. The owners first
// prefetch their V rows into L2; the loads then go out in batches of up to
// MAXB (16 by default) per lane before any is used — a smaller batch keeps a
// register-limited caller from spilling. Requires d % EPV == 0 and 16-byte
// aligned V and O rows. Every lane of the warp must call it (the row data
// moves by shuffles).
template <typename T, int DP, int KC, int MAXB = 16>
__device__ __forceinline__ void coop_gather_store(
    const T* V, int64_t vn, T* O, int64_t on, int row0, int N, int d, int kk,
    const int (&idx)[KC], const float (&w)[KC], bool nan_row) {
  constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte piece
  constexpr int LPR = DP / EPV;             // lanes per row
  constexpr int RPI = 32 / LPR;
  constexpr int GI = KC >= MAXB ? 1 : (MAXB / KC < LPR ? MAXB / KC : LPR);
  constexpr int LINE = 128 / (int)sizeof(T);  // elements per 128-byte line
  static_assert(LPR >= 1 && LPR <= 32, "row width");
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR, rsub = lane / LPR;
  const int c0 = sub * EPV;
  if (row0 + lane < N) {
#pragma unroll
    for (int m = 0; m < KC; ++m)
      if (m < kk && idx[m] >= 0) {
        const T* vr = V + (int64_t)idx[m] * vn;
#pragma unroll
        for (int c = 0; c < DP; c += LINE)
          if (c < d) asm volatile("prefetch.global.L2 [%0];" ::"l"(vr + c));
      }
  }
#pragma unroll
  for (int i0 = 0; i0 < LPR; i0 += GI) {
    uint4 raw[GI][KC];
    float wm[GI][KC];
    bool use[GI][KC];
#pragma unroll
    for (int g = 0; g < GI; ++g) {
      const int src = (i0 + g) * RPI + rsub;
      const bool act = row0 + src < N && c0 < d;
#pragma unroll
      for (int m = 0; m < KC; ++m) {
        const int j = __shfl_sync(0xffffffffu, idx[m], src);
        wm[g][m] = __shfl_sync(0xffffffffu, w[m], src);
        // unused slots load row 0, column 0 (always present) and discard it
        use[g][m] = m < kk && j >= 0 && act;
        raw[g][m] = __ldg(reinterpret_cast<const uint4*>(
            V + (use[g][m] ? (int64_t)j * vn + c0 : 0)));
      }
    }
#pragma unroll
    for (int g = 0; g < GI; ++g) {
      const int src = (i0 + g) * RPI + rsub;
      const int r = row0 + src;
      const bool bad = __shfl_sync(0xffffffffu, (int)nan_row, src) != 0;
      float acc[EPV];
#pragma unroll
      for (int u = 0; u < EPV; ++u) acc[u] = 0.f;
#pragma unroll
      for (int m = 0; m < KC; ++m) {
        const uint32_t h[4] = {raw[g][m].x, raw[g][m].y, raw[g][m].z,
                               raw[g][m].w};
        float f[EPV];
        if constexpr (sizeof(T) == 2) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 t = __bfloat1622float2(
                *reinterpret_cast<const __nv_bfloat162*>(&h[u]));
            f[2 * u] = t.x;
            f[2 * u + 1] = t.y;
          }
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) f[u] = __uint_as_float(h[u]);
        }
#pragma unroll
        for (int u = 0; u < EPV; ++u) {
          const float a = fmaf(wm[g][m], f[u], acc[u]);
          acc[u] = use[g][m] ? a : acc[u];
        }
      }
      if (r < N && c0 < d) {
        uint4 out;
        if constexpr (sizeof(T) == 2) {
          if (bad) {
            out = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u,
                             0x7fc07fc0u);
          } else {
            out.x = pack_bf16x2(acc[0], acc[1]);
            out.y = pack_bf16x2(acc[2], acc[3]);
            out.z = pack_bf16x2(acc[4], acc[5]);
            out.w = pack_bf16x2(acc[6], acc[7]);
          }
        } else {
          if (bad) {
            out = make_uint4(0x7fc00000u, 0x7fc00000u, 0x7fc00000u,
                             0x7fc00000u);
          } else {
            out = make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]),
                             __float_as_uint(acc[2]), __float_as_uint(acc[3]));
          }
        }
        *reinterpret_cast<uint4*>(O + (int64_t)r * on + c0) = out;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// fp32 operands on the bf16 tensor cores
// ---------------------------------------------------------------------------
// An fp32 value x is the exact sum of three bf16 values, each rounded to
// nearest: hi = bf16(x) keeps the leading 8 significant bits; x - hi is exact
// in fp32 and needs at most 16 bits, of which mid = bf16(x - hi) keeps 8; the
// rest, x - hi - mid, needs at most 8 bits and is exact in bf16 (for finite
// |x| below the largest bf16, about 3.39e38). With q = qh + qm + ql and
// k = kh + km + kl, six of the nine partial products,
//     qm.km + ql.kh + qh.kl + qm.kh + qh.km + qh.kh,
// give q.k up to the three dropped ones (qm.kl, ql.km, ql.kl), at most
// 2^-23 * sum_c |q_c k_c| in all; each bf16 x bf16 product is exact and the
// tensor core accumulates in fp32. The small terms go first.
//
// Two values a, b -> the bf16 pairs (hi, mid, lo), a in the low halves.
__device__ __forceinline__ void split3_bf16x2(float a, float b, uint32_t& hi,
                                              uint32_t& mid, uint32_t& lo) {
  hi = pack_bf16x2(a, b);
  const float ra = __fsub_rn(a, __uint_as_float(hi << 16));
  const float rb = __fsub_rn(b, __uint_as_float(hi & 0xffff0000u));
  mid = pack_bf16x2(ra, rb);
  lo = pack_bf16x2(__fsub_rn(ra, __uint_as_float(mid << 16)),
                   __fsub_rn(rb, __uint_as_float(mid & 0xffff0000u)));
}

// A tile of R fp32 rows (DP columns, zero beyond d and beyond the first
// `nvalid` rows) held in registers between a global load and a split store
// into three bf16 core-matrix planes (hi, mid, lo) of `plane` bytes each.
// 128 threads; item e = threadIdx.x + 128 u is the 8-element piece
// (row r = ((e / 8) / KCH) * 8 + e % 8, chunk c = (e / 8) % KCH). K-major
// planes (MN = false): the piece's bf16 image sits at byte 16 e, so the 8
// lanes of a shared-memory wavefront write 128 contiguous bytes and a warp
// reads 16 whole rows. MN-major planes (MN = true, the rows being the
// contraction dimension, as V in P.V): the piece sits at byte
// ((r / 8) + c * (R / 8)) * 128 + (r % 8) * 16, the MN-major layout above.
// Requires d % 8 == 0 and 16-byte aligned rows (row stride % 4 == 0).
template <int DP, int R, bool MN = false>
struct SplitTile {
  static constexpr int KCH = DP / 8;
  static constexpr int U = R * KCH / 128;
  static_assert(U >= 1 && (R * KCH) % 128 == 0, "tile shape");
  float4 x[U][2];

  __device__ __forceinline__ void load(const float* src, int64_t rs,
                                       int nvalid, int d) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = threadIdx.x + 128 * u;
      const int r = ((e >> 3) / KCH) * 8 + (e & 7);
      const int c = (e >> 3) % KCH;
      if (r < nvalid && c * 8 < d) {
        const float4* g =
            reinterpret_cast<const float4*>(src + (int64_t)r * rs + c * 8);
        x[u][0] = __ldg(g);
        x[u][1] = __ldg(g + 1);
      } else {
        x[u][0] = make_float4(0.f, 0.f, 0.f, 0.f);
        x[u][1] = x[u][0];
      }
    }
  }

  __device__ __forceinline__ void store(uint32_t base, uint32_t plane) const {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = threadIdx.x + 128 * u;
      uint32_t off = (uint32_t)e * 16u;
      if constexpr (MN) {
        const int r = ((e >> 3) / KCH) * 8 + (e & 7);
        const int c = (e >> 3) % KCH;
        off = (uint32_t)(((r >> 3) + c * (R / 8)) * 128 + (r & 7) * 16);
      }
      const uint32_t dst = base + off;
      uint32_t h[4], m[4], l[4];
      split3_bf16x2(x[u][0].x, x[u][0].y, h[0], m[0], l[0]);
      split3_bf16x2(x[u][0].z, x[u][0].w, h[1], m[1], l[1]);
      split3_bf16x2(x[u][1].x, x[u][1].y, h[2], m[2], l[2]);
      split3_bf16x2(x[u][1].z, x[u][1].w, h[3], m[3], l[3]);
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst),
                   "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
                   : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst + plane),
                   "r"(m[0]), "r"(m[1]), "r"(m[2]), "r"(m[3])
                   : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(
                       dst + 2 * plane),
                   "r"(l[0]), "r"(l[1]), "r"(l[2]), "r"(l[3])
                   : "memory");
    }
  }
};

}  // namespace tc
}  // namespace tarmac
