// abi.cu — the extern "C" entry points declared in include/tarmac_b200.h.
//
// Each entry point validates its arguments, fills an AttnParams, picks the
// kernel for the (mode, k, N, d, dtype) combination and launches it on the
// caller's stream. No memory is allocated and no stream is synchronised.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <array>
#include <mutex>
#include <unordered_map>

#include "backward.cuh"
#include "comm.cuh"
#include "common.cuh"
#include "topk_chunk.cuh"

namespace tarmac {

cudaError_t raise_smem_limit(const void* fn, size_t bytes) {
  struct Key {
    const void* fn;
    unsigned long long ctx;
    bool operator==(const Key& o) const { return fn == o.fn && ctx == o.ctx; }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.fn) ^ (size_t)(k.ctx * 0x9E3779B97F4A7C15ull);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, size_t, KeyHash> done;
  unsigned long long ctx = 0;
  // without a readable context id the attribute is set on every call
  const bool keyed = current_context_id(&ctx);
  std::lock_guard<std::mutex> lock(mu);
  if (keyed) {
    auto it = done.find(Key{fn, ctx});
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
  }
  cudaError_t e = cudaFuncSetAttribute(
      fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && keyed) done[Key{fn, ctx}] = bytes;
  return e;
}

cudaError_t launch_topk_stream_f32(const AttnParams& p, bool tie_high,
                                   cudaStream_t s);
cudaError_t launch_topk_stream_bf16(const AttnParams& p, bool tie_high,
                                    cudaStream_t s);
cudaError_t launch_topk_chunk_f32_low(const AttnParams& p, cudaStream_t s);
cudaError_t launch_topk_chunk_f32_high(const AttnParams& p, cudaStream_t s);
cudaError_t launch_topk_chunk_bf16_low(const AttnParams& p, cudaStream_t s);
cudaError_t launch_topk_chunk_bf16_high(const AttnParams& p, cudaStream_t s);

bool topk_tc_supported(const AttnParams& p);
cudaError_t launch_topk_tc(const AttnParams& p, bool tie_high, cudaStream_t s);
bool topk_tc_f32_supported(const AttnParams& p);
cudaError_t launch_topk_tc_f32(const AttnParams& p, bool tie_high,
                               cudaStream_t s);
bool topk_small_supported(const AttnParams& p);
cudaError_t launch_topk_small(const AttnParams& p, int dtype, bool tie_high,
                              cudaStream_t s);
bool topk_ws_supported(const AttnParams& p, int dtype);
cudaError_t launch_topk_ws(const AttnParams& p, int dtype, bool tie_high,
                           cudaStream_t s);

// k <= 8 with the lowest- or highest-index tie rule: episodes of 128 agents
// or more (from 65 for k <= 4, from 96 for k <= 8) form their scores on the
// tensor cores (bf16 directly; fp32 as three exact bf16 planes, d a
// multiple of 8 up to 16, 16-byte rows) — batches of at least one (bf16) or
// two (fp32) episodes per SM of 320-512 (bf16) or 352-512 (fp32) agents in
// the persistent warp-specialized kernel (topk_ws.cu) where it
// measured faster, others one 128-query block at a time (topk_tc.cu); both
// return the same bits. Other episodes up to 128 agents with d <= 16 run
// one or two lanes per query row (topk_small.cu); otherwise the chunked
// FFMA kernel when the episode's keys fit its shared memory, else the
// streaming kernel.
enum TopkPlan { TOPK_WS, TOPK_TC, TOPK_SMALL, TOPK_CHUNK, TOPK_STREAM };
static TopkPlan topk_plan(const AttnParams& p, int dtype) {
  const bool tc = dtype == TARMAC_BF16 ? topk_tc_supported(p) : topk_tc_f32_supported(p);
  if (tc && topk_ws_supported(p, dtype)) return TOPK_WS;
  if (tc) return TOPK_TC;
  // short episodes the tensor-core kernel does not take: one or two lanes
  // per query row, several episodes per block
  if (topk_small_supported(p)) return TOPK_SMALL;
  if (chunk_fits(p.N, p.d, p.topk)) return TOPK_CHUNK;
  return TOPK_STREAM;
}

static cudaError_t launch_topk_small_k(const AttnParams& p, int dtype,
                                       bool tie_high, cudaStream_t s) {
  switch (topk_plan(p, dtype)) {
    case TOPK_WS: return launch_topk_ws(p, dtype, tie_high, s);
    case TOPK_TC:
      return dtype == TARMAC_BF16 ? launch_topk_tc(p, tie_high, s)
                                  : launch_topk_tc_f32(p, tie_high, s);
    case TOPK_SMALL: return launch_topk_small(p, dtype, tie_high, s);
    case TOPK_CHUNK:
      if (dtype == TARMAC_BF16)
        return tie_high ? launch_topk_chunk_bf16_high(p, s)
                        : launch_topk_chunk_bf16_low(p, s);
      return tie_high ? launch_topk_chunk_f32_high(p, s)
                      : launch_topk_chunk_f32_low(p, s);
    default:
      return dtype == TARMAC_BF16 ? launch_topk_stream_bf16(p, tie_high, s)
                                  : launch_topk_stream_f32(p, tie_high, s);
  }
}
cudaError_t launch_topk_rows(const AttnParams& p, int dtype, cudaStream_t s);
cudaError_t launch_dense(const AttnParams& p, int dtype, cudaStream_t s);
int dense_plan(const AttnParams& p, int dtype);
cudaError_t launch_prescore(const AttnParams& p, int dtype, const void* idx,
                            bool idx_i64, int kk, cudaStream_t s);
cudaError_t launch_morton_code(const float* pos, int B, int N, int bits,
                               int64_t* out, cudaStream_t s);
cudaError_t launch_morton_select(const float* pos, int B, int N, int k,
                                 int bits, int64_t* idx_out, cudaStream_t s);
cudaError_t launch_knn_select(const float* pos, int B, int N, int k,
                              int64_t* out, cudaStream_t s);
cudaError_t launch_grid_knn_select(const float* pos, int B, int N, int k,
                                   int64_t* out, cudaStream_t s);
cudaError_t launch_random_select(int B, int N, int k, unsigned long long seed,
                                 unsigned long long offset, int64_t* out,
                                 cudaStream_t s);
size_t noalloc_scratch_floats();
cudaError_t noalloc_scratch(float** ptr);
cudaError_t launch_morton_prescore(const AttnParams& p, int dtype,
                                   const float* pos, int bits,
                                   int64_t* idx_out, cudaStream_t s);

constexpr int MAX_D = 128;
constexpr int RESIDENT_MAX_N = 1024;
constexpr int STREAM_MAX_K = 8;
constexpr int REGISTER_MAX_K = 8;
constexpr int MORTON_MAX_N = 4096;
constexpr int SELECT_MAX_N = 8192;
constexpr int SELECT_MAX_K = 32;

static bool aligned(const void* ptr, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0;
}

static int elem_size(int dtype) { return dtype == TARMAC_BF16 ? 2 : 4; }

// Validate the operand block and fill p. Returns TARMAC_OK or an error code.
static int fill_params(AttnParams& p, const void* q, const void* k,
                       const void* v, void* out, const int64_t* strides, int B,
                       int N, int d, int dtype, float scale) {
  if (!q || !k || !v || !out) return TARMAC_ERR_NULL;
  if (dtype != TARMAC_F32 && dtype != TARMAC_BF16) return TARMAC_ERR_DTYPE;
  if (B < 0 || N < 2 || d < 1 || d > MAX_D) return TARMAC_ERR_SHAPE;
  if (!(scale > 0.f) || isinf(scale)) return TARMAC_ERR_SHAPE;
  const int es = elem_size(dtype);
  if (!aligned(q, es) || !aligned(k, es) || !aligned(v, es) || !aligned(out, es))
    return TARMAC_ERR_ALIGN;
  Strides st;
  if (strides) {
    st = Strides{strides[0], strides[1], strides[2], strides[3],
                 strides[4], strides[5], strides[6], strides[7]};
  } else {
    const int64_t rs = d, bs = (int64_t)N * d;
    st = Strides{bs, rs, bs, rs, bs, rs, bs, rs};
  }
  // Vector path: 4-element groups, 16-byte (fp32) / 8-byte (bf16) aligned.
  const uintptr_t va = (uintptr_t)(4 * es);
  bool vec = (d % 4) == 0 && aligned(q, va) && aligned(k, va) &&
             aligned(v, va) && aligned(out, va);
  const int64_t sv[8] = {st.qb, st.qn, st.kb, st.kn, st.vb, st.vn, st.ob, st.on};
  for (int i = 0; i < 8; ++i) vec = vec && (sv[i] % 4) == 0;
  p.q = q; p.k = k; p.v = v; p.o = out;
  p.st = st;
  p.B = B; p.N = N; p.d = d;
  p.topk = 0;
  p.mode = TARMAC_SELECT_ARGMAX;
  // A power-of-two scale is folded into q exactly; any other scale is applied
  // to the scores after the dot product, as the reference applies it.
  int ex = 0;
  const float mant = frexpf(scale, &ex);
  const bool pow2 = scale > 0.f && mant == 0.5f && ex > -100 && ex < 100;
  p.qscale = pow2 ? scale : 1.0f;
  p.post_scale = pow2 ? 1.0f : scale;
  p.idx_out = nullptr;
  p.vec = vec ? 1 : 0;
  return TARMAC_OK;
}

// Validate the gradient operand block (q, k, v, dout and, for dense, out);
// strides holds 8 (gather) or 10 (dense) int64 element strides, or NULL.
static int fill_bwd(BwdParams& p, const void* q, const void* k, const void* v,
                    const void* out, const void* dout, const int64_t* strides,
                    int nstrides, int B, int N, int d, int dtype, float scale,
                    float* dq, float* dk, float* dv) {
  if (!q || !k || !v || !dout || !dq || !dk || !dv) return TARMAC_ERR_NULL;
  if (nstrides == 10 && !out) return TARMAC_ERR_NULL;
  if (dtype != TARMAC_F32 && dtype != TARMAC_BF16) return TARMAC_ERR_DTYPE;
  if (B < 0 || N < 2 || d < 1 || d > MAX_D) return TARMAC_ERR_SHAPE;
  if (!(scale > 0.f) || isinf(scale)) return TARMAC_ERR_SHAPE;
  const int es = elem_size(dtype);
  if (!aligned(q, es) || !aligned(k, es) || !aligned(v, es) ||
      !aligned(dout, es) || (out && !aligned(out, es)))
    return TARMAC_ERR_ALIGN;
  if (!aligned(dq, 4) || !aligned(dk, 4) || !aligned(dv, 4))
    return TARMAC_ERR_ALIGN;
  int64_t st[10];
  const int64_t rs = d, bs = (int64_t)N * d;
  for (int i = 0; i < 10; i += 2) {
    st[i] = bs;
    st[i + 1] = rs;
  }
  if (strides) {
    if (nstrides == 10) {
      for (int i = 0; i < 10; ++i) st[i] = strides[i];
    } else {  // q, k, v, dout: dout's pair goes to the last slot
      for (int i = 0; i < 6; ++i) st[i] = strides[i];
      st[8] = strides[6];
      st[9] = strides[7];
    }
  }
  const uintptr_t va = (uintptr_t)(4 * es);
  bool vec = (d % 4) == 0 && aligned(q, va) && aligned(k, va) &&
             aligned(v, va) && aligned(dout, va) && (!out || aligned(out, va));
  for (int i = 0; i < 10; ++i) vec = vec && (st[i] % 4) == 0;
  p.q = q; p.k = k; p.v = v; p.o = out; p.g = dout;
  p.qb = st[0]; p.qn = st[1]; p.kb = st[2]; p.kn = st[3];
  p.vb = st[4]; p.vn = st[5]; p.ob = st[6]; p.on = st[7];
  p.gb = st[8]; p.gn = st[9];
  p.B = B; p.N = N; p.d = d;
  p.scale = scale;
  p.dq = dq; p.dk = dk; p.dv = dv;
  p.work = nullptr;
  p.idx = nullptr;
  p.idx_i64 = 0;
  p.kk = 0;
  p.vec = vec ? 1 : 0;
  return TARMAC_OK;
}

static int launch_status(cudaError_t e) {
  return e == cudaSuccess ? TARMAC_OK : TARMAC_ERR_LAUNCH;
}

}  // namespace tarmac

using namespace tarmac;

extern "C" {

int tarmac_abi_version(void) { return TARMAC_ABI_VERSION; }

int tarmac_kernel_plan(int op, int B, int N, int d, int dtype, int topk,
                       int mode, const int64_t* strides, char* out, int len) {
  if (!out || len < 1) return TARMAC_ERR_NULL;
  out[0] = '\0';
  // planning reads shapes, strides and pointer alignment only: stand-in
  // pointers on a 256-byte grid, as torch's allocator returns
  const void* a = reinterpret_cast<const void*>((uintptr_t)1 << 20);
  AttnParams p;
  int st = fill_params(p, a, a, a, const_cast<void*>(a), strides, B, N, d, dtype, 1.0f);
  if (st != TARMAC_OK) return st;
  char buf[256];
  if (op == 0) {  // dense
    static const char* names[4] = {"dense_ws", "dense_tc", "dense_tc_f32", "dense_ffma"};
    const int pl = dense_plan(p, dtype);
    if (pl < 3)
      snprintf(buf, sizeof buf,
               "{\"kernel\": \"%s\", \"query_tile\": 128, \"key_tile\": 64}", names[pl]);
    else
      snprintf(buf, sizeof buf, "{\"kernel\": \"%s\"}", names[pl]);
  } else if (op == 1 || op == 2) {  // top-k, streaming top-k
    if (op == 2) mode = TARMAC_SELECT_ARGMAX;
    if (mode != TARMAC_SELECT_ARGMAX && mode != TARMAC_SELECT_THRESHOLD &&
        mode != TARMAC_SELECT_SORT)
      return TARMAC_ERR_MODE;
    if (topk < 1 || topk > N - 1 || (op == 2 && topk > STREAM_MAX_K)) return TARMAC_ERR_TOPK;
    p.topk = topk;
    p.mode = mode;
    const bool reg = mode != TARMAC_SELECT_THRESHOLD && topk <= REGISTER_MAX_K;
    if (!reg) {
      snprintf(buf, sizeof buf, "{\"kernel\": \"topk_rows\"}");
    } else {
      const int kc = chunk_slots(topk);
      switch (topk_plan(p, dtype)) {
        case TOPK_WS:
          snprintf(buf, sizeof buf,
                   "{\"kernel\": \"topk_ws\", \"query_tile\": 128, \"key_tile\": 128, "
                   "\"chunk\": 8, \"chunks_kept\": %d}", kc);
          break;
        case TOPK_TC:
          snprintf(buf, sizeof buf,
                   "{\"kernel\": \"topk_tc\", \"query_tile\": 128, \"key_tile\": %d, "
                   "\"chunk\": 8, \"chunks_kept\": %d}",
                   (dtype == TARMAC_F32 || d <= 16) ? 128 : 64, kc);
          break;
        case TOPK_SMALL:
          snprintf(buf, sizeof buf, "{\"kernel\": \"topk_small\", \"lanes_per_row\": %d}",
                   N <= 64 ? 2 : 1);
          break;
        case TOPK_CHUNK:
          snprintf(buf, sizeof buf, "{\"kernel\": \"topk_chunk\", \"chunks_kept\": %d}", kc);
          break;
        default:
          snprintf(buf, sizeof buf, "{\"kernel\": \"topk_stream\"}");
      }
    }
  } else {
    return TARMAC_ERR_MODE;
  }
  const int n = (int)strlen(buf);
  if (n + 1 > len) return TARMAC_ERR_SHAPE;
  memcpy(out, buf, (size_t)n + 1);
  return TARMAC_OK;
}

const char* tarmac_strerror(int status) {
  switch (status) {
    case TARMAC_OK: return "ok";
    case TARMAC_ERR_NULL: return "a required pointer is NULL";
    case TARMAC_ERR_SHAPE: return "B, N or d outside the supported range (N >= 2, 1 <= d <= 128)";
    case TARMAC_ERR_DTYPE: return "dtype must be TARMAC_F32 or TARMAC_BF16";
    case TARMAC_ERR_TOPK: return "k outside [1, N-1] or above this path's limit";
    case TARMAC_ERR_N_TOO_LARGE: return "N above this path's limit";
    case TARMAC_ERR_ALIGN: return "pointer not aligned to its element size";
    case TARMAC_ERR_MODE: return "unknown selection mode or unsupported combination";
    case TARMAC_ERR_LAUNCH: return "CUDA kernel launch failed";
    case TARMAC_ERR_BITS: return "Morton bits must lie in [1, 16]";
    case TARMAC_ERR_SCRATCH:
      return "problem larger than the library's fixed scratch (B * N <= 524288)";
    default: return "unknown status";
  }
}

int tarmac_dense_attention(const void* q, const void* k, const void* v,
                           void* out, const int64_t* strides, int B, int N,
                           int d, int dtype, float scale, void* stream) {
  AttnParams p;
  int st = fill_params(p, q, k, v, out, strides, B, N, d, dtype, scale);
  if (st != TARMAC_OK) return st;
  if (B == 0) return TARMAC_OK;
  return launch_status(launch_dense(p, dtype, (cudaStream_t)stream));
}

int tarmac_topk_attention(const void* q, const void* k, const void* v,
                          void* out, const int64_t* strides, int B, int N,
                          int d, int dtype, float scale, int topk, int mode,
                          int32_t* idx_out, void* stream) {
  AttnParams p;
  int st = fill_params(p, q, k, v, out, strides, B, N, d, dtype, scale);
  if (st != TARMAC_OK) return st;
  if (mode != TARMAC_SELECT_ARGMAX && mode != TARMAC_SELECT_THRESHOLD &&
      mode != TARMAC_SELECT_SORT)
    return TARMAC_ERR_MODE;
  if (topk < 1 || topk > N - 1) return TARMAC_ERR_TOPK;
  p.topk = topk;
  p.mode = mode;
  const bool reg = mode != TARMAC_SELECT_THRESHOLD && topk <= REGISTER_MAX_K;
  if (idx_out && !reg) return TARMAC_ERR_MODE;
  if (!reg && N > RESIDENT_MAX_N) return TARMAC_ERR_N_TOO_LARGE;
  if (idx_out && !aligned(idx_out, 4)) return TARMAC_ERR_ALIGN;
  p.idx_out = idx_out;
  if (B == 0) return TARMAC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (reg)
    return launch_status(
        launch_topk_small_k(p, dtype, mode == TARMAC_SELECT_SORT, s));
  return launch_status(launch_topk_rows(p, dtype, s));
}

int tarmac_streaming_topk_attention(const void* q, const void* k,
                                    const void* v, void* out,
                                    const int64_t* strides, int B, int N,
                                    int d, int dtype, float scale, int topk,
                                    int32_t* idx_out, void* stream) {
  AttnParams p;
  int st = fill_params(p, q, k, v, out, strides, B, N, d, dtype, scale);
  if (st != TARMAC_OK) return st;
  if (topk < 1 || topk > N - 1 || topk > STREAM_MAX_K) return TARMAC_ERR_TOPK;
  if (idx_out && !aligned(idx_out, 4)) return TARMAC_ERR_ALIGN;
  p.topk = topk;
  p.idx_out = idx_out;
  if (B == 0) return TARMAC_OK;
  return launch_status(
      launch_topk_small_k(p, dtype, false, (cudaStream_t)stream));
}

int tarmac_prescore_attention(const void* q, const void* k, const void* v,
                              void* out, const int64_t* strides,
                              const void* idx, int idx_is_i64, int kk, int B,
                              int N, int d, int dtype, float scale,
                              void* stream) {
  AttnParams p;
  int st = fill_params(p, q, k, v, out, strides, B, N, d, dtype, scale);
  if (st != TARMAC_OK) return st;
  if (!idx) return TARMAC_ERR_NULL;
  if (kk < 1) return TARMAC_ERR_TOPK;
  if (!aligned(idx, idx_is_i64 ? 8 : 4)) return TARMAC_ERR_ALIGN;
  if (B == 0) return TARMAC_OK;
  return launch_status(launch_prescore(p, dtype, idx, idx_is_i64 != 0, kk,
                                       (cudaStream_t)stream));
}

int tarmac_morton_code(const float* pos, int B, int N, int bits,
                       int64_t* code_out, void* stream) {
  if (!pos || !code_out) return TARMAC_ERR_NULL;
  if (B < 0 || N < 1) return TARMAC_ERR_SHAPE;
  if (bits < 1 || bits > 16) return TARMAC_ERR_BITS;
  if (!aligned(pos, 8) || !aligned(code_out, 8)) return TARMAC_ERR_ALIGN;
  if (B == 0) return TARMAC_OK;
  return launch_status(
      launch_morton_code(pos, B, N, bits, code_out, (cudaStream_t)stream));
}

int tarmac_morton_select(const float* pos, int B, int N, int k, int bits,
                         int64_t* idx_out, void* stream) {
  if (!pos || !idx_out) return TARMAC_ERR_NULL;
  if (B < 0 || N < 2) return TARMAC_ERR_SHAPE;
  if (N > MORTON_MAX_N) return TARMAC_ERR_N_TOO_LARGE;
  if (k < 1 || k > N - 1) return TARMAC_ERR_TOPK;
  if (bits < 1 || bits > 16) return TARMAC_ERR_BITS;
  if (!aligned(pos, 8) || !aligned(idx_out, 8)) return TARMAC_ERR_ALIGN;
  if (B == 0) return TARMAC_OK;
  return launch_status(
      launch_morton_select(pos, B, N, k, bits, idx_out, (cudaStream_t)stream));
}

int tarmac_morton_prescore_attention(const void* q, const void* k,
                                     const void* v, void* out,
                                     const int64_t* strides, const float* pos,
                                     int B, int N, int d, int dtype,
                                     float scale, int topk, int bits,
                                     int64_t* idx_out, void* stream) {
  AttnParams p;
  int st = fill_params(p, q, k, v, out, strides, B, N, d, dtype, scale);
  if (st != TARMAC_OK) return st;
  if (!pos) return TARMAC_ERR_NULL;
  if (N > MORTON_MAX_N) return TARMAC_ERR_N_TOO_LARGE;
  if (topk < 1 || topk > N - 1) return TARMAC_ERR_TOPK;
  if (bits < 1 || bits > 16) return TARMAC_ERR_BITS;
  if (!aligned(pos, 8)) return TARMAC_ERR_ALIGN;
  if (idx_out && !aligned(idx_out, 8)) return TARMAC_ERR_ALIGN;
  p.topk = topk;
  if (B == 0) return TARMAC_OK;
  return launch_status(launch_morton_prescore(p, dtype, pos, bits, idx_out,
                                              (cudaStream_t)stream));
}

int tarmac_gather_attention_backward(const void* q, const void* k,
                                     const void* v, const void* dout,
                                     const int64_t* strides, const void* idx,
                                     int idx_is_i64, int kk, int B, int N,
                                     int d, int dtype, float scale, float* dq,
                                     float* dk, float* dv, void* stream) {
  BwdParams p;
  int st = fill_bwd(p, q, k, v, nullptr, dout, strides, 8, B, N, d, dtype,
                    scale, dq, dk, dv);
  if (st != TARMAC_OK) return st;
  if (!idx) return TARMAC_ERR_NULL;
  if (kk < 1) return TARMAC_ERR_TOPK;
  if (!aligned(idx, idx_is_i64 ? 8 : 4)) return TARMAC_ERR_ALIGN;
  p.idx = idx;
  p.idx_i64 = idx_is_i64 != 0;
  p.kk = kk;
  if (B == 0) return TARMAC_OK;
  return launch_status(
      launch_gather_bwd(p, dtype == TARMAC_BF16, (cudaStream_t)stream));
}

int tarmac_dense_attention_backward(const void* q, const void* k,
                                    const void* v, const void* out,
                                    const void* dout, const int64_t* strides,
                                    int B, int N, int d, int dtype, float scale,
                                    float* dq, float* dk, float* dv,
                                    float* work, void* stream) {
  BwdParams p;
  int st = fill_bwd(p, q, k, v, out, dout, strides, 10, B, N, d, dtype, scale,
                    dq, dk, dv);
  if (st != TARMAC_OK) return st;
  if (!work) return TARMAC_ERR_NULL;
  if (!aligned(work, 4)) return TARMAC_ERR_ALIGN;
  p.work = work;
  if (B == 0) return TARMAC_OK;
  return launch_status(
      launch_dense_bwd(p, dtype == TARMAC_BF16, (cudaStream_t)stream));
}

static int check_select(const float* pos, int B, int N, int k,
                        const int64_t* idx_out) {
  if (!pos || !idx_out) return TARMAC_ERR_NULL;
  if (B < 0 || N < 2) return TARMAC_ERR_SHAPE;
  if (N > SELECT_MAX_N) return TARMAC_ERR_N_TOO_LARGE;
  if (k < 1 || k > N - 1 || k > SELECT_MAX_K) return TARMAC_ERR_TOPK;
  if (!aligned(pos, 8) || !aligned(idx_out, 8)) return TARMAC_ERR_ALIGN;
  return TARMAC_OK;
}

int tarmac_knn_select(const float* pos, int B, int N, int k, int64_t* idx_out,
                      void* stream) {
  const int st = check_select(pos, B, N, k, idx_out);
  if (st != TARMAC_OK || B == 0) return st;
  return launch_status(
      launch_knn_select(pos, B, N, k, idx_out, (cudaStream_t)stream));
}

int tarmac_grid_knn_select(const float* pos, int B, int N, int k,
                           int64_t* idx_out, void* stream) {
  const int st = check_select(pos, B, N, k, idx_out);
  if (st != TARMAC_OK || B == 0) return st;
  return launch_status(
      launch_grid_knn_select(pos, B, N, k, idx_out, (cudaStream_t)stream));
}

int tarmac_random_select(int B, int N, int k, unsigned long long seed,
                         unsigned long long offset, int64_t* idx_out,
                         void* stream) {
  if (!idx_out) return TARMAC_ERR_NULL;
  if (B < 0 || N < 2) return TARMAC_ERR_SHAPE;
  if (k < 1 || k > N - 1) return TARMAC_ERR_TOPK;
  if (!aligned(idx_out, 8)) return TARMAC_ERR_ALIGN;
  if (B == 0) return TARMAC_OK;
  return launch_status(launch_random_select(B, N, k, seed, offset, idx_out,
                                            (cudaStream_t)stream));
}

int tarmac_comm_forward(const float* x, const float* w_qkv, const float* b_qkv,
                        const float* w_proj, const float* b_proj, int B, int N,
                        int in_dim, int msg_dim, int topk, float* out,
                        void* stream) {
  if (!x || !w_qkv || !b_qkv || !w_proj || !b_proj || !out)
    return TARMAC_ERR_NULL;
  if (B < 0 || N < 2 || in_dim < 1 || in_dim > 256 || msg_dim < 1 ||
      msg_dim > 64)
    return TARMAC_ERR_SHAPE;
  if (topk < 0 || topk > N - 1 || topk > REGISTER_MAX_K) return TARMAC_ERR_TOPK;
  const void* ptrs[6] = {x, w_qkv, b_qkv, w_proj, b_proj, out};
  for (const void* ptr : ptrs)
    if (!aligned(ptr, 4)) return TARMAC_ERR_ALIGN;
  if (comm_smem_bytes(N, in_dim, msg_dim, comm_padded_m(msg_dim),
                      comm_vec(x, w_qkv, in_dim)) >
      (size_t)227 * 1024)
    return TARMAC_ERR_N_TOO_LARGE;
  if (B == 0) return TARMAC_OK;
  CommParams p;
  p.x = x; p.wqkv = w_qkv; p.bqkv = b_qkv; p.wproj = w_proj; p.bproj = b_proj;
  p.out = out;
  p.B = B; p.N = N; p.in_dim = in_dim; p.m = msg_dim;
  p.topk = topk;
  p.scale = 1.0f / sqrtf((float)msg_dim);
  p.w_smem = 0;
  return launch_status(launch_comm_forward(p, (cudaStream_t)stream));
}

// The dense-attention gradient with the row statistics in the library's
// fixed device scratch (noalloc.cu) instead of a caller workspace; allocates
// nothing.
int tarmac_dense_attention_backward_noalloc(
    const void* q, const void* k, const void* v, const void* out,
    const void* dout, const int64_t* strides, int B, int N, int d, int dtype,
    float scale, float* dq, float* dk, float* dv, void* stream) {
  BwdParams p;
  int st = fill_bwd(p, q, k, v, out, dout, strides, 10, B, N, d, dtype, scale,
                    dq, dk, dv);
  if (st != TARMAC_OK) return st;
  if ((size_t)2 * (size_t)B * (size_t)N > noalloc_scratch_floats())
    return TARMAC_ERR_SCRATCH;
  if (B == 0) return TARMAC_OK;
  float* scratch = nullptr;
  if (noalloc_scratch(&scratch) != cudaSuccess) return TARMAC_ERR_LAUNCH;
  p.work = scratch;
  return launch_status(
      launch_dense_bwd(p, dtype == TARMAC_BF16, (cudaStream_t)stream));
}

}  // extern "C"
