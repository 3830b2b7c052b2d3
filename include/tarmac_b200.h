/*
 * tarmac_b200.h — C ABI of the B200 (sm_100a) TarMAC attention core.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * handle (passed as void*, it is a cudaStream_t; NULL means the legacy default
 * stream). Nothing is allocated inside the library: the caller owns every
 * buffer. Every call is asynchronous on the given stream and returns a status
 * code (TARMAC_OK or one of the TARMAC_ERR_* values below) describing argument
 * validation and the launch; tarmac_strerror() turns a code into text.
 *
 * Tensor layout. Q, K, V and the output O are [B, N, d] arrays of the dtype
 * named by `dtype` (TARMAC_F32 or TARMAC_BF16) whose innermost (d) stride is
 * 1. `strides` points at eight int64 element strides
 *     { q_b, q_n, k_b, k_n, v_b, v_n, o_b, o_n }
 * (batch stride, then row stride, for Q, K, V, O), or is NULL for contiguous
 * [B, N, d] arrays. Base pointers and every stride times the element size must
 * be multiples of 16 bytes when d * element size is a multiple of 16 bytes
 * (TARMAC_ERR_ALIGN otherwise); other d use a scalar path with no alignment
 * rule.
 *
 * Semantics shared by every attention entry point (restated from the
 * reference's eager path, src/kernels/fused_topk_attention.py:390-402):
 *   s[b,i,j] = (q[b,i,:] . k[b,j,:]) * scale, the diagonal j == i excluded;
 *   softmax over the retained peers of row i; out[b,i,:] = sum_j w_ij v[b,j,:].
 * Scores and accumulation are fp32. bf16 inputs with N >= 128 (top-k: from
 * N = 65 for k <= 4 and N = 96 for k <= 8; dense: from N = 65) form their
 * scores on the tensor cores (exact bf16 products, fp32 accumulation; the
 * dense path feeds its softmax weights to P.V as bf16, as the reference's
 * bf16 kernel does); other bf16 inputs are widened to fp32 on load. fp32
 * top-k (k <= 8) inputs of those sizes and dense inputs from N = 96, with d
 * a multiple of 8 up to 16 and 16-byte aligned rows, also run on the tensor
 * cores: every operand (q,
 * k, v and the dense path's softmax weights) is split exactly into three
 * bf16 parts and six part products accumulate in fp32, an fp32-accurate
 * product (error within about 2^-23 * sum_c |a_c b_c| plus fp32
 * accumulation rounding). Other fp32 work uses IEEE fp32 FMA.
 *
 * Row-count and width limits: 2 <= N, 1 <= d <= 128; `scale` must be positive
 * and finite (TARMAC_ERR_SHAPE otherwise).
 */
#ifndef TARMAC_B200_H
#define TARMAC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden default visibility; everything declared in
 * this header is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes -------------------------------------------------------- */
#define TARMAC_OK 0
#define TARMAC_ERR_NULL 1       /* a required pointer is NULL                 */
#define TARMAC_ERR_SHAPE 2      /* B, N or d outside the supported range      */
#define TARMAC_ERR_DTYPE 3      /* dtype is not TARMAC_F32 / TARMAC_BF16       */
#define TARMAC_ERR_TOPK 4       /* k outside [1, N-1] or above the path limit */
#define TARMAC_ERR_N_TOO_LARGE 5 /* N above the resident-row limit (1024)     */
#define TARMAC_ERR_ALIGN 6      /* pointer or stride breaks the 16-byte rule  */
#define TARMAC_ERR_MODE 7       /* unknown selection mode / unsupported combo */
#define TARMAC_ERR_LAUNCH 8     /* the CUDA launch itself failed              */
#define TARMAC_ERR_BITS 9       /* Morton bits outside [1, 16]                */
#define TARMAC_ERR_SCRATCH 10   /* problem larger than the library's fixed
                                   scratch (no-allocation entry point)      */

/* ---- element types ------------------------------------------------------- */
#define TARMAC_F32 0
#define TARMAC_BF16 1

/* ---- selection modes of tarmac_topk_attention ---------------------------- */
/* Rank order is score descending; the modes differ only at an exact tie with
 * the k-th retained score. */
#define TARMAC_SELECT_ARGMAX 0    /* lowest index wins a tie (k argmax rounds,
                                     fused_topk_attention.py:275-284)         */
#define TARMAC_SELECT_THRESHOLD 1 /* every peer tied with the k-th score is
                                     kept, so a tie retains more than k
                                     (fused_topk_attention.py:180-194)       */
#define TARMAC_SELECT_SORT 2      /* highest index wins a tie (descending sort
                                     of (key<<32)|idx,
                                     fused_topk_attention.py:469-474)        */

/* ---- library identity ---------------------------------------------------- */
/* ABI version of this header; bumped on any signature change. */
#define TARMAC_ABI_VERSION 2
int tarmac_abi_version(void);
/* Static text for a status code (never NULL). */
const char *tarmac_strerror(int status);

/* ---- dense attention ----------------------------------------------------- */
/* Softmax over all N-1 peers (diagonal excluded), online softmax, no score
 * matrix written. Replaces fused_dense_attention and its kernel
 * _flash_dense_kernel (src/kernels/fused_dense_attention.py:38-152); the
 * eager forms are dense_unfused / dense_fused
 * (scripts/bench_attention_core.py:74-82). */
int tarmac_dense_attention(const void *q, const void *k, const void *v,
                           void *out, const int64_t *strides, int B, int N,
                           int d, int dtype, float scale, void *stream);

/* ---- fused score-then-select top-k attention ----------------------------- */
/* Scores every peer, keeps `topk` of them under `mode`, softmax over the
 * retained scores, V gather-aggregate; writes only `out` (and `idx_out`).
 * topk must lie in [1, N-1] (the Python layer clamps as the reference does).
 * idx_out: optional int32 [B, N, topk] contiguous, the retained peers in rank
 * order (score descending, ties by the mode's rule); supported for the ARGMAX
 * and SORT modes with topk <= 8, otherwise TARMAC_ERR_MODE.
 * ARGMAX / SORT with topk <= 8 stream the keys (any N); THRESHOLD mode and
 * topk > 8 use the resident-row path, N <= 1024 (TARMAC_ERR_N_TOO_LARGE).
 * Replaces fused_topk_attention, fused_topk_attention_tiled,
 * fused_topk_attention_masked and fused_topk_attention_sort
 * (src/kernels/fused_topk_attention.py:56-110, 127-208, 211-289, 296-387,
 * 405-540). */
int tarmac_topk_attention(const void *q, const void *k, const void *v,
                          void *out, const int64_t *strides, int B, int N,
                          int d, int dtype, float scale, int topk, int mode,
                          int32_t *idx_out, void *stream);

/* ---- streaming top-k attention ------------------------------------------- */
/* Exact top-k with keys streamed through shared memory: no N cap, topk <= 8,
 * lowest index wins a tie. idx_out optional int32 [B, N, topk] contiguous, in
 * rank order. Replaces streaming_topk_attention and _streaming_topk_kernel
 * (src/kernels/streaming_topk_attention.py:66-179, 206-258). */
int tarmac_streaming_topk_attention(const void *q, const void *k,
                                    const void *v, void *out,
                                    const int64_t *strides, int B, int N,
                                    int d, int dtype, float scale, int topk,
                                    int32_t *idx_out, void *stream);

/* ---- attention over a given peer set (select-before-scoring) ------------- */
/* idx: [B, N, kk] contiguous peer indices, int64 when idx_is_i64 else int32.
 * Online softmax over the kk given peers in order; no gathered tensor. A row
 * naming an index outside [0, N) is written as NaN (no out-of-bounds read).
 * Replaces fused_prescore_attention and _fused_prescore_kernel
 * (src/kernels/fused_prescore_attention.py:27-114) and the eager
 * prescore_attention (src/kernels/prescore_selection.py:184-195). */
int tarmac_prescore_attention(const void *q, const void *k, const void *v,
                              void *out, const int64_t *strides,
                              const void *idx, int idx_is_i64, int kk, int B,
                              int N, int d, int dtype, float scale,
                              void *stream);

/* ---- Morton (Z-order) selector ------------------------------------------- */
/* pos: fp32 [B, N, 2] contiguous positions. Per episode: min/max normalise,
 * quantise to `bits` per axis (truncation, clamp), interleave x bits at even
 * and y bits at odd positions. code_out: int64 [B, N].
 * Replaces _morton_code (src/kernels/prescore_selection.py:51-68). */
int tarmac_morton_code(const float *pos, int B, int N, int bits,
                       int64_t *code_out, void *stream);

/* Codes as above, stable ascending sort per episode (ties by agent index),
 * then for agent at rank r the peers at ranks r+1..r+h and r-1..r-(k-h)
 * modulo N, h = (k+1)/2. idx_out: int64 [B, N, k]. N <= 4096, 1 <= k <= N-1.
 * Replaces select_morton_window (src/kernels/prescore_selection.py:71-84),
 * with the bit width as a parameter (the reference fixes 10). */
int tarmac_morton_select(const float *pos, int B, int N, int k, int bits,
                         int64_t *idx_out, void *stream);

/* Fused select-before-scoring: Morton window selection as in
 * tarmac_morton_select followed by attention over the selected peers as in
 * tarmac_prescore_attention, one kernel, no index tensor written unless
 * idx_out (int64 [B, N, k], optional) is given. N <= 4096.
 * Replaces prescore_full(q, k, v, pos, kk, "morton_window")
 * (src/kernels/prescore_selection.py:198-200). */
int tarmac_morton_prescore_attention(const void *q, const void *k,
                                     const void *v, void *out,
                                     const int64_t *strides, const float *pos,
                                     int B, int N, int d, int dtype,
                                     float scale, int topk, int bits,
                                     int64_t *idx_out, void *stream);

/* ---- positional and random selectors ------------------------------------- */
/* Exact k nearest peers of every agent by Euclidean distance (squared
 * distance dx^2 + dy^2 in fp32, self excluded), listed by increasing
 * (distance, index): the lowest index wins an exact tie. pos: fp32
 * [B, N, 2] contiguous; idx_out: int64 [B, N, k]. 2 <= N <= 8192,
 * 1 <= k <= min(N - 1, 32). Replaces select_radius_knn
 * (src/kernels/prescore_selection.py:35-42). */
int tarmac_knn_select(const float *pos, int B, int N, int k, int64_t *idx_out,
                      void *stream);

/* Grid kNN: the k nearest among the 3 x 3 grid cells around each agent, with
 * the reference's grid side G = floor(sqrt(N / max(2, k))) and per-cell
 * capacity M = floor(mean + 3 sqrt(mean) + 2) (mean = N / G^2); each of the
 * three column runs of the 3 x 3 block is cut at 3M agents in cell order
 * (cells sorted stably: equal cells keep agent order). When 9M >= N the exact
 * selector runs instead, as in the reference; an agent whose runs hold fewer
 * than k candidates takes its exact k nearest. Same layout and limits as
 * tarmac_knn_select. Replaces select_grid_knn
 * (src/kernels/prescore_selection.py:87-164). */
int tarmac_grid_knn_select(const float *pos, int B, int N, int k,
                           int64_t *idx_out, void *stream);

/* k distinct peers per agent, uniform over the k-subsets of the other N - 1
 * agents, from a Philox stream keyed by (seed, row, offset): the selection
 * rule of the random_k arm (src/agents/mappo.py:233-263). idx_out: int64
 * [B, N, k], 1 <= k <= N - 1. */
int tarmac_random_select(int B, int N, int k, unsigned long long seed,
                         unsigned long long offset, int64_t *idx_out,
                         void *stream);

/* ---- the whole communication module (inference) --------------------------- */
/* AttentionComm.forward for the dense and top-k modes in one kernel
 * (src/agents/mappo.py:332-353, 361-373, 419-420):
 *   q, k, v = split(x W_qkv^T + b_qkv)      (nn.Linear layout: W [out, in])
 *   msg = dense attention (topk == 0) or top-k attention (1 <= topk <= 8,
 *         lowest index on a tie), diagonal excluded, scale 1/sqrt(msg_dim)
 *   out = gelu(msg) W_proj^T + b_proj          (exact erf GELU)
 * x: fp32 [B, N, in_dim] contiguous; weights fp32 contiguous; out: fp32
 * [B, N, msg_dim]. Q, K, V never leave the SM. 2 <= N, 1 <= in_dim <= 256,
 * 1 <= msg_dim <= 64, topk <= N - 1; the episode's Q, K and V must fit
 * shared memory (N * msg_dim up to about 16 K values; TARMAC_ERR_N_TOO_LARGE
 * otherwise). */
int tarmac_comm_forward(const float *x, const float *w_qkv, const float *b_qkv,
                        const float *w_proj, const float *b_proj, int B, int N,
                        int in_dim, int msg_dim, int topk, float *out,
                        void *stream);

/* ---- gradients (training) ------------------------------------------------ */
/* The reference trains through its eager path and autograd
 * (src/agents/mappo.py:192-231 topk_gather, 265-292 zorder_k, 361-373 dense);
 * these entry points give the same gradients for the kernels above.
 * dout = dL/dout has the layout of q. dq, dk, dv are fp32 [B, N, d]
 * contiguous and are written in full. */

/* Attention over a fixed peer set: the peers a top-k call retained (its
 * idx_out), the Morton window, or the indices given to
 * tarmac_prescore_attention. With s_m = (q_i . k_{j_m}) * scale,
 * w = softmax(s) and g = dout_i:
 *   ds_m = w_m (g . v_{j_m} - sum_m' w_m' g . v_{j_m'}),
 *   dq_i = scale sum_m ds_m k_{j_m},
 *   dk_j = scale sum_{(i,m): j_m = j} ds_m q_i,
 *   dv_j = sum_{(i,m): j_m = j} w_m g.
 * The selection carries no gradient (torch.topk's backward scatters only into
 * the selected entries). dk and dv are zeroed on the stream, then
 * accumulated with atomic adds, so their summation order is not fixed. A row
 * naming an index outside [0, N) gets a NaN dq row and adds nothing to dk/dv.
 * strides: 8 int64 { q_b, q_n, k_b, k_n, v_b, v_n, dout_b, dout_n } or NULL.
 * idx: contiguous [B, N, kk], int64 when idx_is_i64 else int32. */
int tarmac_gather_attention_backward(const void *q, const void *k,
                                     const void *v, const void *dout,
                                     const int64_t *strides, const void *idx,
                                     int idx_is_i64, int kk, int B, int N,
                                     int d, int dtype, float scale, float *dq,
                                     float *dk, float *dv, void *stream);

/* Dense masked-diagonal attention (tarmac_dense_attention). With
 * P = softmax(Q K^T scale) over j != i, `out` the forward output and
 * D_i = dout_i . out_i:
 *   dq_i = scale sum_j P_ij (dout_i . v_j - D_i) k_j,
 *   dk_j = scale sum_i P_ij (dout_i . v_j - D_i) q_i,
 *   dv_j = sum_i P_ij dout_i.
 * P is recomputed, never stored; deterministic. work: fp32 [2, B, N] scratch
 * (row log-sum-exp, then D). strides: 10 int64
 * { q_b, q_n, k_b, k_n, v_b, v_n, out_b, out_n, dout_b, dout_n } or NULL. */
int tarmac_dense_attention_backward(const void *q, const void *k,
                                    const void *v, const void *out,
                                    const void *dout, const int64_t *strides,
                                    int B, int N, int d, int dtype, float scale,
                                    float *dq, float *dk, float *dv,
                                    float *work, void *stream);

/* Dense-attention gradients without a caller workspace: the same result as
 * tarmac_dense_attention_backward, with the row statistics held in a fixed
 * 4 MiB device array inside the library instead of the `work` buffer. It has
 * no counterpart in the reference. It is for callers that cannot allocate
 * device memory: code run under a memory manager that owns every device
 * allocation and hands the library only its inputs and outputs, or a loop
 * that must not allocate once running, because a device allocation can
 * synchronise the device and take unbounded time. This call allocates
 * nothing (no cudaMalloc, no allocating library routine); the array is part
 * of the library image, so every GPU that loads the library holds it until
 * the process exits.
 * Limit: B * N <= 524288 query rows (TARMAC_ERR_SCRATCH beyond).
 * The array's device address belongs to a CUDA context: the first call in
 * each context (the context current at the call, which must own the
 * pointers) looks the address up and caches it under that context's id, so
 * a context created after cudaDeviceReset, or one the caller made current
 * through the driver API, gets its own lookup. Make the first call in a
 * context before any stream capture in it. Every call
 * shares the one array: calls that overlap on the GPU (other streams, other
 * threads) race on it, so serialise them. No scratch contents need to start
 * at zero (each call writes the statistics before reading them).
 * Arguments as tarmac_dense_attention_backward, without `work`. */
int tarmac_dense_attention_backward_noalloc(
    const void *q, const void *k, const void *v, const void *out,
    const void *dout, const int64_t *strides, int B, int N, int d, int dtype,
    float scale, float *dq, float *dk, float *dv, void *stream);

/* Which kernel, and with which tiling, a call with these arguments would
 * take — host-only: no launch, no device access, callable without a GPU.
 * Replaces the tuned-configuration lookup of the reference
 * (src/kernels/streaming_topk_attention.py:186-203 `_tuned_cfg`, and
 * scripts/bench_attention_core.py:120-145 for the dense tilings): there the
 * launch tiles come from a searched table; here the library chooses the
 * kernel and its tiles from the shape, and this call reports that choice.
 * op: 0 dense (tarmac_dense_attention), 1 top-k (tarmac_topk_attention, with
 * `mode`), 2 streaming top-k (tarmac_streaming_topk_attention). Pointers are
 * assumed on a 256-byte grid; strides as for those calls (NULL: contiguous).
 * Writes a NUL-terminated JSON object of at most `len` bytes, e.g.
 * {"kernel": "topk_ws", "query_tile": 128, "key_tile": 128, "chunk": 8,
 * "chunks_kept": 2}. Status codes as those calls' argument checks. */
int tarmac_kernel_plan(int op, int B, int N, int d, int dtype, int topk,
                       int mode, const int64_t *strides, char *out, int len);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* TARMAC_B200_H */
