/*
 * dsb.h - C ABI of libdsb.so, the B200 (sm_100a) decode hot path of
 * deepseek_cpp_infer.
 *
 * The reference crosses from its C++ model code into the GPU through the free
 * functions of ds::rt::cuda (include/ds/models/deepseek/cuda_backend.h:49-80)
 * and the kernel launchers of ds::rt::cuda::kernels
 * (include/ds/models/deepseek/cuda_kernels.h:10-25).  This header replaces
 * that boundary with plain C: opaque handles, raw pointers and sizes, no C++
 * or torch types.  Each entry point names the reference interface it stands
 * in for.
 *
 * Conventions
 *  - Every function returns DSB_OK (0) or a DSB_E* code; dsb_last_error()
 *    gives the message.  Nothing throws across the boundary (the reference's
 *    *_to_slot functions return bool for the same reason,
 *    cuda_backend.cpp:782-807).
 *  - Device pointers are raw CUDA device addresses (bf16 = 16-bit bfloat16
 *    payload).  Work is enqueued asynchronously on the context stream;
 *    dsb_sync() waits for it and reports kernel-side errors.
 *  - One context per GPU and per host thread (the reference keeps one global
 *    context on device 0, cuda_backend.cpp:565-568; here contexts are
 *    independent objects).
 *  - There is no CPU fallback: a call that cannot run on the GPU fails.
 */
#ifndef DSB_DSB_H_
#define DSB_DSB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSB_API __attribute__((visibility("default")))
#else
#define DSB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DSB_OK 0
#define DSB_EINVAL 1       /* bad argument, shape or size */
#define DSB_ECUDA 2        /* a CUDA runtime/driver call failed */
#define DSB_ENOMEM 3       /* device allocation failed */
#define DSB_ETIMEOUT 4     /* a kernel's bounded wait ran out (device status word) */
#define DSB_EUNSUPPORTED 5 /* shape not covered by the sm_100a kernels */
#define DSB_ELIMIT 6       /* request exceeds the fixed scratch of dsb_mla_decode_noalloc */

typedef struct dsb_ctx dsb_ctx;

/* Per-context counters; replaces the process-global CudaStats
 * (cuda_backend.h:26-45, cuda_backend.cpp:573) as the "really ran on the GPU"
 * evidence. */
typedef struct dsb_stats {
  uint64_t kernel_launches; /* kernels enqueued by this context */
  uint64_t mla_calls;
  uint64_t mla_work_items; /* cluster work items summed over calls */
  uint64_t mla_partials;   /* work items that wrote a split-KV partial */
  uint64_t workspace_bytes;
  uint64_t gemm_calls;     /* dsb_linear launches */
  uint64_t decode_steps;   /* dsb_decode_step calls */
  uint64_t prefill_tokens; /* token rows run by dsb_prefill */
} dsb_stats;

/* Library version (major*10000 + minor*100 + patch). */
DSB_API int dsb_version(void);

/* Create / destroy a context bound to CUDA device `device`.
 * Replaces ensure_initialized / create_executor_state / destroy_executor_state
 * (cuda_backend.h:49-56). */
DSB_API int dsb_ctx_create(int device, dsb_ctx** out);
DSB_API int dsb_ctx_destroy(dsb_ctx* ctx);

/* Use `stream` (a cudaStream_t) for all work of the context; NULL restores
 * the context's own stream.  The caller keeps ownership of `stream`. */
DSB_API int dsb_ctx_set_stream(dsb_ctx* ctx, void* stream);
DSB_API void* dsb_ctx_stream(dsb_ctx* ctx);

/* Message of the last failed call on this context ("" when none). */
DSB_API const char* dsb_last_error(const dsb_ctx* ctx);

/* Wait for the context stream, then read and clear the device status word:
 * DSB_ETIMEOUT if a kernel's bounded wait ran out since the last dsb_sync. */
DSB_API int dsb_sync(dsb_ctx* ctx);

/* Time limit of the expert-parallel flag waits of kernels launched on this
 * context from now on (default 2 s, accepted range 1 ms .. 60 s): a wait that
 * runs out sets the status word (dsb_sync returns DSB_ETIMEOUT) and its kernel
 * returns.  The reference has no bounded waits: no counterpart. */
DSB_API int dsb_ctx_set_wait_limit(dsb_ctx* ctx, uint64_t limit_ns);

/* Copy the context counters (replaces stats(), cuda_backend.h:52). */
DSB_API int dsb_get_stats(const dsb_ctx* ctx, dsb_stats* out);
DSB_API int dsb_reset_stats(dsb_ctx* ctx); /* replaces reset_stats(), cuda_backend.h:51 */

/*
 * Absorbed-weight MLA decode attention over a paged latent cache: one query
 * token per sequence, all heads.
 *
 * Replaces the per-head attention loop of mla_decode_to_slot
 * (src/models/deepseek/cuda_backend.cpp:953-991: ds_scores_kernel,
 * ds_softmax_kernel, ds_weighted_sum_kernel per head) and of mla_decode_step
 * (src/models/deepseek/mla.cpp:86-116).  With q_lat = W_UK^T q_nope the
 * reference's scores q.k/sqrt(nope+rope) equal [q_lat | q_rope].[c | kr] *
 * softmax_scale, and its per-head output equals W_UV * out_lat, so this call
 * returns the latent output out_lat.
 *
 * Work is split into runs of whole 64-token pages ("work items") planned on
 * the host from the sequence lengths.  A plan depends only on (seq_lens, H,
 * R, P) and is reused by every layer of a decode step.
 *
 *  q_lat        bf16 [B, H, R]     absorbed nope query
 *  q_rope       bf16 [B, H, P]     rotated rope query
 *  kv_cache     bf16 [n_blocks, block_size, R + P]   rows [c | kr]
 *  block_table  int32 device [B, max_blocks]  page ids of each sequence
 *  seq_lens     int32 HOST [B]  tokens in the cache per sequence (>= 1)
 *  out_lat      bf16 [B, H, R]  softmax(q.k * scale) . c
 * Supported: block_size 64, (R, P) in {(512, 64), (128, 32)}, 1 <= H <= 128.
 * Rows of a page past a sequence's length must hold finite values (the
 * paged-cache pool of dsb is zero-filled at creation).
 */
typedef struct dsb_mla_plan dsb_mla_plan;

DSB_API int dsb_mla_plan_create(dsb_ctx* ctx, const int32_t* seq_lens, int B, int H, int R, int P, int block_size,
                                dsb_mla_plan** out);
DSB_API int dsb_mla_plan_destroy(dsb_mla_plan* plan);
/* Number of work items and of split-KV partials of a plan. */
DSB_API int dsb_mla_plan_info(const dsb_mla_plan* plan, int* n_items, int* n_partial);

/* Enqueue the decode for a plan (asynchronous on the context stream). */
DSB_API int dsb_mla_decode_planned(dsb_ctx* ctx, const dsb_mla_plan* plan, const void* q_lat, const void* q_rope,
                                   const void* kv_cache, int64_t n_blocks, const int32_t* block_table, int max_blocks,
                                   float softmax_scale, void* out_lat);

/* Plan + decode in one call (the plan goes to a context-owned device buffer;
 * still asynchronous on the context stream). */
DSB_API int dsb_mla_decode(dsb_ctx* ctx, const void* q_lat, const void* q_rope, const void* kv_cache, int64_t n_blocks,
                           int block_size, const int32_t* block_table, int max_blocks, const int32_t* seq_lens, int B,
                           int H, int R, int P, float softmax_scale, void* out_lat);

/*
 * Allocation-free MLA decode: the same computation as dsb_mla_decode, for
 * callers that cannot allocate device memory while they run this call - a
 * host runtime that owns all device memory through its own allocator and
 * forbids stray cudaMalloc/cudaFree (a cudaFree also synchronises the whole
 * device), or a plug-in that only receives a stream and its buffers.  It
 * takes no dsb_ctx (creating one allocates) and calls no cudaMalloc/cudaFree:
 * its scratch (work list, split-KV partials, status word) is one fixed
 * device array of about 6.4 MB inside libdsb.so, held by every GPU that loads
 * the library until the process exits.  No counterpart in the reference.
 *
 *  stream  cudaStream_t to enqueue on (NULL = the legacy default stream);
 *          the current CUDA device must be the one that holds the buffers.
 *  other arguments as dsb_mla_decode.
 * Limits: at most 4096 work items and 24 split-KV partials per call.  When
 * the usual plan needs more than 24 partials, the call falls back to one
 * work item per 16384 tokens of each sequence; only sequences longer than
 * 16384 tokens then split, into ceil(len / 16384) partials each.  A call
 * whose fallback still needs more than 24 partials (for example 13 sequences
 * of 17000 tokens, 2 partials each) returns DSB_ELIMIT and enqueues nothing.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) and sets kernel attributes; make that first call
 * before any stream capture on the device.  Every call reuses the
 * same array, so calls that overlap on the GPU (different streams, or
 * different host threads on one device) race and must be serialised by the
 * caller.  Each call clears the status word; dsb_mla_noalloc_status reads it.
 */
DSB_API int dsb_mla_decode_noalloc(void* stream, const void* q_lat, const void* q_rope, const void* kv_cache,
                                   int64_t n_blocks, int block_size, const int32_t* block_table, int max_blocks,
                                   const int32_t* seq_lens, int B, int H, int R, int P, float softmax_scale,
                                   void* out_lat);
/* Waits for `stream` and returns the status of the last dsb_mla_decode_noalloc
 * call on the current device: DSB_OK, or DSB_ETIMEOUT when a bounded wait in
 * its kernel ran out (its output is then not valid).  Allocates nothing.
 * No counterpart in the reference. */
DSB_API int dsb_mla_noalloc_status(void* stream);

/*
 * Grouped bf16 linear layer (tcgen05, fp32 accumulation):
 *   for each group g and token row t of the group,
 *   acc[t, n] = sum_k x[t, g*x_group_col + k] * w[g*M + n, k],  n < M
 * then an epilogue writes column g*y_group_col + n of row t of y.
 *
 * Replaces the reference's GEMV path - cublasSgemv / cublasGemmEx in
 * gemv_row_major_mixed (src/models/deepseek/cuda_backend.cpp:459-498) behind
 * linear_to_slot (cuda_backend.cpp:782-807) and ds::rt::linear
 * (src/models/deepseek/ops.cpp:49-86) - and the per-expert GEMV chains of
 * dense_mlp_to_slot / moe_to_slot (cuda_backend.cpp:820-883).
 *
 * Groups cover: one plain linear (G = 1); per-head absorbed projections
 * (G = heads, same tokens, x_group_col / y_group_col select the head's
 * slice); routed experts (G = experts, tok_offsets gives each expert's rows of
 * a permuted activation matrix).
 *
 * Epilogues:
 *  DSB_EPI_STORE      y = acc (bf16 or fp32 per y_f32)
 *  DSB_EPI_ADD        y += acc (fp32 y; residual add, replaces ds_add_inplace_kernel)
 *  DSB_EPI_SILU_GATE  w holds gate and up rows interleaved (row 2f = gate row f,
 *                     row 2f+1 = up row f); y[t, f] = silu(gate) * up
 *                     (dense_mlp_step's silu(gate)*up, ops.cpp:103-105)
 *  DSB_EPI_ROWSCALE   y = acc * row_scale[t] (routed weight of a permuted row)
 * Requirements: K, ldw, ldx, x_group_col multiples of 64/8/8/8; 16-byte
 * aligned w and x.  max_tokens_per_group bounds the rows of any group (T when
 * tok_offsets is NULL); it sets the MMA N tile (16..256).
 */
#define DSB_EPI_STORE 0
#define DSB_EPI_ADD 1
#define DSB_EPI_SILU_GATE 2
#define DSB_EPI_ROWSCALE 3

typedef struct dsb_linear_args {
  const void* w;              /* bf16 [G * M, ldw] */
  int64_t ldw;                /* row pitch of w (elements) */
  const void* x;              /* bf16 [T, ldx] */
  int64_t ldx;                /* row pitch of x (elements) */
  int64_t x_group_col;        /* group g reads x columns [g*x_group_col, +K) */
  const int32_t* tok_offsets; /* device int32 [G + 1] row ranges, or NULL: every group uses rows [0, T) */
  int T, M, K, G;
  int max_tokens_per_group;   /* host bound on rows per group (<= 0: T) */
  void* y;                    /* output (bf16 or fp32 per y_f32) */
  int64_t ldy;                /* row pitch of y (elements) */
  int64_t y_group_col;        /* group g writes y columns [g*y_group_col, ...) */
  int y_f32;                  /* 1: y is fp32, 0: bf16 */
  int epilogue;               /* DSB_EPI_* */
  const float* row_scale;     /* DSB_EPI_ROWSCALE: fp32 [T] */
} dsb_linear_args;

DSB_API int dsb_linear(dsb_ctx* ctx, const dsb_linear_args* args);

/* -------------------------------------------------------------- FP8 e4m3
 *
 * DeepSeek-V3 block-scaled FP8: weights e4m3 with one fp32 scale per 128x128
 * block (the checkpoints' weight_scale_inv), activations e4m3 with one fp32
 * scale per token and 128 columns.  The reference has no FP8 path (its
 * safetensors dtype parser, src/hf/safetensors.cpp:12-20, knows F32/F16/BF16
 * only); these replace linear_to_slot / moe_to_slot's GEMVs
 * (src/models/deepseek/cuda_backend.cpp:782-883) for FP8 checkpoints. */

/* q = e4m3(x / s) with s = amax / 448 over each 128 columns of a row (1 for an
 * all-zero group), round to nearest even, saturating; s written to
 * scales[row * ld_scales + col / 128].  x bf16 or fp32 (x_dtype DSB_DTYPE_*)
 * [.., ldx]; with src_rows (device int32 [T]) row t reads x row
 * src_rows[t] / k (the permuted-token gather of dsb_gather_rows), else row t.
 * K a multiple of 128. */
DSB_API int dsb_quant_act_1x128(dsb_ctx* ctx, const void* x, int x_dtype, int64_t ldx, const int32_t* src_rows,
                                int k, int T, int K, void* q, int64_t ldq, float* scales, int64_t ld_scales);

/* Weight quantisation for bf16/fp32 checkpoints: w [M, K] -> e4m3 q [M, K]
 * and scales [ceil(M/128), ceil(K/128)] = amax / 448 of each 128x128 block
 * (1 for an all-zero block); the same rounding as dsb_quant_act_1x128. */
DSB_API int dsb_quant_weight_128x128(dsb_ctx* ctx, const void* w, int w_dtype, int64_t M, int64_t K, void* q,
                                     float* scales);

/* Grouped block-scaled FP8 linear; same grouping, token ranges and epilogues
 * as dsb_linear:
 *   acc[t, n] = sum_kb sw(g, n, kb) * x_scale[t, g*x_group_col/128 + kb]
 *               * sum_{k in kb} x[t, g*x_group_col + k] * w[g*M + n, k]
 * Weight scales are per 128-row tile of a group: with scale_rows 1,
 * w_scale[(g*ceil(M/128) + n/128) * K/128 + kb] (the checkpoints' per-matrix
 * [ceil(M/128), K/128] layout stacked over groups); with scale_rows 2 (a
 * row-interleaved gate|up matrix for DSB_EPI_SILU_GATE), tile j holds
 * gate and up rows 64j..64j+63 and w_scale[((g*M/128 + j) * 2 + (n & 1)) * K/128 + kb]
 * is the gate (n even) or up (n odd) scale of those rows.  K, x_group_col
 * multiples of 128; ldw, ldx multiples of 16 bytes. */
typedef struct dsb_linear_fp8_args {
  const void* w;              /* e4m3 [G * M, ldw] */
  int64_t ldw;                /* row pitch of w (bytes) */
  const float* w_scale;       /* fp32, layout above */
  int scale_rows;             /* 1 or 2 */
  const void* x;              /* e4m3 [T, ldx] */
  int64_t ldx;                /* row pitch of x (bytes) */
  const float* x_scale;       /* fp32 [T, ld_xs] */
  int64_t ld_xs;              /* row pitch of x_scale (floats) */
  int64_t x_group_col;        /* group g reads x columns [g*x_group_col, +K) */
  const int32_t* tok_offsets; /* device int32 [G + 1] row ranges, or NULL */
  int T, M, K, G;
  int max_tokens_per_group;   /* host bound on rows per group (<= 0: T) */
  void* y;                    /* output (bf16 or fp32 per y_f32) */
  int64_t ldy;
  int64_t y_group_col;
  int y_f32;
  int epilogue;               /* DSB_EPI_* */
  const float* row_scale;     /* DSB_EPI_ROWSCALE: fp32 [T] */
} dsb_linear_fp8_args;

DSB_API int dsb_linear_fp8(dsb_ctx* ctx, const dsb_linear_fp8_args* args);

/* One MoE layer's experts in block-scaled FP8, for routed picks (ids, weights
 * from dsb_moe_route, [T, k]) plus n_shared shared experts stacked after the
 * E routed ones (groups E .. E+n_shared-1, weight 1 for every token):
 *   h[t] += sum_j weights[t,j] * expert_{ids[t,j]}(x[t]) + sum_s shared_s(x[t])
 * summed in that order (moe_step, src/models/deepseek/ops.cpp:133-145).
 * expert(x) = down(silu(gate x) * up x): x is quantised per token and 128
 * columns, gate|up run as one grouped GEMM with the SiLU epilogue (bf16 out),
 * that is quantised again and the down GEMM scales each row by its routing
 * weight.  Weights over G = E + n_shared groups:
 *   gate_up       e4m3 [G, 2I, D], rows interleaved (2f gate f, 2f+1 up f)
 *   gate_up_scale fp32 [G, 2I/128, 2, D/128] (dsb_linear_fp8 scale_rows 2)
 *   down          e4m3 [G, D, I]
 *   down_scale    fp32 [G, D/128, I/128]
 * x bf16 [T, D] (row pitch ldx), h fp32 [T, D].  D and I multiples of 128.
 * Scratch comes from the context.  Replaces moe_to_slot's expert loop
 * (src/models/deepseek/cuda_backend.cpp:836-883) for FP8 checkpoints. */
typedef struct dsb_moe_fp8_layer {
  const void* gate_up;
  const float* gate_up_scale;
  const void* down;
  const float* down_scale;
  int E, n_shared, D, I;
} dsb_moe_fp8_layer;

DSB_API int dsb_moe_ffn_fp8(dsb_ctx* ctx, const dsb_moe_fp8_layer* layer, const void* x, int64_t ldx, int T, int k,
                            const int32_t* ids, const float* weights, float* h);

/* ---------------------------------------------------------------- row ops */

/* y = x / sqrt(mean(x^2) + eps) * w per row, written as bf16 (y_bf16) and/or
 * fp32 (y_f32).  x fp32 [rows, ldx], w fp32 [n].
 * Replaces rmsnorm_to_slot / ds_rmsnorm_kernel (cuda_backend.cpp:809,
 * src/ops/cuda/elementwise_kernels.cu:13-28) and rmsnorm_f32
 * (src/ops/core/ops.cpp:17-23). */
DSB_API int dsb_rmsnorm(dsb_ctx* ctx, const float* x, int64_t ldx, const float* w, int rows, int n, float eps,
                        void* y_bf16, int64_t ldy_bf16, float* y_f32, int64_t ldy_f32);

/* Fused latent-cache append for B tokens at positions[b] (device int32):
 *   c = rmsnorm(kv_a[b, :R]) * w_norm, kr = rope(kv_a[b, R:R+P], pos)
 * written as bf16 into row pos of sequence b in the paged cache
 * (block_table[b * max_blocks + pos / 64], row pos % 64), and
 * q_rope[b, h] = rope(q[b, h, nope:nope+P], pos) (bf16) for every head.
 * kv_a fp32 [B, R+P]; q bf16 [B, H*(nope+P)]; cache bf16 [n_blocks, 64, R+P].
 * Replaces the kv_a split / rmsnorm / RoPE / per-head cache copies of
 * mla_decode_to_slot (cuda_backend.cpp:922-982) and mla.cpp:71-102. */
DSB_API int dsb_kv_norm_rope_append(dsb_ctx* ctx, const float* kv_a, const float* w_norm, const void* q,
                                    const int32_t* positions, const int32_t* block_table, int max_blocks, int B, int H,
                                    int nope, int R, int P, float eps, float theta, void* cache, void* q_rope);

/* fp32 router logits [T, E] = x [T, D] . W_gate [E, D]^T (ops.cpp:115-117). */
DSB_API int dsb_router_logits(dsb_ctx* ctx, const float* x, const float* w_gate, int T, int D, int E, float* logits);

#define DSB_SCORE_SOFTMAX 0
#define DSB_SCORE_SIGMOID 1

/* Expert selection per token from fp32 logits [T, E] (E <= 256, k <= 8):
 *  DSB_SCORE_SOFTMAX: softmax, top-k, optional renormalisation, times
 *    routed_scale (moe_step, ops.cpp:110-131,137; ds_select_topk_kernel,
 *    routing_kernels.cu:8-44).  bias unused.
 *  DSB_SCORE_SIGMOID: sigmoid + bias[E], n_group groups ranked by their
 *    top-2 biased scores, topk_group groups kept, top-k by biased score,
 *    weights = unbiased scores (normalised when norm_topk) times routed_scale.
 * Ties go to the lower expert id.  ids int32 [T, k], weights fp32 [T, k]. */
DSB_API int dsb_moe_route(dsb_ctx* ctx, const float* logits, const float* bias, int T, int E, int k, int scoring,
                          int n_group, int topk_group, int norm_topk, float routed_scale, int32_t* ids,
                          float* weights);

/* Histogram and permutation of the T*k (token, slot) pairs by expert:
 * counts [E], offsets [E+1] (exclusive prefix sum), dest [T*k] (position of
 * pair t*k+j in expert order, stable in pair order), src_pair [T*k] (its
 * inverse); when weights [T*k] is given, w_perm[dest[i]] = weights[i].
 * Replaces the per-expert host loop of moe_to_slot (cuda_backend.cpp:854-874)
 * and its top-k download + sync. */
DSB_API int dsb_moe_permute(dsb_ctx* ctx, const int32_t* ids, int T, int k, int E, int32_t* counts, int32_t* offsets,
                            int32_t* dest, int32_t* src_pair, const float* weights, float* w_perm);

/* out[p] = x[src_pair[p] / k] for bf16 rows of D (D, ldx multiples of 8). */
DSB_API int dsb_gather_rows(dsb_ctx* ctx, const void* x, int64_t ldx, const int32_t* src_pair, int n_pairs, int k,
                            int D, void* out);

/* h[t] += (sum_j y[dest[t*k + j]]) + shared[t] (shared may be NULL): the
 * routed-expert combine of moe_step (ops.cpp:133-145) plus the residual add
 * (model.cpp:209); replaces ds_scale_add_kernel / ds_add_inplace_kernel. */
DSB_API int dsb_moe_combine(dsb_ctx* ctx, const float* y, const int32_t* dest, int T, int k, int D,
                            const float* shared, float* h);

/* ------------------------------------------------------ expert parallelism
 *
 * world ranks (one process and GPU each, world <= 8) split the E routed
 * experts: expert e lives on rank e / (E / world).  Every rank keeps its own
 * tokens and, per MoE layer, sends each pick's token row to the expert's
 * rank and gets the expert's output back, by kernels that write straight
 * into the other GPUs' memory (one CUDA IPC window per rank; no collective
 * library on the data path).  The reference is single-GPU: no counterpart.
 *
 * Set-up: dsb_ep_create on every rank, exchange the 64-byte window handles
 * (dsb_ep_window_handle) by any host channel, then dsb_ep_connect with all
 * world handles in rank order.  Per layer, every rank (also one with T = 0)
 * calls dsb_ep_dispatch and then dsb_ep_combine, in the same order; the
 * kernels wait for the peers with bounded waits (dsb_sync reports a timeout).
 *
 * dispatch: x bf16 [T, ldx] and the global expert ids [T, top_k] of this
 *   rank's tokens.  Returns (device pointers owned by the group, valid until
 *   the next dispatch) the received rows recv_x bf16 [capacity, hidden],
 *   grouped by local expert (sources in rank order, then pick order), and
 *   recv_offsets int32 [E_local + 1], the row range of each local expert:
 *   the tok_offsets of a grouped dsb_linear over the local experts.
 * combine: y fp32 [capacity, ldy], the experts' outputs in recv_x row order
 *   (unweighted); every output goes back to its token's rank, which adds
 *     h[t] += sum_j weights[t,j] * out[t,j] + sum_s shared[s*T + t]
 *   in that order (moe_step, src/models/deepseek/ops.cpp:133-145); shared
 *   fp32 [n_shared, T, hidden] holds this rank's shared-expert outputs. */
typedef struct dsb_ep dsb_ep;
#define DSB_EP_HANDLE_BYTES 64

DSB_API int dsb_ep_create(dsb_ctx* ctx, int rank, int world, int n_experts, int hidden, int top_k, int max_tokens,
                          dsb_ep** out);
DSB_API int dsb_ep_window_handle(dsb_ep* ep, void* handle);
DSB_API int dsb_ep_connect(dsb_ep* ep, const void* handles);
DSB_API int dsb_ep_info(const dsb_ep* ep, int* E_local, int* recv_capacity, uint64_t* window_bytes);
DSB_API int dsb_ep_dispatch(dsb_ep* ep, const void* x, int64_t ldx, int T, const int32_t* ids, void** recv_x,
                            int32_t** recv_offsets);
DSB_API int dsb_ep_combine(dsb_ep* ep, const float* y, int64_t ldy, int T, const float* weights,
                           const float* shared, int n_shared, float* h);
DSB_API int dsb_ep_destroy(dsb_ep* ep);
/* Ranks driven from ONE process (one GPU each, peer access enabled by the
 * caller): connect with the device pointers of every rank's window
 * (dsb_ep_window_ptr; windows[rank] is ignored) instead of IPC handles.  The
 * ranks' kernels wait on one another, so two ranks of a group must never be
 * driven on the same GPU. */
DSB_API int dsb_ep_window_ptr(dsb_ep* ep, void** ptr);
DSB_API int dsb_ep_connect_local(dsb_ep* ep, void* const* windows);

/* Greedy ids: first index of the row maximum of logits [B, ld] (argmax_f32,
 * src/core/math.cpp:29-40; the reference downloads the logits and does this
 * on the host, cuda_backend.cpp:746-757). */
DSB_API int dsb_argmax(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, int32_t* out);

/* Stochastic sampling: ds::core::Sampler::sample (src/core/sampler.cpp:23-77)
 * for B rows of logits [B, V] (row pitch ld, fp32, device) at once.
 * Temperature (<= 0 reads as 1), then a top-k cut (0 < top_k < V; ties at the
 * boundary keep the lower ids), softmax over the kept items, a top-p nucleus
 * cut (0 < top_p < 1: the shortest descending-probability prefix whose mass
 * reaches top_p, renormalised), and the item at which the cumulative mass
 * reaches uniforms[b] (device, one draw in [0, 1) per row, from the caller's
 * generator, as the reference draws one per call).  The cumulative mass runs
 * in id order when no cut is active (the reference's order) and in
 * descending probability, ties to the lower id, when one is (the reference's
 * order there is unspecified).  Deterministic for given inputs.  Rows
 * holding NaN give an unspecified id in [0, V).  V <= 2^21.  out_ids [B]
 * int32 on the device. */
DSB_API int dsb_sample(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, float temperature, int top_k,
                       float top_p, const float* uniforms, int32_t* out_ids);

/* h[b] = fp32 embedding row tokens[b] of table [V, D] (bf16 when table_bf16,
 * else fp32); replaces embedding_to_slot (cuda_backend.cpp:716-732). */
DSB_API int dsb_embed(dsb_ctx* ctx, const void* table, int table_bf16, const int32_t* tokens, int B, int D, float* h);

/* ------------------------------------------------------ whole-model decode */

#define DSB_DTYPE_F32 0
#define DSB_DTYPE_BF16 1
#define DSB_DTYPE_F8E4M3 3 /* raw e4m3 bytes (model weights with *_scale_inv) */
#define DSB_DTYPE_F16 2

/* The model hyper-parameters the decode path reads: the fields of
 * ds::hf::DeepSeekConfig (include/ds/models/deepseek/config.h:10-39) plus the
 * DeepSeek-V3 router fields that config parser lacks (n_group, topk_group,
 * scoring_func as DSB_SCORE_*). */
typedef struct dsb_model_config {
  int hidden_size, num_hidden_layers, num_attention_heads, vocab_size, max_position_embeddings;
  int intermediate_size;     /* dense FFN */
  int moe_intermediate_size; /* per routed expert */
  int n_routed_experts, n_shared_experts, num_experts_per_tok, first_k_dense_replace;
  int q_lora_rank; /* 0: q_proj */
  int kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, v_head_dim;
  int scoring_func, n_group, topk_group, norm_topk_prob;
  float routed_scaling_factor, rms_norm_eps, rope_theta;
  /* dsb_model_init_random only: 1 = the projections and FFN / expert weights
   * in block-scaled FP8 (e4m3 + 128x128 fp32 scales, DeepSeek-V3 style). */
  int weights_fp8;
} dsb_model_config;

typedef struct dsb_model dsb_model;

/* Device-resident model.  Replaces DeepSeekWeightRegistry
 * (src/models/deepseek/weights.cpp:54-113) plus the executor's weight cache
 * (cuda_backend.cpp:402-457): tensors are uploaded once by checkpoint name and
 * kept in the layouts the kernels read (bf16 matrices; kv_b_proj split into
 * per-head W_UK^T and W_UV; gate/up interleaved; norms and router fp32).
 * A layer is MoE when its routed experts are given (weights.cpp:89-96). */
DSB_API int dsb_model_create(dsb_ctx* ctx, const dsb_model_config* cfg, dsb_model** out);
DSB_API int dsb_model_destroy(dsb_model* model);
/* Upload one checkpoint tensor from HOST memory, named as in the HF
 * safetensors ("model.layers.3.self_attn.kv_b_proj.weight", ...); dtype is
 * DSB_DTYPE_*.  The caller keeps ownership of `data`.
 * Block-scaled FP8 checkpoints: a projection, FFN or expert weight given as
 * DSB_DTYPE_F8E4M3 (raw e4m3 bytes) is kept in FP8 and needs its fp32
 * "<name>_scale_inv" tensor [ceil(rows/128), ceil(cols/128)] (either order);
 * those layers then run the FP8 GEMM with 1x128-quantised activations.
 * kv_b_proj is dequantised to bf16 at load (absorbed attention). */
DSB_API int dsb_model_set_tensor(dsb_model* model, const char* name, int dtype, const int64_t* shape, int ndim,
                                 const void* data);
/* Fill every weight on the device with N(0, stddev) (norms 1), layer kinds
 * from first_k_dense_replace; for benchmarks of random-init models.
 * Finalizes the model. */
DSB_API int dsb_model_init_random(dsb_model* model, uint64_t seed, float stddev);
/* Check completeness (every layer's attention and FFN weights present). */
DSB_API int dsb_model_finalize(dsb_model* model);

/* Bind a model to an expert-parallel group before any of its tensors is set:
 * it then keeps only this rank's routed experts (set_tensor accepts and
 * skips the others; init_random makes only these) plus the shared experts,
 * and dsb_decode_step exchanges every MoE layer's picks through the group.
 * Every rank of the group calls dsb_decode_step in step (B >= 1 each, at most
 * the group's max_tokens). */
DSB_API int dsb_model_set_ep(dsb_model* m, dsb_ep* ep);

DSB_API int dsb_model_weight_bytes(const dsb_model* model, uint64_t* bytes);

typedef struct dsb_kvcache dsb_kvcache;

/* Paged latent KV cache for every layer: n_blocks pages of 64 tokens x
 * (kv_lora_rank + rope) bf16 per layer, zero-filled, shared by up to
 * max_seqs sequences of at most max_blocks_per_seq pages.  Replaces MLACache
 * (src/models/deepseek/mla.cpp:16-39) / CudaMLACache (cuda_backend.cpp:81-88),
 * which hold full per-head K and V in fp32. */
DSB_API int dsb_kvcache_create(dsb_ctx* ctx, const dsb_model* model, int64_t n_blocks, int max_seqs,
                               int max_blocks_per_seq, dsb_kvcache** out);
DSB_API int dsb_kvcache_destroy(dsb_kvcache* kv);
DSB_API int dsb_kvcache_alloc_seq(dsb_kvcache* kv, int* seq_id);
DSB_API int dsb_kvcache_free_seq(dsb_kvcache* kv, int seq_id);
/* Free every sequence (DeepSeekSession::reset, model.cpp:57-69). */
DSB_API int dsb_kvcache_reset(dsb_kvcache* kv);
DSB_API int dsb_kvcache_seq_len(const dsb_kvcache* kv, int seq_id, int* len);
DSB_API int dsb_kvcache_free_blocks(const dsb_kvcache* kv, int64_t* n);
/* Append n_tokens synthetic positions to a live sequence: pages are taken as
 * decoding would take them and every layer's rows get N(0, stddev) bf16
 * latents (seeded).  For benchmarks that need a long context without
 * prefilling it token by token; no counterpart in the reference. */
DSB_API int dsb_kvcache_fill_random(dsb_kvcache* kv, int seq_id, int n_tokens, uint64_t seed, float stddev);

/* One decode step: token tokens[b] of sequence seq_ids[b] (HOST arrays, B
 * distinct live sequences) is appended at the sequence's current length and
 * run through every layer; greedy ids (HOST int32 [B]) and, when logits is
 * not NULL, the logits (HOST fp32 [B, vocab]) are returned.  Batched
 * replacement of DeepSeekModel::decode_next (model.cpp:112-221); returns
 * after the step completed on the device. */
DSB_API int dsb_decode_step(dsb_ctx* ctx, dsb_model* model, dsb_kvcache* kv, const int32_t* seq_ids,
                            const int32_t* tokens, int B, float* logits, int32_t* greedy);

/* Most token rows of one dsb_prefill call (longer prompts are fed in chunks). */
#define DSB_PREFILL_MAX_TOKENS 4096

/* Chunked prefill: n_tok token rows in one pass through every layer.  Row i
 * is token tokens[i] of live sequence seq_ids[i] (HOST arrays); a sequence
 * may appear several times, its tokens in prompt order, appended at
 * consecutive positions after its current length.  Each row attends to its
 * sequence's cache up to and including its own position, so the result is
 * the same computation as feeding the rows one at a time through
 * dsb_decode_step (the reference's token-by-token forward(),
 * model.cpp:104-110), with every GEMM and the MoE batched over all rows.
 * The lm_head runs only on the last row of each distinct sequence, in order
 * of first appearance in seq_ids: *n_seq (HOST, may be NULL) of them; their
 * greedy ids go to greedy (HOST int32 [n_seq]) and, when logits is not NULL,
 * their logits to logits (HOST fp32 [n_seq, vocab]).  n_tok <=
 * DSB_PREFILL_MAX_TOKENS.  A model bound to an expert-parallel group
 * exchanges every MoE layer's picks of all n_tok rows: every rank calls
 * dsb_prefill in step (at least one row each, at most the group's
 * max_tokens).  No counterpart in the reference (it prefills token by
 * token). */
DSB_API int dsb_prefill(dsb_ctx* ctx, dsb_model* model, dsb_kvcache* kv, const int32_t* seq_ids,
                        const int32_t* tokens, int n_tok, float* logits, int32_t* greedy, int* n_seq);

/* Batched greedy generation: ds::rt::generate (src/runtime/model.cpp:14-49)
 * for B sequences of the cache at once, on the host over dsb_decode_step.
 * Sequence b's prompt is prompt_tokens[prompt_offsets[b] .. prompt_offsets[b+1])
 * (at least one token), consumed token by token as the reference's forward()
 * does; then its greedy ids are fed back until max_new_tokens ids or eos_id
 * (>= 0, kept in the output; < 0 for none).  out_ids [B, max_new_tokens]
 * (host), out_counts [B] (host) the ids written per sequence.  Greedy; see
 * dsb_generate_sampled for temperature / top-k / top-p.  Not for models
 * bound to an expert-parallel group (their ranks step together). */
DSB_API int dsb_generate(dsb_ctx* ctx, dsb_model* model, dsb_kvcache* kv, const int32_t* seq_ids, int B,
                         const int32_t* prompt_tokens, const int32_t* prompt_offsets, int max_new_tokens,
                         int32_t eos_id, int32_t* out_ids, int32_t* out_counts);

/* Sampling settings: ds::core::SamplerConfig (include/ds/core/sampler.h:9-14)
 * as ds::rt::GenerationConfig carries them. */
typedef struct dsb_sampling {
  float temperature; /* <= 0 reads as 1 */
  int top_k;         /* 0 (or >= vocab) disables the top-k cut */
  float top_p;       /* 0 (or >= 1) disables the top-p cut */
  uint32_t seed;     /* dsb_generate_sampled: 0 = std::random_device, as the reference */
} dsb_sampling;

/* dsb_decode_step whose next id per row is sampled on the device (dsb_sample)
 * instead of the greedy argmax: uniforms_host[B] holds one draw in [0, 1]
 * per row (the caller's generator), ids_host[B] receives the sampled ids,
 * logits_host as in dsb_decode_step.  No counterpart in the reference, whose
 * sampler runs on the host over downloaded logits (sampler.cpp:23-77). */
DSB_API int dsb_decode_step_sampled(dsb_ctx* ctx, dsb_model* model, dsb_kvcache* kv, const int32_t* seq_ids,
                                    const int32_t* tokens, int B, const dsb_sampling* sampling,
                                    const float* uniforms_host, float* logits_host, int32_t* ids_host);

/* dsb_generate with ds::rt::generate's sampling branch
 * (src/runtime/model.cpp:21-34): when temperature, top_k or top_p is above
 * 0 every generated id is sampled on the device, else greedy.  Sequence b
 * draws one uniform per generated id from its own std::mt19937 seeded with
 * seed + b through std::uniform_real_distribution<float>(0, 1), so for B = 1
 * the draws are the reference Sampler's own (sampler.cpp:21, 69-70). */
DSB_API int dsb_generate_sampled(dsb_ctx* ctx, dsb_model* model, dsb_kvcache* kv, const int32_t* seq_ids, int B,
                                 const int32_t* prompt_tokens, const int32_t* prompt_offsets, int max_new_tokens,
                                 int32_t eos_id, const dsb_sampling* sampling, int32_t* out_ids,
                                 int32_t* out_counts);

/* ------------------------------------------------------ checkpoint ingest */

/* A Hugging Face model directory opened on the host: config.json plus either
 * model.safetensors.index.json and the shards it names, or a single
 * model.safetensors.  Shards are memory-mapped read-only; no tensor bytes are
 * copied until dsb_model_upload_checkpoint.  Replaces the reference's loader
 * chain: load_model_dir (src/hf/model_loader.cpp:17-94),
 * load_safetensors_index (src/hf/weights_index.cpp:10-59),
 * load_safetensors_header (src/hf/safetensors.cpp:42-95) and
 * parse_deepseek_config (src/models/deepseek/config.cpp:9-52).  Beyond the
 * reference: the F8_E4M3 dtype (its parse_dtype, safetensors.cpp:12-20, has
 * none), the DeepSeek-V3 router fields of config.json, and checks that every
 * tensor's byte range fits its shard and matches its dtype and shape, and
 * that shard names stay inside the directory.  Host only: no GPU, no
 * context. */
typedef struct dsb_checkpoint dsb_checkpoint;

#define DSB_DTYPE_OTHER (-1) /* a safetensors dtype the model does not take (I64, BOOL, F8_E5M2, ...) */
#define DSB_CKPT_MAX_DIMS 8

typedef struct dsb_tensor_info {
  const char* name;       /* checkpoint name; valid until dsb_checkpoint_close */
  const char* dtype_name; /* the safetensors dtype string ("BF16", "F8_E4M3", ...) */
  int dtype;              /* DSB_DTYPE_* (F32, BF16, F16, F8E4M3) or DSB_DTYPE_OTHER */
  int ndim;
  int64_t shape[DSB_CKPT_MAX_DIMS];
  const void* data; /* the tensor's bytes inside the mapped shard (host memory) */
  uint64_t nbytes;
} dsb_tensor_info;

/* Open `dir`.  Fails with DSB_EINVAL (message from dsb_checkpoint_error) on a
 * missing or malformed file, DSB_EUNSUPPORTED on a config this build does not
 * run (a scoring_func other than softmax / sigmoid, FP8 blocks other than
 * 128 x 128). */
DSB_API int dsb_checkpoint_open(const char* dir, dsb_checkpoint** out);
DSB_API int dsb_checkpoint_close(dsb_checkpoint* ck);
/* The message of this thread's last failed dsb_checkpoint_* call. */
DSB_API const char* dsb_checkpoint_error(void);
/* config.json as a dsb_model_config, read the way parse_deepseek_config
 * reads it (same keys, aliases and defaults), except:
 *  - moe_intermediate_size is the key of that name; intermediate_size only
 *    when it is absent (the reference lets intermediate_size override it,
 *    config.cpp:35-36, and takes expert sizes from the weight shapes);
 *  - scoring_func "sigmoid" with n_group / topk_group (DeepSeek-V3); softmax
 *    routing is the plain top-k of the reference's moe_step (topk_method is
 *    not read, as in the reference);
 *  - weights_fp8 = 1 when quantization_config.quant_method is "fp8"
 *    (informational: FP8 layers are chosen by each tensor's dtype). */
DSB_API int dsb_checkpoint_config(const dsb_checkpoint* ck, dsb_model_config* out);
DSB_API int dsb_checkpoint_num_tensors(const dsb_checkpoint* ck, int* n);
/* Tensor i (0 <= i < n) in name order; dsb_checkpoint_find gives -1 in
 * *index for a name the checkpoint lacks. */
DSB_API int dsb_checkpoint_tensor(const dsb_checkpoint* ck, int i, dsb_tensor_info* out);
DSB_API int dsb_checkpoint_find(const dsb_checkpoint* ck, const char* name, int* index);
/* Upload every decode-path tensor of `ck` into `model` through
 * dsb_model_set_tensor (create the model from dsb_checkpoint_config and bind
 * it with dsb_model_set_ep first when expert-parallel; finalize afterwards).
 * Skipped, and counted in *n_skipped: tensors of layers at or beyond the
 * model's num_hidden_layers (DeepSeek-V3 ships its multi-token-prediction
 * module as layer 61, which decoding does not run) and rotary_emb.inv_freq
 * buffers.  Any other tensor the model does not know, or of a dtype it does
 * not take, fails the call with the tensor's name. */
DSB_API int dsb_model_upload_checkpoint(dsb_model* model, const dsb_checkpoint* ck, int* n_uploaded, int* n_skipped);

/* ---------------------------------------------------------------- tokenizer */

/* ds::rt::Tokenizer (src/runtime/tokenizer.cpp:1-171) on the host: the
 * reference's greedy longest-match encoder and trimming decoder over a
 * Hugging Face tokenizer.json (model.vocab, model.unk_token_id,
 * added_tokens, root bos/eos ids).  Same ids and text as the reference for
 * the same file, except that an added token's "special": true counts as
 * special (the reference reads JSON booleans as false) and ids must lie in
 * [0, 2^24).  Host only: no GPU, no context; messages from
 * dsb_tokenizer_error. */
typedef struct dsb_tokenizer dsb_tokenizer;

DSB_API int dsb_tokenizer_load(const char* path, dsb_tokenizer** out);
DSB_API int dsb_tokenizer_destroy(dsb_tokenizer* tok);
/* The message of this thread's last failed dsb_tokenizer_* call. */
DSB_API const char* dsb_tokenizer_error(void);
/* Number of ids (largest id + 1) and the bos / eos / unk ids (-1: none). */
DSB_API int dsb_tokenizer_info(const dsb_tokenizer* tok, int* n_ids, int32_t* bos_id, int32_t* eos_id,
                               int32_t* unk_id);
/* Tokenizer::encode (tokenizer.cpp:116-155) of text[0, len): *n_ids receives
 * the number of ids, written to ids[0, cap); a call with too small a buffer
 * (cap = 0 to ask) fails with DSB_EINVAL after setting *n_ids.  Text the
 * vocabulary cannot cover fails with DSB_EINVAL and the byte offset. */
DSB_API int dsb_tokenizer_encode(const dsb_tokenizer* tok, const char* text, size_t len, int32_t* ids, size_t cap,
                                 size_t* n_ids);
/* Tokenizer::decode (tokenizer.cpp:157-171): the pieces of ids[0, n),
 * trimmed, special ids left out when skip_special; *len receives the byte
 * count, written to out[0, cap) (NUL-terminated when there is room); too
 * small a buffer fails with DSB_EINVAL after setting *len. */
DSB_API int dsb_tokenizer_decode(const dsb_tokenizer* tok, const int32_t* ids, size_t n, int skip_special, char* out,
                                 size_t cap, size_t* len);

#ifdef __cplusplus
}
#endif

#endif /* DSB_DSB_H_ */
