// Internal (non-ABI) declarations shared by the .cu files of libdsb.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <new>
#include <stdexcept>
#include <string>

#include "dsb/dsb.h"

struct dsb_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int sm_count = 0;
  int* d_status = nullptr;  // device status word written by bounded waits
  uint64_t wait_limit_ns = 2000000000ull;  // bound of the expert-parallel flag waits
  void* ws = nullptr;       // reusable device workspace
  size_t ws_bytes = 0;
  void* aux = nullptr;      // reusable device buffer for per-call plans
  size_t aux_bytes = 0;
  int* counters = nullptr;  // zeroed tickets for split-K reductions (kernels re-zero them)
  size_t n_counters = 0;
  void* step = nullptr;     // activations of dsb_decode_step
  size_t step_bytes = 0;
  void* perm = nullptr;     // per-chunk expert histograms of the multi-block permute
  size_t perm_bytes = 0;
  void* moe = nullptr;      // activations of dsb_moe_ffn_fp8
  size_t moe_bytes = 0;
  std::string last_error;
  dsb_stats stats{};
};

// A split-KV work plan of the MLA decode for one set of sequence lengths.
struct dsb_mla_plan {
  int B = 0, H = 0, R = 0, P = 0;
  int n_items = 0, n_combines = 0, n_partial = 0;
  int max_len = 0;
  void* d_items = nullptr;     // work items on the device
  void* d_combines = nullptr;  // split-sequence merge list on the device
  int device = 0;
};

namespace dsb {

// Split-K count for a small dense decode GEMM: `tiles` 128-row weight tiles
// of tile_bytes each over `sm` SMs, every split at least min_kb of the KB K
// blocks.  Time model per count s: the busiest CTA streams its waves of
// tile_bytes / s at the per-SM rate (75 GB/s, or the HBM rate shared by the
// busy SMs when that is lower), the fp32 partials (tiles * s * 128 * NT * 8
// bytes written and read back) move at the HBM rate, and s > 1 adds the
// split reduction's fixed latency (partial store, fence, ticket, two L2
// round trips: about 4 us measured on B200).  The fastest count wins.
inline int pick_splits(int tiles, int KB, int sm, int min_kb, double tile_bytes, int NT) {
  constexpr double kSmRate = 75e9, kHbmRate = 6.5e12, kReduceLatency = 4e-6;
  int best = 1;
  double best_t = 0.0;
  for (int s = 1; s <= 8; ++s) {
    if (s > 1 && KB / s < min_kb) break;
    const int units = tiles * s, waves = (units + sm - 1) / sm, active = units < sm ? units : sm;
    const double rate = kSmRate < kHbmRate / active ? kSmRate : kHbmRate / active;
    double t = waves * (tile_bytes / s) / rate;
    if (s > 1) t += (double)tiles * s * 128.0 * NT * 8.0 / kHbmRate + kReduceLatency;
    if (s == 1 || t < best_t) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

// Launch a kernel on `stream` with programmatic stream serialization: it may
// be scheduled while the previous kernel of the stream drains (the kernel
// calls pdl_wait() before reading that kernel's results).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// dsb_linear / dsb_linear_fp8; with offsets_ready (grouped launches whose
// token offsets were written before the previous kernel of the stream began)
// the unit table is built and the first weight stages are loaded before the
// wait on the previous kernel, as for a dense launch.
int linear_ex(dsb_ctx* ctx, const dsb_linear_args* a, bool offsets_ready);
int linear_fp8_ex(dsb_ctx* ctx, const dsb_linear_fp8_args* a, bool offsets_ready);

// Record an error message on the context and return `code`.
int fail(dsb_ctx* ctx, int code, const char* fmt, ...);

// The context and configuration a model was created with (for the host-side
// checkpoint reader, which uploads through dsb_model_set_tensor).
dsb_ctx* model_ctx(const dsb_model* m);
const dsb_model_config* model_config(const dsb_model* m);

// Run an entry point's body so that no C++ exception crosses the C ABI: host
// allocation failures become DSB_ENOMEM, anything else DSB_EINVAL, with the
// message recorded on ctx (when there is one).
template <class F>
int guarded(dsb_ctx* ctx, const char* fn, F&& body) {
  try {
    return body();
  } catch (const std::bad_alloc&) {
    return ctx ? fail(ctx, DSB_ENOMEM, "%s: out of host memory", fn) : DSB_ENOMEM;
  } catch (const std::exception& e) {
    return ctx ? fail(ctx, DSB_EINVAL, "%s: %s", fn, e.what()) : DSB_EINVAL;
  } catch (...) {
    return ctx ? fail(ctx, DSB_EINVAL, "%s: unexpected error", fn) : DSB_EINVAL;
  }
}

// Devices a process may drive; per-device one-time state is sized by it.
constexpr int kMaxDevices = 64;

// Raise `kernel`'s dynamic shared memory limit to `bytes` the first time it
// runs on ctx's device (the attribute belongs to the kernel in each device's
// context).  `done` is the caller's per-kernel flag array.
template <class Kernel>
int smem_attr_once(dsb_ctx* ctx, Kernel kernel, size_t bytes, std::atomic<bool> (&done)[kMaxDevices]) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices) return fail(ctx, DSB_EUNSUPPORTED, "device %d", ctx->device);
  if (!done[ctx->device].load(std::memory_order_acquire)) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return fail(ctx, DSB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done[ctx->device].store(true, std::memory_order_release);
  }
  return DSB_OK;
}

// Check a CUDA runtime call; on failure record it and return DSB_ECUDA.
#define DSB_CUDA_TRY(ctx, call)                                                                     \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess) return ::dsb::fail((ctx), DSB_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// Grow one of the context's device buffers (*buf, capacity *cap) to `bytes`.
int ensure_buffer(dsb_ctx* ctx, void** buf, size_t* cap, size_t bytes, size_t first, const char* what);
// Ensure ctx->ws holds at least `bytes`; grows (never shrinks) the buffer.
int ensure_workspace(dsb_ctx* ctx, size_t bytes);
// Same for ctx->aux (small per-call metadata such as work lists).
int ensure_aux(dsb_ctx* ctx, size_t bytes);
// Same for ctx->step (decode-step activations).
int ensure_step(dsb_ctx* ctx, size_t bytes);
// Ensure ctx->counters holds at least n zeroed ints.  GEMM split tickets use
// [0, kTicketFront) (at most one per CTA of a launch), the fused MoE front's
// per-token tickets start at kTicketFront.
int ensure_counters(dsb_ctx* ctx, size_t n);
constexpr int kTicketFront = 1024;
// the routing kernel's ticket (expert-parallel count publication), after the
// fused front's per-token tickets (at most 4096 rows + 1)
constexpr int kTicketRoute = kTicketFront + 4096 + 2;

// 2D bf16/u8/f32 tiled tensor map over a row-major matrix [rows, cols] with
// row pitch `pitch_bytes`; box = box_cols x box_rows; swizzle per CU enum.
int make_tmap_2d(dsb_ctx* ctx, CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols,
                 uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle);

// Launchers shared by the C ABI entry points and the decode step (ops.cu).
int rmsnorm_rows(dsb_ctx* ctx, const float* x, int64_t ldx, const float* w, int rows, int n, float eps,
                 void* y_bf16, int64_t ldyb, float* y_f32, int64_t ldyf);
// kv_a rows of pitch ld_kv; the query either bf16 q [B, H*(nope+P)] or fp32 qf
// (row pitch ld_qf), whose nope parts are then also written to q_out as bf16.
int kv_norm_rope_append(dsb_ctx* ctx, const float* kv_a, int64_t ld_kv, const float* w_norm, const void* q,
                        const float* qf, int64_t ld_qf, void* q_out, const int32_t* pos, const int32_t* block_table,
                        int max_blocks, int B, int H, int nope, int R, int P, float eps, float theta, void* cache,
                        void* q_rope);
int router_logits(dsb_ctx* ctx, const float* x, const float* w, int T, int D, int E, float* logits);
// Sizes of an expert-parallel group (ep.cu); any output may be null.
int ep_params(const dsb_ep* ep, int* rank, int* world, int* n_experts, int* top_k, int* hidden, int* max_tokens,
              int* E_local);

// e4m3 per-token 1x128 quantisation (quant_fp8.cu); arguments as
// dsb_quant_act_1x128, unchecked.
int quant_act_1x128(dsb_ctx* ctx, const void* x, int x_dtype, int64_t ldx, const int32_t* src_rows, int k, int T,
                    int K, void* q, int64_t ldq, float* scales, int64_t ld_scales);
// n_extra > 0 appends groups E..E+n_extra-1 with weight 1 to every token's
// picks (the shared experts); ids/weights rows then hold k + n_extra entries.
// pub (expert parallel, may be NULL): the last CTA also writes the picks'
// slots and this rank's pick counts for the dispatch (ep_publish_args),
// which replaces ep_publish's own launch.
struct EpPublishArgs;
int moe_route(dsb_ctx* ctx, const float* logits, const float* bias, int T, int E, int k, int scoring, int n_group,
              int topk_group, int norm_topk, float routed_scale, int32_t* ids, float* weights, int n_extra,
              const EpPublishArgs* pub = nullptr);
int moe_permute(dsb_ctx* ctx, const int32_t* ids, int N, int E, int32_t* counts, int32_t* offsets, int32_t* dest,
                int32_t* src_pair, const float* weights, float* w_perm);
int gather_rows(dsb_ctx* ctx, const void* x, int64_t ldx, const int32_t* src_pair, int n_pairs, int k, int D,
                void* out);
// h[t] += sum of the row's picks (+ shared); with w_next, also writes the
// row's next RMSNorm (weights w_next) to xn_next as bf16.
int moe_combine(dsb_ctx* ctx, const float* y, const int32_t* dest, int T, int k, int D, const float* shared,
                float* h, const float* w_next = nullptr, float eps = 0.0f, void* xn_next = nullptr);
// Post-attention RMSNorm + router logits + routing (+ with `permute`, the
// permutation of moe_permute over E + n_extra groups) in one launch, for
// decode batches where moe_front_fits.  logits: [T, E] scratch.
bool moe_front_fits(int T, int D, int E, int N);
int moe_front(dsb_ctx* ctx, const float* h, const float* w_norm, int T, int D, float eps, const float* w_router,
              int E, const float* bias, int k, int scoring, int n_group, int topk_group, int norm_topk,
              float routed_scale, int n_extra, void* xn, float* logits, int32_t* ids, float* weights, int permute,
              int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* src_pair, float* w_perm,
              const EpPublishArgs* pub = nullptr);
// dsb_ep_dispatch in two parts, so that local work can run between them:
// ep_publish computes every pick's slot and this rank's pick counts (and
// starts the call's epoch); ep_send then copies the rows and the counts to
// their owners and, once every source's rows have arrived here, lays out the
// rows this rank received for the expert GEMMs.
int ep_publish(dsb_ep* ep, int T, const int32_t* ids);
// ep_publish's bookkeeping without its launch: the arguments with which a
// routing kernel (moe_front / moe_route) computes the slots and counts itself.
struct EpPublishArgs;
int ep_publish_args(dsb_ep* ep, int T, EpPublishArgs* out);
// With n_shared > 0 the receive side also copies this rank's T rows once per
// shared expert after the rows it receives (recv_offsets[E_local + j + 1] ends
// copy j), so one grouped GEMM over E_local + n_shared groups runs both.
int ep_send(dsb_ep* ep, const void* x, int64_t ldx, int T, const int32_t* ids, void** recv_x, int32_t** recv_offsets,
            int n_shared);
// dsb_ep_combine with the next RMSNorm fused as in moe_combine.
// shared_row0 (device, may be NULL): the shared outputs start at that row of `shared`.
int ep_combine(dsb_ep* ep, const float* y, int64_t ldy, int T, const float* weights, const float* shared,
               int n_shared, float* h, const float* w_next, float eps, void* xn_next, const int32_t* shared_row0);
int argmax_rows(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, int32_t* out);
// Sampled id per row (ds::core::Sampler::sample); uniforms[B] on the device.
int sample_rows(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, float temperature, int top_k, float top_p,
                const float* uniforms, int32_t* out);
int embed(dsb_ctx* ctx, const void* table, int bf16, const int32_t* tokens, int B, int D, float* h);

}  // namespace dsb
