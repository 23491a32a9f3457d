// One MoE layer's expert FFN in block-scaled FP8 (dsb_moe_ffn_fp8):
//   picks [T, k] (+ n_shared always-on groups) -> stable permutation by expert
//   -> gather + 1x128 quantisation of x -> gate|up grouped FP8 GEMM with the
//   SiLU epilogue -> 1x128 quantisation of the bf16 product -> down grouped FP8
//   GEMM scaling each row by its routing weight -> combine in moe_step order.
// Every stage is a kernel on the context stream; nothing leaves the device.
// Follows moe_step (src/models/deepseek/ops.cpp:110-146) with the expert loop
// of moe_to_slot (src/models/deepseek/cuda_backend.cpp:836-883) replaced.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

namespace dsb {
namespace {

// ids/weights [T, k] -> [T, k + ns] with groups E .. E+ns-1 at weight 1 appended.
__global__ void append_shared_kernel(const int32_t* __restrict__ ids, const float* __restrict__ weights, int T, int k,
                                     int E, int ns, int32_t* __restrict__ ids_out, float* __restrict__ w_out) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int kk = k + ns;
  for (int j = 0; j < k; ++j) {
    ids_out[(int64_t)t * kk + j] = ids[(int64_t)t * k + j];
    w_out[(int64_t)t * kk + j] = weights[(int64_t)t * k + j];
  }
  for (int s = 0; s < ns; ++s) {
    ids_out[(int64_t)t * kk + k + s] = E + s;
    w_out[(int64_t)t * kk + k + s] = 1.0f;
  }
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace
}  // namespace dsb

extern "C" int dsb_moe_ffn_fp8(dsb_ctx* ctx, const dsb_moe_fp8_layer* w, const void* x, int64_t ldx, int T, int k,
                               const int32_t* ids, const float* weights, float* h) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (w == nullptr || w->gate_up == nullptr || w->gate_up_scale == nullptr || w->down == nullptr ||
      w->down_scale == nullptr || x == nullptr || ids == nullptr || weights == nullptr || h == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_moe_ffn_fp8: null argument");
  const int E = w->E, ns = w->n_shared, D = w->D, I = w->I;
  if (T <= 0 || k <= 0 || E <= 0 || ns < 0 || E + ns > 4096 || D <= 0 || I <= 0 || (D % 128) || (I % 128) ||
      ldx < D || (ldx % 8))
    return fail(ctx, DSB_EINVAL, "dsb_moe_ffn_fp8: bad sizes (D, I multiples of 128)");
  const int kk = k + ns, G = E + ns;
  const int64_t N = (int64_t)T * kk;
  if (N > INT32_MAX / 2) return fail(ctx, DSB_EINVAL, "dsb_moe_ffn_fp8: too many token rows");

  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align256(bytes);
    return o;
  };
  const size_t o_ids = take(N * 4), o_w = take(N * 4), o_cnt = take((size_t)(G + 1) * 4),
               o_off = take((size_t)(G + 2) * 4), o_dest = take(N * 4), o_src = take(N * 4), o_wp = take(N * 4),
               o_xq = take(N * D), o_sx = take(N * (D / 128) * 4), o_mid = take(N * I * 2), o_mq = take(N * I),
               o_msx = take(N * (I / 128) * 4), o_y = take(N * D * 4);
  int rc = ensure_buffer(ctx, &ctx->moe, &ctx->moe_bytes, off, (size_t)1 << 20, "moe scratch");
  if (rc != DSB_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(ctx->moe);
  auto I32 = [&](size_t o) { return reinterpret_cast<int32_t*>(base + o); };
  auto F32 = [&](size_t o) { return reinterpret_cast<float*>(base + o); };
  int32_t *ids_x = I32(o_ids), *cnt = I32(o_cnt), *offs = I32(o_off), *dest = I32(o_dest), *src = I32(o_src);
  float *w_x = F32(o_w), *wperm = F32(o_wp), *sx = F32(o_sx), *msx = F32(o_msx), *y = F32(o_y);

  launch_pdl(append_shared_kernel, (T + 127) / 128, 128, 0, ctx->stream, ids, weights, T, k, E, ns, ids_x, w_x);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches++;
  rc = moe_permute(ctx, ids_x, (int)N, G, cnt, offs, dest, src, w_x, wperm);
  if (rc != DSB_OK) return rc;
  rc = quant_act_1x128(ctx, x, DSB_DTYPE_BF16, ldx, src, kk, (int)N, D, base + o_xq, D, sx, D / 128);
  if (rc != DSB_OK) return rc;

  // tokens per routed expert ~ T*k/E (the shared groups see all T, in several token tiles)
  const int hint = std::max(16, std::min(128, 2 * (int)(((int64_t)T * k + E - 1) / E)));
  dsb_linear_fp8_args a{};
  a.w = w->gate_up;
  a.ldw = D;
  a.w_scale = w->gate_up_scale;
  a.scale_rows = 2;
  a.x = base + o_xq;
  a.ldx = D;
  a.x_scale = sx;
  a.ld_xs = D / 128;
  a.tok_offsets = offs;
  a.T = (int)N;
  a.M = 2 * I;
  a.K = D;
  a.G = G;
  a.max_tokens_per_group = hint;
  a.y = base + o_mid;
  a.ldy = I;
  a.y_f32 = 0;
  a.epilogue = DSB_EPI_SILU_GATE;
  rc = dsb_linear_fp8(ctx, &a);
  if (rc != DSB_OK) return rc;
  rc = quant_act_1x128(ctx, base + o_mid, DSB_DTYPE_BF16, I, nullptr, 1, (int)N, I, base + o_mq, I, msx, I / 128);
  if (rc != DSB_OK) return rc;

  dsb_linear_fp8_args b{};
  b.w = w->down;
  b.ldw = I;
  b.w_scale = w->down_scale;
  b.scale_rows = 1;
  b.x = base + o_mq;
  b.ldx = I;
  b.x_scale = msx;
  b.ld_xs = I / 128;
  b.tok_offsets = offs;
  b.T = (int)N;
  b.M = D;
  b.K = I;
  b.G = G;
  b.max_tokens_per_group = hint;
  b.y = y;
  b.ldy = D;
  b.y_f32 = 1;
  b.epilogue = DSB_EPI_ROWSCALE;
  b.row_scale = wperm;
  rc = dsb_linear_fp8(ctx, &b);
  if (rc != DSB_OK) return rc;
  return moe_combine(ctx, y, dest, T, kk, D, nullptr, h);
}
