// e4m3 quantisation in the DeepSeek-V3 block-scaled layout: per token and 128
// columns for activations, per 128x128 block for weights.  scale = amax / 448
// (correctly rounded fp32 division; 1 for an all-zero group), q = e4m3(x /
// scale) with round-to-nearest-even and saturation at +-448 (the
// cvt.rn.satfinite conversion).  HBM-bound byte work: one warp per 128-column
// group of a row, four elements per lane, 4-byte stores.
//
// No counterpart in the reference (it has no FP8 dtype:
// src/hf/safetensors.cpp:12-20).

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

namespace dsb {
namespace {

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <bool kBf16>
__global__ void quant_act_kernel(const void* __restrict__ x, int64_t ldx, const int32_t* __restrict__ src_rows,
                                 int k, int T, int G, uint8_t* __restrict__ q, int64_t ldq,
                                 float* __restrict__ scales, int64_t ld_scales) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)T * G) return;
  const int t = (int)(w / G), g = (int)(w % G);
  const int64_t srow = src_rows != nullptr ? src_rows[t] / k : t;
  const int64_t c0 = (int64_t)g * 128 + lane * 4;
  float v[4];
  if (kBf16) {
    const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x) + srow * ldx + c0);
    v[0] = __uint_as_float(raw.x << 16);
    v[1] = __uint_as_float(raw.x & 0xFFFF0000u);
    v[2] = __uint_as_float(raw.y << 16);
    v[3] = __uint_as_float(raw.y & 0xFFFF0000u);
  } else {
    const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + srow * ldx + c0);
    v[0] = f.x;
    v[1] = f.y;
    v[2] = f.z;
    v[3] = f.w;
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  const float s = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
  *reinterpret_cast<uint32_t*>(q + (int64_t)t * ldq + c0) =
      e4m3x4(__fdiv_rn(v[0], s), __fdiv_rn(v[1], s), __fdiv_rn(v[2], s), __fdiv_rn(v[3], s));
  if (lane == 0) scales[(int64_t)t * ld_scales + g] = s;
}

// One CTA per 128x128 block: amax over the block, then quantise.
template <bool kBf16>
__global__ void quant_weight_kernel(const void* __restrict__ w, int64_t M, int64_t K, uint8_t* __restrict__ q,
                                    float* __restrict__ scales) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int64_t r0 = (int64_t)blockIdx.y * 128, c0 = (int64_t)blockIdx.x * 128;
  auto load = [&](int64_t r, int64_t c) -> float {
    if (kBf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[r * K + c]);
    return static_cast<const float*>(w)[r * K + c];
  };
  float amax = 0.0f;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
    const int64_t r = r0 + i / 128, c = c0 + i % 128;
    if (r < M && c < K) amax = fmaxf(amax, fabsf(load(r, c)));
  }
  __shared__ float red[32];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    m = warp_max(m);
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  amax = red[0];
  const float s = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
  if (threadIdx.x == 0) scales[blockIdx.y * gridDim.x + blockIdx.x] = s;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
    const int64_t r = r0 + i / 128, c = c0 + i % 128;
    if (r < M && c < K)
      q[r * K + c] = (uint8_t)__nv_cvt_float_to_fp8(__fdiv_rn(load(r, c), s), __NV_SATFINITE, __NV_E4M3);
  }
}

}  // namespace

int quant_act_1x128(dsb_ctx* ctx, const void* x, int x_dtype, int64_t ldx, const int32_t* src_rows, int k, int T,
                    int K, void* q, int64_t ldq, float* scales, int64_t ld_scales) {
  const int G = K / 128;
  const int64_t warps = (int64_t)T * G;
  const int blocks = (int)((warps + 7) / 8);
  if (x_dtype == DSB_DTYPE_BF16)
    launch_pdl(quant_act_kernel<true>, blocks, 256, 0, ctx->stream, x, ldx, src_rows, k, T, G, static_cast<uint8_t*>(q), ldq,
                                                            scales, ld_scales);
  else
    launch_pdl(quant_act_kernel<false>, blocks, 256, 0, ctx->stream, x, ldx, src_rows, k, T, G, static_cast<uint8_t*>(q),
                                                             ldq, scales, ld_scales);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches++;
  return DSB_OK;
}

}  // namespace dsb

extern "C" int dsb_quant_act_1x128(dsb_ctx* ctx, const void* x, int x_dtype, int64_t ldx, const int32_t* src_rows,
                                   int k, int T, int K, void* q, int64_t ldq, float* scales, int64_t ld_scales) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (x == nullptr || q == nullptr || scales == nullptr || T <= 0 || K <= 0 || (K % 128) ||
      (x_dtype != DSB_DTYPE_BF16 && x_dtype != DSB_DTYPE_F32) || ldx < K || ldq < K || ld_scales < K / 128 ||
      (src_rows != nullptr && k <= 0))
    return fail(ctx, DSB_EINVAL, "dsb_quant_act_1x128: bad arguments (K a multiple of 128, ldx/ldq >= K)");
  if ((ldx % 4) || (ldq % 4) || (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(q) & 3u))
    return fail(ctx, DSB_EINVAL, "dsb_quant_act_1x128: rows must be 16-byte aligned (x) and 4-byte aligned (q)");
  return quant_act_1x128(ctx, x, x_dtype, ldx, src_rows, k, T, K, q, ldq, scales, ld_scales);
}

extern "C" int dsb_quant_weight_128x128(dsb_ctx* ctx, const void* w, int w_dtype, int64_t M, int64_t K, void* q,
                                        float* scales) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (w == nullptr || q == nullptr || scales == nullptr || M <= 0 || K <= 0 ||
      (w_dtype != DSB_DTYPE_BF16 && w_dtype != DSB_DTYPE_F32))
    return fail(ctx, DSB_EINVAL, "dsb_quant_weight_128x128: bad arguments");
  const dim3 grid((unsigned)((K + 127) / 128), (unsigned)((M + 127) / 128));
  if (grid.y > 65535) return fail(ctx, DSB_EINVAL, "dsb_quant_weight_128x128: too many rows");
  if (w_dtype == DSB_DTYPE_BF16)
    launch_pdl(quant_weight_kernel<true>, grid, 256, 0, ctx->stream, w, M, K, static_cast<uint8_t*>(q), scales);
  else
    launch_pdl(quant_weight_kernel<false>, grid, 256, 0, ctx->stream, w, M, K, static_cast<uint8_t*>(q), scales);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches++;
  return DSB_OK;
}
