// Row kernels' shared pieces: the block reduction and the MoE combine row
// (h += picks' outputs in order + shared outputs, then optionally the next
// RMSNorm of the row), used by the single-GPU combine (ops.cu) and by the
// expert-parallel combine (ep.cu) so both produce the same bits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace dsb {

__device__ __forceinline__ float rows_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum (blockDim.x a multiple of 32): warp sums, then the warps'
// partials added in warp order.  `red` is 32 floats of shared memory.
__device__ __forceinline__ float rows_block_sum(float v, float* red) {
  v = rows_warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r += red[i];
  return r;
}

__device__ __forceinline__ void add4(float4& a, const float4 b) {
  a.x = __fadd_rn(a.x, b.x);
  a.y = __fadd_rn(a.y, b.y);
  a.z = __fadd_rn(a.z, b.z);
  a.w = __fadd_rn(a.w, b.w);
}

// Threads per token row for combine_row: enough that a row's float4 columns
// go out in one step of two columns per thread (all of a row's loads in
// flight together), at least 64 and at most 1024, a multiple of 32.  The
// row's sum of squares is accumulated in this thread order, so every combine
// of the same D (single GPU or expert parallel) must use the same count.
__host__ __device__ inline int combine_threads(int D) {
  int n = ((D / 4) / 2 + 31) / 32 * 32;
  return n < 64 ? 64 : (n > 1024 ? 1024 : n);
}

// One token row of D (a multiple of 4), 16-byte vectors: acc = pick(0) + ...
// + pick(k-1) + shared_0 + ... (fp32, in that order), h += acc; with w_next,
// then xn = bf16(h * rsqrt(mean(h^2) + eps) * w_next).
template <class Pick>
__device__ __forceinline__ void combine_row(Pick pick, int k, int D, const float* __restrict__ shared, int n_shared,
                                            int64_t shared_stride, float* __restrict__ h, const float* __restrict__ w_next,
                                            float eps, __nv_bfloat16* __restrict__ xn, float* red) {
  const int D4 = D / 4;
  float ss = 0.0f;
  // two columns (i4 and i4 + blockDim.x) per step keep twice the row loads
  // in flight; every column's sum and the squares' order are unchanged
  const int stride = (int)blockDim.x;
  for (int i4 = threadIdx.x; i4 < D4; i4 += 2 * stride) {
    const int i4b = i4 + stride;
    const bool two = i4b < D4;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f), accb = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4
    for (int j = 0; j < k; ++j) {
      add4(acc, pick(j, i4));
      if (two) add4(accb, pick(j, i4b));
    }
    for (int s = 0; s < n_shared; ++s) {
      const float4* sh = reinterpret_cast<const float4*>(shared + s * shared_stride);
      add4(acc, sh[i4]);
      if (two) add4(accb, sh[i4b]);
    }
    float4 hv = reinterpret_cast<float4*>(h)[i4];
    add4(hv, acc);
    reinterpret_cast<float4*>(h)[i4] = hv;
    ss = __fadd_rn(ss, __fmul_rn(hv.x, hv.x));
    ss = __fadd_rn(ss, __fmul_rn(hv.y, hv.y));
    ss = __fadd_rn(ss, __fmul_rn(hv.z, hv.z));
    ss = __fadd_rn(ss, __fmul_rn(hv.w, hv.w));
    if (two) {
      float4 hb = reinterpret_cast<float4*>(h)[i4b];
      add4(hb, accb);
      reinterpret_cast<float4*>(h)[i4b] = hb;
      ss = __fadd_rn(ss, __fmul_rn(hb.x, hb.x));
      ss = __fadd_rn(ss, __fmul_rn(hb.y, hb.y));
      ss = __fadd_rn(ss, __fmul_rn(hb.z, hb.z));
      ss = __fadd_rn(ss, __fmul_rn(hb.w, hb.w));
    }
  }
  if (w_next == nullptr) return;
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(rows_block_sum(ss, red), (float)D), eps)));
  for (int i4 = threadIdx.x; i4 < D4; i4 += blockDim.x) {
    const float4 hv = reinterpret_cast<const float4*>(h)[i4];
    const float4 wv = reinterpret_cast<const float4*>(w_next)[i4];
    __nv_bfloat162 lo = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(hv.x, inv), wv.x), __fmul_rn(__fmul_rn(hv.y, inv), wv.y));
    __nv_bfloat162 hi = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(hv.z, inv), wv.z), __fmul_rn(__fmul_rn(hv.w, inv), wv.w));
    reinterpret_cast<__nv_bfloat162*>(xn)[2 * i4] = lo;
    reinterpret_cast<__nv_bfloat162*>(xn)[2 * i4 + 1] = hi;
  }
}

}  // namespace dsb
