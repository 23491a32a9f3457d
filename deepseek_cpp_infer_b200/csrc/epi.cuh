// Vectorised output of one warp's block of a GEMM tile (shared by the bf16
// and FP8 GEMM epilogues).
//
// The accumulator arrives from TMEM with one weight row per lane and the
// tokens along the registers, while the output is token-major (y[t, col]).
// Writing it directly takes one 2- or 4-byte store per lane and token, and a
// warp's stores are then limited by the number of requests in flight, not by
// bytes (about 3 us for a 32 x 32 block).  Here the block is transposed
// through a warp-private 32 x 32 fp32 staging area in shared memory and
// leaves as 16-byte vectors along the output rows: 4 (f32) or 8 (bf16)
// columns per store, 4-8x fewer requests.

#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace dsb {

__device__ __forceinline__ void red_add_v4(float* p, float4 v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// One warp writes NTOK (<= 32) token rows of its output columns.
//   v[OFF+i] this lane's value for token row tok0 + i (i < NTOK).
//           With HALF (the SiLU gate|up epilogue) only even lanes carry
//           values, for output column col0 + lane/2 (16 columns); otherwise
//           column col0 + lane (32).
//   tcount  token rows to write (those from tok0 + tcount on are skipped).
//   ncols   output columns to write (a multiple of the vector width; the
//           rest lie beyond the matrix).
//   add     reduce into y (fp32) instead of storing: each element receives
//           exactly one add, so the result is y + v rounded once.
// Requirements (checked by the host): y 16-byte aligned; ldy, col0 and ncols
// multiples of the vector width (4 for f32, 8 for bf16).
template <int NTOK, bool HALF, int OFF = 0, int N>
__device__ __forceinline__ void warp_store_block(float* stg, const float (&v)[N], uint32_t lane, int tcount,
                                                 int ncols, void* y, int64_t ldy, int64_t col0, int64_t tok0,
                                                 int y_f32, bool add) {
  static_assert(NTOK <= 32 && OFF + NTOK <= N, "token rows per block");
  __syncwarp();  // the previous block's reads of stg are done
#pragma unroll
  for (int i = 0; i < NTOK; ++i) {
    if (!HALF) stg[i * 32 + lane] = v[OFF + i];
    else if ((lane & 1) == 0) stg[i * 32 + (lane >> 1)] = v[OFF + i];
  }
  __syncwarp();
  constexpr int COLS = HALF ? 16 : 32;
  if (y_f32) {
    constexpr int NV = COLS / 4;  // float4 vectors per token row
#pragma unroll 1
    for (int k = 0; k < (NTOK * NV + 31) / 32; ++k) {
      const int idx = k * 32 + (int)lane, t = idx / NV, q = idx % NV;
      if (idx < NTOK * NV && t < tcount && q * 4 < ncols) {
        const float4 a = *reinterpret_cast<const float4*>(stg + t * 32 + q * 4);
        float* dst = static_cast<float*>(y) + (tok0 + t) * ldy + col0 + q * 4;
        if (add) red_add_v4(dst, a);
        else *reinterpret_cast<float4*>(dst) = a;
      }
    }
  } else {
    constexpr int NV = COLS / 8;  // 8 x bf16 vectors per token row
#pragma unroll 1
    for (int k = 0; k < (NTOK * NV + 31) / 32; ++k) {
      const int idx = k * 32 + (int)lane, t = idx / NV, q = idx % NV;
      if (idx < NTOK * NV && t < tcount && q * 8 < ncols) {
        const float4 a = *reinterpret_cast<const float4*>(stg + t * 32 + q * 8);
        const float4 b = *reinterpret_cast<const float4*>(stg + t * 32 + q * 8 + 4);
        __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                               __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(y) + (tok0 + t) * ldy + col0 + q * 8) =
            *reinterpret_cast<const uint4*>(h);
      }
    }
  }
}

// The alignment the vector path needs, checked on the host: y 16-byte
// aligned, and ldy, the group column offset and the output width multiples
// of the vector width.
inline bool vec_out_ok(const void* y, int y_f32, int64_t ldy, int64_t y_group_col, int64_t out_cols) {
  const int64_t vw = y_f32 ? 4 : 8;
  return ((uintptr_t)y % 16) == 0 && ldy % vw == 0 && y_group_col % vw == 0 && out_cols % vw == 0;
}

}  // namespace dsb
