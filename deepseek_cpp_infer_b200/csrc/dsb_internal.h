// Internal (non-ABI) declarations shared by the .cu files of libdsb.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "dsb/dsb.h"

struct dsb_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int sm_count = 0;
  int* d_status = nullptr;  // device status word written by bounded waits
  void* ws = nullptr;       // reusable device workspace
  size_t ws_bytes = 0;
  void* aux = nullptr;      // reusable device buffer for per-call plans
  size_t aux_bytes = 0;
  int* counters = nullptr;  // zeroed tickets for split-K reductions (kernels re-zero them)
  size_t n_counters = 0;
  std::string last_error;
  dsb_stats stats{};
};

namespace dsb {

// Record an error message on the context and return `code`.
int fail(dsb_ctx* ctx, int code, const char* fmt, ...);

// Check a CUDA runtime call; on failure record it and return DSB_ECUDA.
#define DSB_CUDA_TRY(ctx, call)                                                                     \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess) return ::dsb::fail((ctx), DSB_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// Ensure ctx->ws holds at least `bytes`; grows (never shrinks) the buffer.
int ensure_workspace(dsb_ctx* ctx, size_t bytes);
// Same for ctx->aux (small per-call metadata such as work lists).
int ensure_aux(dsb_ctx* ctx, size_t bytes);
// Ensure ctx->counters holds at least n zeroed ints.
int ensure_counters(dsb_ctx* ctx, size_t n);

// 2D bf16/u8/f32 tiled tensor map over a row-major matrix [rows, cols] with
// row pitch `pitch_bytes`; box = box_cols x box_rows; swizzle per CU enum.
int make_tmap_2d(dsb_ctx* ctx, CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols,
                 uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle);

}  // namespace dsb
