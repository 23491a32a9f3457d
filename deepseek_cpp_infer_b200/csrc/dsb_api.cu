// Context management, error reporting and tensor-map encoding for libdsb.so.
// Replaces the singleton CudaContext of the reference
// (src/models/deepseek/cuda_backend.cpp:153-563) with per-device contexts.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <new>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

namespace dsb {

int fail(dsb_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx != nullptr) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return code;
}

// Grow (never shrink) one of the context's device buffers to `bytes`,
// doubling from `first`.  The old buffer may still be read by queued kernels,
// so the stream is drained before it is freed.
int ensure_buffer(dsb_ctx* ctx, void** buf, size_t* cap, size_t bytes, size_t first, const char* what) {
  if (bytes <= *cap) return DSB_OK;
  size_t grow = *cap ? *cap : first;
  while (grow < bytes) grow *= 2;
  if (*buf != nullptr) {
    DSB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    DSB_CUDA_TRY(ctx, cudaFree(*buf));
    *buf = nullptr;
    *cap = 0;
  }
  cudaError_t e = cudaMalloc(buf, grow);
  if (e != cudaSuccess) {
    *buf = nullptr;
    return fail(ctx, DSB_ENOMEM, "%s cudaMalloc(%zu): %s", what, grow, cudaGetErrorString(e));
  }
  *cap = grow;
  return DSB_OK;
}

int ensure_workspace(dsb_ctx* ctx, size_t bytes) {
  const int rc = ensure_buffer(ctx, &ctx->ws, &ctx->ws_bytes, bytes, (size_t)1 << 20, "workspace");
  ctx->stats.workspace_bytes = ctx->ws_bytes;
  return rc;
}

int ensure_aux(dsb_ctx* ctx, size_t bytes) {
  return ensure_buffer(ctx, &ctx->aux, &ctx->aux_bytes, bytes, (size_t)64 << 10, "aux");
}

int ensure_step(dsb_ctx* ctx, size_t bytes) {
  return ensure_buffer(ctx, &ctx->step, &ctx->step_bytes, bytes, (size_t)1 << 20, "step");
}

int ensure_counters(dsb_ctx* ctx, size_t n) {
  if (n <= ctx->n_counters) return DSB_OK;
  size_t grow = ctx->n_counters ? ctx->n_counters : 4096;
  while (grow < n) grow *= 2;
  if (ctx->counters != nullptr) {
    DSB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    DSB_CUDA_TRY(ctx, cudaFree(ctx->counters));
    ctx->counters = nullptr;
    ctx->n_counters = 0;
  }
  cudaError_t e = cudaMalloc(&ctx->counters, grow * sizeof(int));
  if (e != cudaSuccess) {
    ctx->counters = nullptr;
    return fail(ctx, DSB_ENOMEM, "counters cudaMalloc: %s", cudaGetErrorString(e));
  }
  DSB_CUDA_TRY(ctx, cudaMemsetAsync(ctx->counters, 0, grow * sizeof(int), ctx->stream));
  ctx->n_counters = grow;
  return DSB_OK;
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

size_t elem_size(CUtensorMapDataType t) {
  switch (t) {
    case CU_TENSOR_MAP_DATA_TYPE_UINT8: return 1;
    case CU_TENSOR_MAP_DATA_TYPE_BFLOAT16:
    case CU_TENSOR_MAP_DATA_TYPE_FLOAT16: return 2;
    case CU_TENSOR_MAP_DATA_TYPE_FLOAT32:
    case CU_TENSOR_MAP_DATA_TYPE_INT32: return 4;
    default: return 0;
  }
}

}  // namespace

int make_tmap_2d(dsb_ctx* ctx, CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols,
                 uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(ctx, DSB_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const size_t es = elem_size(dtype);
  if (es == 0 || (reinterpret_cast<uintptr_t>(base) & 15u) || (pitch_bytes & 15u) || (box_cols * es) % 16 != 0)
    return fail(ctx, DSB_EINVAL, "tensor map: base/pitch/box not 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, DSB_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSB_OK;
}

}  // namespace dsb

extern "C" {

int dsb_version(void) { return 100; }

int dsb_ctx_create(int device, dsb_ctx** out) {
  if (out == nullptr) return DSB_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return DSB_ECUDA;
  if (cudaSetDevice(device) != cudaSuccess) return DSB_ECUDA;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) return DSB_EUNSUPPORTED;  // kernels are built for sm_100a only
  auto* ctx = new (std::nothrow) dsb_ctx();
  if (ctx == nullptr) return DSB_ENOMEM;
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete ctx;
    return DSB_ECUDA;
  }
  ctx->own_stream = true;
  if (cudaMalloc(&ctx->d_status, sizeof(int)) != cudaSuccess ||
      cudaMemset(ctx->d_status, 0, sizeof(int)) != cudaSuccess) {
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return DSB_ENOMEM;
  }
  *out = ctx;
  return DSB_OK;
}

int dsb_ctx_destroy(dsb_ctx* ctx) {
  if (ctx == nullptr) return DSB_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->aux) cudaFree(ctx->aux);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->step) cudaFree(ctx->step);
  if (ctx->perm) cudaFree(ctx->perm);
  if (ctx->moe) cudaFree(ctx->moe);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return DSB_OK;
}

int dsb_ctx_set_stream(dsb_ctx* ctx, void* stream) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (stream == nullptr) {
    if (!ctx->own_stream) {
      cudaStream_t s;
      DSB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
      ctx->stream = s;
      ctx->own_stream = true;
    }
    return DSB_OK;
  }
  if (ctx->own_stream) {
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
  }
  ctx->stream = static_cast<cudaStream_t>(stream);
  ctx->own_stream = false;
  return DSB_OK;
}

void* dsb_ctx_stream(dsb_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

const char* dsb_last_error(const dsb_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int dsb_sync(dsb_ctx* ctx) {
  if (ctx == nullptr) return DSB_EINVAL;
  DSB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  DSB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  int st = 0;
  DSB_CUDA_TRY(ctx, cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st != 0) {
    DSB_CUDA_TRY(ctx, cudaMemset(ctx->d_status, 0, sizeof(int)));
    if (st == dsb::kStatusBadInput)
      return dsb::fail(ctx, DSB_EINVAL, "a kernel dropped an out-of-range index (device status %d)", st);
    return dsb::fail(ctx, DSB_ETIMEOUT, "a kernel's bounded wait ran out (device status %d)", st);
  }
  return DSB_OK;
}

int dsb_ctx_set_wait_limit(dsb_ctx* ctx, uint64_t limit_ns) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (limit_ns < 1000000ull || limit_ns > 60000000000ull)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_ctx_set_wait_limit: %llu ns outside [1 ms, 60 s]",
                     (unsigned long long)limit_ns);
  ctx->wait_limit_ns = limit_ns;
  return DSB_OK;
}

int dsb_get_stats(const dsb_ctx* ctx, dsb_stats* out) {
  if (ctx == nullptr || out == nullptr) return DSB_EINVAL;
  *out = ctx->stats;
  return DSB_OK;
}

int dsb_reset_stats(dsb_ctx* ctx) {
  if (ctx == nullptr) return DSB_EINVAL;
  const uint64_t ws = ctx->stats.workspace_bytes;
  ctx->stats = dsb_stats{};
  ctx->stats.workspace_bytes = ws;
  return DSB_OK;
}

}  // extern "C"
