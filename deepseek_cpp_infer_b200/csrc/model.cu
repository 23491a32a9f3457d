// Whole-model batched decode on one GPU: device weights registry, paged latent
// KV cache manager and the per-token decode step.
//
// Replaces the CUDA branch of DeepSeekModel::decode_next
// (src/models/deepseek/model.cpp:117-184), the slot-addressed executor of
// src/models/deepseek/cuda_backend.cpp (weight cache :402-457, MLA cache
// :81-88, per-op *_to_slot functions) and its per-MoE-layer host round trip
// (:854-860).  One step runs B sequences (one token each) through all layers
// with every intermediate on the device; the host only plans the split-KV
// work from the sequence lengths and reads back the greedy ids.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <random>
#include <vector>

#include "dsb_internal.h"
#include "ep_common.cuh"
#include "dsb_ptx.cuh"

struct dsb_model {
  struct Layer {
    bool moe = false;
    bool has_moe_tensors = false;
    float* in_norm = nullptr;
    float* post_norm = nullptr;
    __nv_bfloat16* w_q = nullptr;    // [H*(nope+P), D]        (no q-LoRA)
    __nv_bfloat16* w_qa = nullptr;   // [q_lora, D]            (q-LoRA)
    float* qa_norm = nullptr;        // [q_lora]
    __nv_bfloat16* w_qb = nullptr;   // [H*(nope+P), q_lora]
    __nv_bfloat16* w_kva = nullptr;  // [R+P, D]
    // w_q (or w_qa) and w_kva are row ranges of one buffer [Mq + R + P, D]
    // (Mq = H*(nope+P), or q_lora_rank), so one GEMM projects both from x
    __nv_bfloat16* w_qkv = nullptr;
    float* kva_norm = nullptr;       // [R]
    __nv_bfloat16* w_uk_t = nullptr; // [H*R, nope]   W_UK^T per head (from kv_b_proj)
    __nv_bfloat16* w_uv = nullptr;   // [H*v, R]      W_UV per head (from kv_b_proj)
    __nv_bfloat16* w_o = nullptr;    // [D, H*v]
    __nv_bfloat16* w_gu = nullptr;   // dense gate|up, rows interleaved (2f gate, 2f+1 up) [2I, D]
    __nv_bfloat16* w_down = nullptr; // [D, I]
    int inter = 0;
    float* w_router = nullptr;       // [E, D] fp32
    float* router_bias = nullptr;    // [E]
    // routed experts followed by the shared experts cut into expert-sized
    // groups: a shared MLP with intermediate n*I equals the sum of n MLPs of
    // intermediate I, so all of them run in one grouped GEMM
    __nv_bfloat16* e_gu = nullptr;   // [E + n_shared, 2I, D]
    __nv_bfloat16* e_down = nullptr; // [E + n_shared, D, I]
    int e_inter = 0;
    int n_shared = 0;                // shared groups after the routed experts
    uint8_t shared_seen = 0;         // bit 0 gate, 1 up, 2 down uploaded
    uint8_t seen_gate = 0, seen_up = 0;  // dense gate-up halves uploaded
    // Block-scaled FP8 variants (e4m3 bytes + fp32 scale per 128x128 block, in
    // the dsb_linear_fp8 layouts); a matrix runs in FP8 when its q8 is set.
    //   qkv8   [Mq + R + P, D], scales [ceil(rows/128)][D/128] (q|kv_a fused as w_qkv)
    //   qb8    [H*(nope+P), q_lora];  o8 [D, H*v];  down8 [D, I]
    //   gu8    [2I, D] rows interleaved, scales [2I/128][2][D/128] (scale_rows 2)
    //   e_gu8 / e_down8: per group (routed then shared) as gu8 / down8
    uint8_t *qkv8 = nullptr, *qb8 = nullptr, *o8 = nullptr, *gu8 = nullptr, *down8 = nullptr;
    uint8_t *e_gu8 = nullptr, *e_down8 = nullptr;
    float *qkv8_s = nullptr, *qb8_s = nullptr, *o8_s = nullptr, *gu8_s = nullptr, *down8_s = nullptr;
    float *e_gu8_s = nullptr, *e_down8_s = nullptr;
    std::vector<float> gu8_s_host, e_gu8_s_host;  // fused gate|up scales, assembled on the host
    std::vector<uint8_t> kvb8;                    // FP8 kv_b_proj waiting for its scales (or the reverse)
    std::vector<float> kvb8_s;
    int64_t fp8_weights = 0, fp8_scales = 0;      // FP8 weight / scale tensors received
  };
  dsb_ctx* ctx = nullptr;
  dsb_model_config cfg{};
  std::vector<Layer> layers;
  void* embed = nullptr;
  int embed_bf16 = 1;
  float* final_norm = nullptr;
  __nv_bfloat16* lm_head = nullptr;
  std::vector<void*> allocs;
  bool finalized = false;
  uint64_t weight_bytes = 0;
  // expert parallelism: this rank holds routed experts [e_first, e_first + E_own)
  dsb_ep* ep = nullptr;
  int e_first = 0, E_own = 0;
};

struct dsb_kvcache {
  dsb_ctx* ctx = nullptr;
  int n_layers = 0, R = 0, P = 0;
  int64_t n_blocks = 0;
  int max_seqs = 0, max_blocks_per_seq = 0;
  __nv_bfloat16* pool = nullptr;  // [n_layers][n_blocks][64][R+P]
  std::vector<int32_t> free_pages;
  std::vector<std::vector<int32_t>> seq_pages;
  std::vector<int32_t> seq_len;
  std::vector<uint8_t> seq_live;
};

namespace dsb {
namespace {

using bf16 = __nv_bfloat16;

float host_to_f32(const void* src, int dtype, int64_t i) {
  switch (dtype) {
    case DSB_DTYPE_F32: return static_cast<const float*>(src)[i];
    case DSB_DTYPE_BF16: {
      uint32_t u = static_cast<uint32_t>(static_cast<const uint16_t*>(src)[i]) << 16;
      float f;
      std::memcpy(&f, &u, 4);
      return f;
    }
    default: {
      __half h;
      std::memcpy(&h, static_cast<const uint16_t*>(src) + i, 2);
      return __half2float(h);
    }
  }
}

uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

std::vector<uint16_t> to_bf16(const void* src, int dtype, int64_t n) {
  std::vector<uint16_t> out(static_cast<size_t>(n));
  if (dtype == DSB_DTYPE_BF16) {
    std::memcpy(out.data(), src, static_cast<size_t>(n) * 2);
  } else {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16_bits(host_to_f32(src, dtype, i));
  }
  return out;
}

std::vector<float> to_f32(const void* src, int dtype, int64_t n) {
  std::vector<float> out(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i) out[i] = host_to_f32(src, dtype, i);
  return out;
}

// e4m3 (1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no infinities,
// S.1111.111 = NaN) to float, by its bit definition.
float e4m3_to_f32(uint8_t v) {
  const int e = (v >> 3) & 0xF, mant = v & 7;
  float mag;
  if (e == 0xF && mant == 7) return NAN;
  if (e == 0) mag = std::ldexp((float)mant, -9);
  else mag = std::ldexp(1.0f + mant / 8.0f, e - 7);
  return (v & 0x80) ? -mag : mag;
}

template <class T>
int dev_alloc(dsb_model* m, T** p, size_t count) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, count * sizeof(T));
  if (e != cudaSuccess) return fail(m->ctx, DSB_ENOMEM, "model cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(e));
  m->allocs.push_back(v);
  m->weight_bytes += count * sizeof(T);
  *p = static_cast<T*>(v);
  return DSB_OK;
}

template <class T>
int upload(dsb_model* m, T** p, const void* host, size_t count) {
  if (*p == nullptr) {
    int rc = dev_alloc(m, p, count);
    if (rc != DSB_OK) return rc;
  }
  DSB_CUDA_TRY(m->ctx, cudaMemcpy(*p, host, count * sizeof(T), cudaMemcpyHostToDevice));
  return DSB_OK;
}

// Row f of a gate (half 0) or up (half 1) projection [I, D] goes to row
// 2f + half of the fused [2I, D] matrix, so an output feature's gate and up
// rows sit in adjacent TMEM lanes (the SiLU-gate epilogue of dsb_linear pairs
// lanes 2j and 2j+1 with a warp shuffle).
int upload_gate_up_half(dsb_model* m, bf16* dst, const std::vector<uint16_t>& src, int I, int D, int half) {
  if (I % 64 != 0) return fail(m->ctx, DSB_EUNSUPPORTED, "intermediate size %d is not a multiple of 64", I);
  const size_t row = static_cast<size_t>(D) * 2;
  DSB_CUDA_TRY(m->ctx, cudaMemcpy2D(reinterpret_cast<uint8_t*>(dst) + half * row, 2 * row, src.data(), row, row, I,
                                    cudaMemcpyHostToDevice));
  return DSB_OK;
}

// Decimal digits [i, j) of s as an int; false past 9 digits (no exception
// can leave the C ABI on a malformed name).
bool parse_index(const std::string& s, size_t i, size_t j, int* out) {
  if (j == i || j - i > 9) return false;
  int v = 0;
  for (size_t k = i; k < j; ++k) v = v * 10 + (s[k] - '0');
  *out = v;
  return true;
}

bool parse_layer(const std::string& name, int* layer, std::string* rest) {
  static const std::string pre = "model.layers.";
  if (name.compare(0, pre.size(), pre) != 0) return false;
  size_t i = pre.size(), j = i;
  while (j < name.size() && name[j] >= '0' && name[j] <= '9') ++j;
  if (j == i || j >= name.size() || name[j] != '.') return false;
  if (!parse_index(name, i, j, layer)) return false;
  *rest = name.substr(j + 1);
  return true;
}

bool parse_expert(const std::string& rest, int* e, std::string* proj) {
  static const std::string pre = "mlp.experts.";
  if (rest.compare(0, pre.size(), pre) != 0) return false;
  size_t i = pre.size(), j = i;
  while (j < rest.size() && rest[j] >= '0' && rest[j] <= '9') ++j;
  if (j == i || j >= rest.size() || rest[j] != '.') return false;
  if (!parse_index(rest, i, j, e)) return false;
  *proj = rest.substr(j + 1);
  return true;
}

int64_t numel(const int64_t* shape, int ndim) {
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= shape[i];
  return n;
}

// ----------------------------------------------------- synthetic random init

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

// N(0, std) bf16 values from a counter-based hash (Box-Muller on two 24-bit
// uniforms), so a multi-GB random model needs no host traffic.
__global__ void init_normal_bf16_kernel(bf16* p, int64_t n, uint64_t seed, float stddev) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(seed * 0x9e3779b97f4a7c15ull + (uint64_t)i);
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)((h >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
    p[i] = __float2bfloat16_rn(stddev * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
  }
}

__global__ void init_normal_f32_kernel(float* p, int64_t n, uint64_t seed, float stddev, float mean) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(seed * 0x9e3779b97f4a7c15ull + (uint64_t)i);
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)((h >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
    p[i] = mean + stddev * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  }
}

int rand_bf16(dsb_model* m, bf16** p, int64_t n, uint64_t seed, float stddev) {
  int rc = dev_alloc(m, p, (size_t)n);
  if (rc != DSB_OK) return rc;
  init_normal_bf16_kernel<<<1184, 256, 0, m->ctx->stream>>>(*p, n, seed, stddev);
  DSB_CUDA_TRY(m->ctx, cudaGetLastError());
  return DSB_OK;
}

int rand_f32(dsb_model* m, float** p, int64_t n, uint64_t seed, float stddev, float mean) {
  int rc = dev_alloc(m, p, (size_t)n);
  if (rc != DSB_OK) return rc;
  init_normal_f32_kernel<<<1184, 256, 0, m->ctx->stream>>>(*p, n, seed, stddev, mean);
  DSB_CUDA_TRY(m->ctx, cudaGetLastError());
  return DSB_OK;
}

// Scale rows of one half (0 gate, 1 up) of a row-interleaved gate|up matrix:
// tile j holds rows 64j..64j+63 of each half, i.e. scale row j/2 of that half.
__global__ void gate_up_scale_kernel(const float* __restrict__ src, int T2, int KB, int h, float* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T2 * KB) return;
  const int j = i / KB, kb = i % KB;
  dst[((size_t)j * 2 + h) * KB + kb] = src[(size_t)(j / 2) * KB + kb];
}

// FP8 random init: N(0, stddev) bf16 in `tmp`, quantised per 128x128 block
// into q / sc (the dsb_quant_weight_128x128 rule a checkpoint would carry).
int rand_fp8(dsb_model* m, uint8_t* q, float* sc, int64_t rows, int64_t cols, uint64_t seed, float stddev, bf16* tmp) {
  init_normal_bf16_kernel<<<1184, 256, 0, m->ctx->stream>>>(tmp, rows * cols, seed, stddev);
  DSB_CUDA_TRY(m->ctx, cudaGetLastError());
  return dsb_quant_weight_128x128(m->ctx, tmp, DSB_DTYPE_BF16, rows, cols, q, sc);
}

// Gate and up halves quantised separately (as checkpoint matrices), then
// interleaved by row with their scales arranged for scale_rows 2.
int rand_fp8_gate_up(dsb_model* m, uint8_t* q, float* sc, int64_t I, int64_t D, uint64_t seed, float stddev, bf16* tmp,
                     uint8_t* tmp8, float* tmps) {
  const int KB = (int)((D + 127) / 128), T2 = (int)(2 * I / 128);
  for (int h = 0; h < 2; ++h) {
    int rc = rand_fp8(m, tmp8, tmps, I, D, seed * 2 + h, stddev, tmp);
    if (rc != DSB_OK) return rc;
    DSB_CUDA_TRY(m->ctx, cudaMemcpy2DAsync(q + h * D, 2 * D, tmp8, D, D, I, cudaMemcpyDeviceToDevice, m->ctx->stream));
    gate_up_scale_kernel<<<(T2 * KB + 255) / 256, 256, 0, m->ctx->stream>>>(tmps, T2, KB, h, sc);
    DSB_CUDA_TRY(m->ctx, cudaGetLastError());
  }
  return DSB_OK;
}

// ------------------------------------------------------------- decode step

struct StepBuffers {
  float *h, *xn32, *kv_a, *qa, *logits_r, *wts, *w_perm, *y_perm, *s_out, *logits;
  bf16 *xn, *q, *q_rope, *q_lat, *o_lat, *attn, *mid, *x_perm, *mid_perm, *qa_n;
  int32_t *ids, *counts, *offsets, *dest, *src, *greedy, *tokens, *pos, *bt;
  void* items;
  size_t items_off_comb;
};

int linear(dsb_ctx* ctx, const void* w, int64_t ldw, const void* x, int64_t ldx, int T, int M, int K, void* y,
           int64_t ldy, int y_f32, int epi, int G = 1, int64_t xgc = 0, int64_t ygc = 0,
           const int32_t* tok_offsets = nullptr, int max_tok = 0, const float* row_scale = nullptr,
           bool offsets_ready = false) {
  dsb_linear_args a{};
  a.w = w;
  a.ldw = ldw;
  a.x = x;
  a.ldx = ldx;
  a.x_group_col = xgc;
  a.tok_offsets = tok_offsets;
  a.T = T;
  a.M = M;
  a.K = K;
  a.G = G;
  a.max_tokens_per_group = max_tok;
  a.y = y;
  a.ldy = ldy;
  a.y_group_col = ygc;
  a.y_f32 = y_f32;
  a.epilogue = epi;
  a.row_scale = row_scale;
  return linear_ex(ctx, &a, offsets_ready);
}

}  // namespace
}  // namespace dsb

using namespace dsb;

namespace {

// kv_b_proj [H*(nope+v), R] (bf16 bits): rows per head [nope rows of W_UK |
// v rows of W_UV] (mla.cpp:99-102), kept as per-head W_UK^T [R, nope] and W_UV.
int upload_kv_b(dsb_model* m, dsb_model::Layer& L, const std::vector<uint16_t>& b) {
  const dsb_model_config& c = m->cfg;
  const int H = c.num_attention_heads, R = c.kv_lora_rank, nope = c.qk_nope_head_dim, v = c.v_head_dim;
  std::vector<uint16_t> uk_t((size_t)H * R * nope), uv((size_t)H * v * R);
  for (int h = 0; h < H; ++h) {
    const uint16_t* base = b.data() + (size_t)h * (nope + v) * R;
    for (int i = 0; i < nope; ++i)
      for (int r = 0; r < R; ++r) uk_t[((size_t)h * R + r) * nope + i] = base[(size_t)i * R + r];
    std::memcpy(uv.data() + (size_t)h * v * R, base + (size_t)nope * R, (size_t)v * R * 2);
  }
  int rc = upload(m, &L.w_uk_t, uk_t.data(), uk_t.size());
  if (rc != DSB_OK) return rc;
  return upload(m, &L.w_uv, uv.data(), uv.size());
}

// Allocate a layer's stacked expert matrices: E routed + n_shared groups of
// moe_intermediate_size (from the config, so tensors may arrive in any order).
int ensure_experts(dsb_model* m, dsb_model::Layer& L) {
  if (L.e_gu != nullptr) return DSB_OK;
  const dsb_model_config& c = m->cfg;
  const int I = c.moe_intermediate_size, D = c.hidden_size;
  if (I <= 0 || I % 64 != 0) return fail(m->ctx, DSB_EUNSUPPORTED, "moe_intermediate_size %d must be a positive multiple of 64", I);
  L.e_inter = I;
  L.n_shared = std::max(0, c.n_shared_experts);
  const int G = m->E_own + L.n_shared;
  int rc = dev_alloc(m, &L.e_gu, (size_t)G * 2 * I * D);
  if (rc == DSB_OK) rc = dev_alloc(m, &L.e_down, (size_t)G * D * I);
  return rc;
}

int cdiv(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Storage of one FP8 matrix (G groups of rows x cols, 128x128 scale blocks;
// gate_up: rows interleaved from gate / up halves with scale_rows 2).
int ensure_fp8(dsb_model* m, uint8_t** q, float** sc, int64_t G, int64_t rows, int64_t cols, bool gate_up) {
  if (*q != nullptr) return DSB_OK;
  int rc = dev_alloc(m, q, (size_t)(G * rows * cols));
  const int64_t srows = gate_up ? (rows / 128) * 2 : cdiv(rows, 128);
  if (rc == DSB_OK) rc = dev_alloc(m, sc, (size_t)(G * srows * cdiv(cols, 128)));
  return rc;
}

// One tensor of a block-scaled FP8 checkpoint: an e4m3 weight (dtype
// DSB_DTYPE_F8E4M3) or its "<weight>_scale_inv" fp32 scales, routed to the
// layer's FP8 storage.  `base` is the weight's name within the layer.
int set_fp8(dsb_model* m, dsb_model::Layer& L, const std::string& base, bool is_scale, int dtype,
            const int64_t* shape, int ndim, const void* data, const char* cname) {
  dsb_ctx* ctx = m->ctx;
  const dsb_model_config& c = m->cfg;
  const int D = c.hidden_size, H = c.num_attention_heads, R = c.kv_lora_rank, P = c.qk_rope_head_dim;
  const int nope = c.qk_nope_head_dim, v = c.v_head_dim, QH = H * (nope + P);
  const int64_t Mq = c.q_lora_rank > 0 ? c.q_lora_rank : QH;
  if (ndim != 2) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s must be 2-D", cname);
  if (is_scale && dtype == DSB_DTYPE_F8E4M3)
    return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s must be a float tensor", cname);
  const int64_t n = shape[0] * shape[1];
  std::vector<float> sf;
  if (is_scale) sf = to_f32(data, dtype, n);
  const uint8_t* w8 = static_cast<const uint8_t*>(data);
  auto shape_is = [&](int64_t rows, int64_t cols) {
    return is_scale ? (shape[0] == cdiv(rows, 128) && shape[1] == cdiv(cols, 128)) : (shape[0] == rows && shape[1] == cols);
  };
  auto bad = [&]() { return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s has an unexpected shape", cname); };
  auto put = [&](void* dst, const void* src, size_t bytes) -> int {
    DSB_CUDA_TRY(ctx, cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return DSB_OK;
  };
  (is_scale ? L.fp8_scales : L.fp8_weights)++;
  // plain matrix (group g of G): weight rows, or its [rows/128][cols/128] scales
  auto plain = [&](uint8_t** q, float** sc, int64_t G, int64_t g, int64_t rows, int64_t cols) -> int {
    if (!shape_is(rows, cols)) return bad();
    int rc = ensure_fp8(m, q, sc, G, rows, cols, false);
    if (rc != DSB_OK) return rc;
    if (is_scale) return put(*sc + g * n, sf.data(), n * 4);
    return put(*q + g * rows * cols, w8, (size_t)n);
  };
  // half h (0 gate, 1 up) of a row-interleaved gate|up matrix (group g of G, I rows per half)
  auto gate_up = [&](uint8_t** q, float** sc, std::vector<float>& shadow, int64_t G, int64_t g, int64_t I, int h,
                     const float* sfp, const uint8_t* wp, int64_t src_row_pitch) -> int {
    if (I % 128) return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_set_tensor: FP8 intermediate size must be a multiple of 128");
    int rc = ensure_fp8(m, q, sc, G, 2 * I, D, true);
    if (rc != DSB_OK) return rc;
    const int64_t KB = cdiv(D, 128), T2 = 2 * I / 128;
    if (is_scale) {
      // tile j holds rows 64j..64j+63 of each half: scale row j/2 of that half
      if (shadow.empty()) shadow.assign((size_t)(G * T2 * 2 * KB), 0.0f);
      for (int64_t j = 0; j < T2; ++j)
        for (int64_t kb = 0; kb < KB; ++kb) shadow[((g * T2 + j) * 2 + h) * KB + kb] = sfp[(j / 2) * KB + kb];
      return put(*sc + g * T2 * 2 * KB, shadow.data() + g * T2 * 2 * KB, (size_t)(T2 * 2 * KB * 4));
    }
    DSB_CUDA_TRY(ctx, cudaMemcpy2D(*q + g * 2 * I * D + h * D, 2 * D, wp, src_row_pitch, D, I, cudaMemcpyHostToDevice));
    return DSB_OK;
  };
  if (base == "self_attn.q_proj.weight" || base == "self_attn.q_a_proj.weight" ||
      base == "self_attn.kv_a_proj_with_mqa.weight") {
    const bool kv = base == "self_attn.kv_a_proj_with_mqa.weight";
    const int64_t row0 = kv ? Mq : 0, rows = kv ? R + P : Mq;
    if (Mq % 128) return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_set_tensor: FP8 q rows must be a multiple of 128");
    if (!shape_is(rows, D)) return bad();
    int rc = ensure_fp8(m, &L.qkv8, &L.qkv8_s, 1, Mq + R + P, D, false);
    if (rc != DSB_OK) return rc;
    if (is_scale) return put(L.qkv8_s + (row0 / 128) * cdiv(D, 128), sf.data(), n * 4);
    return put(L.qkv8 + row0 * D, w8, (size_t)n);
  }
  if (base == "self_attn.q_b_proj.weight") return plain(&L.qb8, &L.qb8_s, 1, 0, QH, c.q_lora_rank);
  if (base == "self_attn.o_proj.weight") return plain(&L.o8, &L.o8_s, 1, 0, D, (int64_t)H * v);
  if (base == "self_attn.kv_b_proj.weight") {
    // absorbed attention keeps kv_b in bf16: dequantise once both halves are here
    const int64_t rows = (int64_t)H * (nope + v);
    if (!shape_is(rows, R)) return bad();
    if (is_scale) L.kvb8_s = sf;
    else L.kvb8.assign(w8, w8 + n);
    if (L.kvb8.empty() || L.kvb8_s.empty()) return DSB_OK;
    const int64_t KB = cdiv(R, 128);
    std::vector<uint16_t> b((size_t)(rows * R));
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t col = 0; col < R; ++col)
        b[r * R + col] = f32_to_bf16_bits(e4m3_to_f32(L.kvb8[r * R + col]) * L.kvb8_s[(r / 128) * KB + col / 128]);
    L.kvb8.clear();
    L.kvb8_s.clear();
    return upload_kv_b(m, L, b);
  }
  if (base == "mlp.gate_proj.weight" || base == "mlp.up_proj.weight") {
    const int64_t I = is_scale ? shape[0] * 128 : shape[0];
    if (is_scale ? shape[1] != cdiv(D, 128) : shape[1] != D) return bad();
    if (L.inter != 0 && L.inter != I) return bad();
    L.inter = (int)I;
    const int h = base == "mlp.up_proj.weight" ? 1 : 0;
    (h ? L.seen_up : L.seen_gate) |= 1;
    return gate_up(&L.gu8, &L.gu8_s, L.gu8_s_host, 1, 0, I, h, sf.data(), w8, D);
  }
  if (base == "mlp.down_proj.weight") {
    const int64_t I = is_scale ? shape[1] * 128 : shape[1];
    if (L.inter != 0 && L.inter != I) return bad();
    L.inter = (int)I;
    return plain(&L.down8, &L.down8_s, 1, 0, D, I);
  }
  const int I = c.moe_intermediate_size, E = c.n_routed_experts;
  const int ns = std::max(0, c.n_shared_experts), G = m->E_own + ns;
  static const std::string sp = "mlp.shared_experts.";
  int e = -1;
  std::string proj;
  const bool shared = base.compare(0, sp.size(), sp) == 0;
  if (shared || parse_expert(base, &e, &proj)) {
    if (shared) proj = base.substr(sp.size());
    const bool is_down = proj == "down_proj.weight";
    if (!is_down && proj != "gate_proj.weight" && proj != "up_proj.weight")
      return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: unknown tensor %s", cname);
    if (I % 128) return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_set_tensor: FP8 moe_intermediate_size must be a multiple of 128");
    L.has_moe_tensors = true;
    L.e_inter = I;
    L.n_shared = ns;
    if (!shared) {
      if (e < 0 || e >= E) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: expert index out of range in %s", cname);
      if (e < m->e_first || e >= m->e_first + m->E_own) {  // another rank's expert
        (is_scale ? L.fp8_scales : L.fp8_weights)--;
        return DSB_OK;
      }
      e -= m->e_first;
      if (is_down) return plain(&L.e_down8, &L.e_down8_s, G, e, D, I);
      return gate_up(&L.e_gu8, &L.e_gu8_s, L.e_gu8_s_host, G, e, I, proj == "up_proj.weight" ? 1 : 0, sf.data(), w8, D);
    }
    // shared experts [ns*I, D] / [D, ns*I] -> groups E_own .. E_own+ns-1
    if (ns <= 0) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s given but the config has no shared experts", cname);
    const int KBD = cdiv(D, 128), KBI = I / 128;
    if (is_down ? !shape_is(D, (int64_t)ns * I) : !shape_is((int64_t)ns * I, D)) return bad();
    L.shared_seen |= is_down ? 4 : (proj == "up_proj.weight" ? 2 : 1);
    for (int j = 0; j < ns; ++j) {
      const int g = m->E_own + j;
      int rc;
      if (is_down) {
        rc = ensure_fp8(m, &L.e_down8, &L.e_down8_s, G, D, I, false);
        if (rc != DSB_OK) return rc;
        if (is_scale) {
          DSB_CUDA_TRY(ctx, cudaMemcpy2D(L.e_down8_s + (int64_t)g * KBD * KBI, KBI * 4, sf.data() + (int64_t)j * KBI,
                                         (size_t)ns * KBI * 4, KBI * 4, KBD, cudaMemcpyHostToDevice));
        } else {
          DSB_CUDA_TRY(ctx, cudaMemcpy2D(L.e_down8 + (int64_t)g * D * I, I, w8 + (int64_t)j * I, (size_t)ns * I, I, D,
                                         cudaMemcpyHostToDevice));
        }
      } else {
        rc = gate_up(&L.e_gu8, &L.e_gu8_s, L.e_gu8_s_host, G, g, I, proj == "up_proj.weight" ? 1 : 0,
                     is_scale ? sf.data() + (int64_t)j * KBI * KBD : nullptr, is_scale ? nullptr : w8 + (int64_t)j * I * D,
                     D);
        if (rc != DSB_OK) return rc;
      }
    }
    return DSB_OK;
  }
  return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s cannot be FP8", cname);
}

}  // namespace

// ===================================================================== model

static int model_create_impl(dsb_ctx* ctx, const dsb_model_config* cfg, dsb_model** out) {
  if (ctx == nullptr || cfg == nullptr || out == nullptr) return DSB_EINVAL;
  *out = nullptr;
  const dsb_model_config& c = *cfg;
  if (c.hidden_size <= 0 || c.num_hidden_layers <= 0 || c.num_attention_heads <= 0 || c.vocab_size <= 0 ||
      c.kv_lora_rank <= 0 || c.qk_rope_head_dim <= 0 || c.v_head_dim <= 0 || c.qk_nope_head_dim <= 0)
    return fail(ctx, DSB_EINVAL, "dsb_model_create: missing required sizes");
  if (c.hidden_size % 64 || c.qk_nope_head_dim % 64 || c.kv_lora_rank % 64 || (c.num_attention_heads * c.v_head_dim) % 64)
    return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_create: hidden, nope, kv_lora_rank and heads*v must be multiples of 64");
  if (!((c.kv_lora_rank == 512 && c.qk_rope_head_dim == 64) || (c.kv_lora_rank == 128 && c.qk_rope_head_dim == 32)))
    return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_create: (kv_lora_rank, rope) must be (512, 64) or (128, 32)");
  if (c.num_attention_heads > 128) return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_create: at most 128 heads");
  if (c.n_routed_experts > 256 || c.num_experts_per_tok > 8)
    return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_create: at most 256 experts and top-8");
  auto* m = new dsb_model();
  m->ctx = ctx;
  m->cfg = c;
  m->E_own = std::max(0, c.n_routed_experts);
  m->layers.resize(c.num_hidden_layers);
  *out = m;
  return DSB_OK;
}

extern "C" int dsb_model_set_ep(dsb_model* m, dsb_ep* ep) {
  if (m == nullptr || ep == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = m->ctx;
  if (!m->allocs.empty() || m->finalized)
    return fail(ctx, DSB_EINVAL, "dsb_model_set_ep: call before any tensor is set");
  int rank = 0, world = 0, E = 0, k = 0, D = 0, T_max = 0, E_local = 0;
  ep_params(ep, &rank, &world, &E, &k, &D, &T_max, &E_local);
  const dsb_model_config& c = m->cfg;
  if (E != c.n_routed_experts || k != c.num_experts_per_tok || D != c.hidden_size)
    return fail(ctx, DSB_EINVAL, "dsb_model_set_ep: the group's experts, top-k or hidden size differ from the model's");
  m->ep = ep;
  m->e_first = rank * E_local;
  m->E_own = E_local;
  return DSB_OK;
}

extern "C" int dsb_model_destroy(dsb_model* m) {
  if (m == nullptr) return DSB_OK;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (void* p : m->allocs) cudaFree(p);
  delete m;
  return DSB_OK;
}

static int model_set_tensor_impl(dsb_model* m, const char* cname, int dtype, const int64_t* shape, int ndim,
                                    const void* data) {
  if (m == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = m->ctx;
  if (cname == nullptr || shape == nullptr || data == nullptr || ndim < 1 || ndim > 2 ||
      (dtype != DSB_DTYPE_F32 && dtype != DSB_DTYPE_BF16 && dtype != DSB_DTYPE_F16 && dtype != DSB_DTYPE_F8E4M3))
    return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: bad arguments");
  if (m->finalized) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: model already finalized");
  const dsb_model_config& c = m->cfg;
  const std::string name(cname);
  const int64_t n = numel(shape, ndim);
  const int D = c.hidden_size, H = c.num_attention_heads, R = c.kv_lora_rank, P = c.qk_rope_head_dim;
  const int nope = c.qk_nope_head_dim, v = c.v_head_dim;
  auto expect = [&](int64_t r0, int64_t r1) -> bool {
    return (ndim == 2 && shape[0] == r0 && shape[1] == r1) || (ndim == 1 && r1 == 0 && shape[0] == r0);
  };
  auto bad_shape = [&]() { return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s has an unexpected shape", cname); };

  if (name == "model.embed_tokens.weight") {
    if (!expect(c.vocab_size, D)) return bad_shape();
    if (dtype == DSB_DTYPE_F32) {
      m->embed_bf16 = 0;
      float* p = nullptr;
      int rc = upload(m, &p, data, (size_t)n);
      m->embed = p;
      return rc;
    }
    m->embed_bf16 = 1;
    auto b = to_bf16(data, dtype, n);
    bf16* p = nullptr;
    int rc = upload(m, &p, b.data(), (size_t)n);
    m->embed = p;
    return rc;
  }
  if (name == "model.norm.weight") {
    if (!expect(D, 0)) return bad_shape();
    auto f = to_f32(data, dtype, n);
    return upload(m, &m->final_norm, f.data(), (size_t)n);
  }
  if (name == "lm_head.weight") {
    if (!expect(c.vocab_size, D)) return bad_shape();
    auto b = to_bf16(data, dtype, n);
    return upload(m, &m->lm_head, b.data(), (size_t)n);
  }
  int li = -1;
  std::string rest;
  if (!parse_layer(name, &li, &rest) || li < 0 || li >= c.num_hidden_layers)
    return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: unknown tensor %s", cname);
  auto& L = m->layers[li];
  {
    static const std::string suffix = "_scale_inv";
    const bool is_scale = rest.size() > suffix.size() && rest.compare(rest.size() - suffix.size(), suffix.size(), suffix) == 0;
    if (is_scale || dtype == DSB_DTYPE_F8E4M3)
      return set_fp8(m, L, is_scale ? rest.substr(0, rest.size() - suffix.size()) : rest, is_scale, dtype, shape, ndim,
                     data, cname);
  }
  auto norm_f32 = [&](float** dst, int64_t len) -> int {
    if (!expect(len, 0)) return bad_shape();
    auto f = to_f32(data, dtype, n);
    return upload(m, dst, f.data(), (size_t)n);
  };
  auto mat_bf16 = [&](bf16** dst, int64_t r0, int64_t r1) -> int {
    if (!expect(r0, r1)) return bad_shape();
    auto b = to_bf16(data, dtype, n);
    return upload(m, dst, b.data(), (size_t)n);
  };
  // q (or q_a) and kv_a projections: row ranges of the layer's fused buffer
  const int64_t Mq = c.q_lora_rank > 0 ? c.q_lora_rank : (int64_t)H * (nope + P);
  auto qkv_rows = [&](int64_t row0, int64_t rows) -> int {
    if (!expect(rows, D)) return bad_shape();
    if (L.w_qkv == nullptr) {
      int rc = dev_alloc(m, &L.w_qkv, (size_t)(Mq + R + P) * D);
      if (rc != DSB_OK) return rc;
    }
    auto b = to_bf16(data, dtype, n);
    DSB_CUDA_TRY(ctx, cudaMemcpy(L.w_qkv + row0 * D, b.data(), b.size() * 2, cudaMemcpyHostToDevice));
    if (row0 == 0) (c.q_lora_rank > 0 ? L.w_qa : L.w_q) = L.w_qkv;
    else L.w_kva = L.w_qkv + Mq * D;
    return DSB_OK;
  };
  if (rest == "input_layernorm.weight") return norm_f32(&L.in_norm, D);
  if (rest == "post_attention_layernorm.weight") return norm_f32(&L.post_norm, D);
  if (rest == "self_attn.q_proj.weight") {
    if (c.q_lora_rank > 0) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: q_proj given but q_lora_rank > 0");
    return qkv_rows(0, (int64_t)H * (nope + P));
  }
  if (rest == "self_attn.q_a_proj.weight") {
    if (c.q_lora_rank <= 0) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: q_a_proj given but q_lora_rank = 0");
    return qkv_rows(0, c.q_lora_rank);
  }
  if (rest == "self_attn.q_a_layernorm.weight") return norm_f32(&L.qa_norm, c.q_lora_rank);
  if (rest == "self_attn.q_b_proj.weight") return mat_bf16(&L.w_qb, (int64_t)H * (nope + P), c.q_lora_rank);
  if (rest == "self_attn.kv_a_proj_with_mqa.weight") return qkv_rows(Mq, R + P);
  if (rest == "self_attn.kv_a_layernorm.weight") return norm_f32(&L.kva_norm, R);
  if (rest == "self_attn.o_proj.weight") return mat_bf16(&L.w_o, D, (int64_t)H * v);
  if (rest == "self_attn.kv_b_proj.weight") {
    if (!expect((int64_t)H * (nope + v), R)) return bad_shape();
    return upload_kv_b(m, L, to_bf16(data, dtype, n));
  }
  if (rest == "mlp.gate.weight") {
    if (ndim != 2 || shape[0] != c.n_routed_experts || shape[1] != D) return bad_shape();
    L.has_moe_tensors = true;
    auto f = to_f32(data, dtype, n);
    return upload(m, &L.w_router, f.data(), (size_t)n);
  }
  if (rest == "mlp.gate.e_score_correction_bias") {
    if (!expect(c.n_routed_experts, 0)) return bad_shape();
    auto f = to_f32(data, dtype, n);
    return upload(m, &L.router_bias, f.data(), (size_t)n);
  }
  {
    // shared experts [n*I, D] / [D, n*I] -> expert groups E .. E+n-1
    static const std::string sp = "mlp.shared_experts.";
    if (rest.compare(0, sp.size(), sp) == 0) {
      const std::string proj = rest.substr(sp.size());
      const bool is_down = proj == "down_proj.weight";
      if (!is_down && proj != "gate_proj.weight" && proj != "up_proj.weight")
        return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: unknown tensor %s", cname);
      if (c.n_routed_experts <= 0 || c.n_shared_experts <= 0)
        return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s given but the config has no shared experts", cname);
      int rc = ensure_experts(m, L);
      if (rc != DSB_OK) return rc;
      const int I = L.e_inter, ns = L.n_shared, E = m->E_own;
      if (ndim != 2 || (is_down ? (shape[0] != D || shape[1] != (int64_t)ns * I) : (shape[0] != (int64_t)ns * I || shape[1] != D)))
        return fail(ctx, DSB_EUNSUPPORTED, "dsb_model_set_tensor: %s must be n_shared_experts x moe_intermediate_size", cname);
      L.has_moe_tensors = true;
      auto b = to_bf16(data, dtype, n);
      for (int j = 0; j < ns; ++j) {
        if (is_down) {
          // columns [jI, (j+1)I) of [D, nI] -> group E+j's [D, I]
          DSB_CUDA_TRY(ctx, cudaMemcpy2D(L.e_down + (size_t)(E + j) * D * I, (size_t)I * 2, b.data() + (size_t)j * I,
                                         (size_t)ns * I * 2, (size_t)I * 2, D, cudaMemcpyHostToDevice));
        } else {
          std::vector<uint16_t> part(b.begin() + (size_t)j * I * D, b.begin() + (size_t)(j + 1) * I * D);
          rc = upload_gate_up_half(m, L.e_gu + (size_t)(E + j) * 2 * I * D, part, I, D, proj == "up_proj.weight" ? 1 : 0);
          if (rc != DSB_OK) return rc;
        }
      }
      L.shared_seen |= is_down ? 4 : (proj == "up_proj.weight" ? 2 : 1);
      return DSB_OK;
    }
  }
  // dense MLP: gate and up go to one row-interleaved matrix
  for (int half = 0; half < 2; ++half) {
    if (rest == (half ? "mlp.up_proj.weight" : "mlp.gate_proj.weight")) {
      if (ndim != 2 || shape[1] != D) return bad_shape();
      const int I = (int)shape[0];
      if (L.inter != 0 && L.inter != I) return bad_shape();
      L.inter = I;
      if (L.w_gu == nullptr) {
        int rc = dev_alloc(m, &L.w_gu, (size_t)2 * I * D);
        if (rc != DSB_OK) return rc;
      }
      auto b = to_bf16(data, dtype, n);
      (half ? L.seen_up : L.seen_gate) |= 1;
      return upload_gate_up_half(m, L.w_gu, b, I, D, half);
    }
  }
  if (rest == "mlp.down_proj.weight") {
    if (ndim != 2 || shape[0] != D) return bad_shape();
    const int I = (int)shape[1];
    if (L.inter != 0 && L.inter != I) return bad_shape();
    L.inter = I;
    auto b = to_bf16(data, dtype, n);
    return upload(m, &L.w_down, b.data(), (size_t)n);
  }
  int e = -1;
  std::string proj;
  if (parse_expert(rest, &e, &proj)) {
    const int E = c.n_routed_experts;
    if (e < 0 || e >= E) return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: expert index out of range in %s", cname);
    L.has_moe_tensors = true;
    // with expert parallelism another rank owns this expert: nothing to keep here
    if (e < m->e_first || e >= m->e_first + m->E_own) return DSB_OK;
    e -= m->e_first;
    const bool is_down = proj == "down_proj.weight";
    if (!is_down && proj != "gate_proj.weight" && proj != "up_proj.weight")
      return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: unknown tensor %s", cname);
    if (ndim != 2) return bad_shape();
    const int I = is_down ? (int)shape[1] : (int)shape[0];
    if ((is_down ? shape[0] : shape[1]) != D) return bad_shape();
    if (I != c.moe_intermediate_size)
      return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: %s does not match moe_intermediate_size", cname);
    int rc0 = ensure_experts(m, L);
    if (rc0 != DSB_OK) return rc0;
    auto b = to_bf16(data, dtype, n);
    if (is_down) {
      DSB_CUDA_TRY(ctx, cudaMemcpy(L.e_down + (size_t)e * D * I, b.data(), b.size() * 2, cudaMemcpyHostToDevice));
      return DSB_OK;
    }
    return upload_gate_up_half(m, L.e_gu + (size_t)e * 2 * I * D, b, I, D, proj == "up_proj.weight" ? 1 : 0);
  }
  return fail(ctx, DSB_EINVAL, "dsb_model_set_tensor: unknown tensor %s", cname);
}

extern "C" int dsb_model_init_random(dsb_model* m, uint64_t seed, float stddev) {
  if (m == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = m->ctx;
  if (m->finalized || !m->allocs.empty()) return fail(ctx, DSB_EINVAL, "dsb_model_init_random: model not empty");
  const dsb_model_config& c = m->cfg;
  const int D = c.hidden_size, H = c.num_attention_heads, R = c.kv_lora_rank, P = c.qk_rope_head_dim;
  const int nope = c.qk_nope_head_dim, v = c.v_head_dim, E = c.n_routed_experts;
  uint64_t s = seed * 1000003ull;
  int rc = DSB_OK;
  auto nb = [&](bf16** p, int64_t n) { if (rc == DSB_OK) rc = rand_bf16(m, p, n, ++s, stddev); };
  auto ones = [&](float** p, int64_t n) { if (rc == DSB_OK) rc = rand_f32(m, p, n, ++s, 0.0f, 1.0f); };
  m->embed_bf16 = 1;
  bf16* emb = nullptr;
  nb(&emb, (int64_t)c.vocab_size * D);
  m->embed = emb;
  ones(&m->final_norm, D);
  nb(&m->lm_head, (int64_t)c.vocab_size * D);
  const bool f8 = c.weights_fp8 != 0;
  // FP8: each matrix is drawn in bf16 into a scratch buffer and quantised from there
  bf16* tmp = nullptr;
  uint8_t* tmp8 = nullptr;
  float* tmps = nullptr;
  if (f8) {
    const int64_t Mq0 = c.q_lora_rank > 0 ? c.q_lora_rank : (int64_t)H * (nope + P);
    const int64_t I0 = std::max<int64_t>(c.intermediate_size, c.moe_intermediate_size);
    const int64_t mx = std::max({(Mq0 + R + P) * D, (int64_t)H * (nope + P) * std::max(c.q_lora_rank, 1),
                                 (int64_t)D * H * v, I0 * D});
    if (cudaMalloc(&tmp, mx * 2) != cudaSuccess || cudaMalloc(&tmp8, I0 * D) != cudaSuccess ||
        cudaMalloc(&tmps, ((I0 + 127) / 128) * ((D + 127) / 128) * 4) != cudaSuccess) {
      cudaFree(tmp);
      cudaFree(tmp8);
      return fail(ctx, DSB_ENOMEM, "dsb_model_init_random: FP8 scratch");
    }
  }
  auto f8mat = [&](uint8_t** q, float** sc, int64_t G, int64_t rows, int64_t cols) {
    if (rc != DSB_OK) return;
    rc = ensure_fp8(m, q, sc, G, rows, cols, false);
    const int64_t ss = ((rows + 127) / 128) * ((cols + 127) / 128);
    for (int64_t g = 0; g < G && rc == DSB_OK; ++g)
      rc = rand_fp8(m, *q + g * rows * cols, *sc + g * ss, rows, cols, ++s, stddev, tmp);
  };
  auto f8gu = [&](uint8_t** q, float** sc, int64_t G, int64_t I) {
    if (rc != DSB_OK) return;
    rc = ensure_fp8(m, q, sc, G, 2 * I, D, true);
    const int64_t ss = (2 * I / 128) * 2 * ((D + 127) / 128);
    for (int64_t g = 0; g < G && rc == DSB_OK; ++g)
      rc = rand_fp8_gate_up(m, *q + g * 2 * I * D, *sc + g * ss, I, D, ++s, stddev, tmp, tmp8, tmps);
  };
  for (int li = 0; li < c.num_hidden_layers && rc == DSB_OK; ++li) {
    auto& L = m->layers[li];
    ones(&L.in_norm, D);
    ones(&L.post_norm, D);
    const int64_t Mq = c.q_lora_rank > 0 ? c.q_lora_rank : (int64_t)H * (nope + P);
    if (f8) {
      f8mat(&L.qkv8, &L.qkv8_s, 1, Mq + R + P, D);
    } else {
      nb(&L.w_qkv, (Mq + R + P) * D);
      if (rc == DSB_OK) {
        (c.q_lora_rank > 0 ? L.w_qa : L.w_q) = L.w_qkv;
        L.w_kva = L.w_qkv + Mq * D;
      }
    }
    if (c.q_lora_rank > 0) {
      ones(&L.qa_norm, c.q_lora_rank);
      if (f8) f8mat(&L.qb8, &L.qb8_s, 1, (int64_t)H * (nope + P), c.q_lora_rank);
      else nb(&L.w_qb, (int64_t)H * (nope + P) * c.q_lora_rank);
    }
    ones(&L.kva_norm, R);
    nb(&L.w_uk_t, (int64_t)H * R * nope);
    nb(&L.w_uv, (int64_t)H * v * R);
    if (f8) f8mat(&L.o8, &L.o8_s, 1, D, (int64_t)H * v);
    else nb(&L.w_o, (int64_t)D * H * v);
    const bool moe = E > 0 && li >= c.first_k_dense_replace;
    if (!moe) {
      L.inter = c.intermediate_size;
      if (f8) {
        f8gu(&L.gu8, &L.gu8_s, 1, L.inter);
        f8mat(&L.down8, &L.down8_s, 1, D, L.inter);
      } else {
        nb(&L.w_gu, (int64_t)2 * L.inter * D);
        nb(&L.w_down, (int64_t)D * L.inter);
      }
    } else {
      L.has_moe_tensors = true;
      if (rc == DSB_OK) rc = rand_f32(m, &L.w_router, (int64_t)E * D, ++s, stddev, 0.0f);
      if (c.scoring_func == DSB_SCORE_SIGMOID && rc == DSB_OK) rc = rand_f32(m, &L.router_bias, E, ++s, 0.01f, 0.0f);
      L.e_inter = c.moe_intermediate_size;
      L.n_shared = std::max(0, c.n_shared_experts);
      L.shared_seen = 7;
      if (f8) {
        f8gu(&L.e_gu8, &L.e_gu8_s, m->E_own + L.n_shared, L.e_inter);
        f8mat(&L.e_down8, &L.e_down8_s, m->E_own + L.n_shared, D, L.e_inter);
      } else {
        nb(&L.e_gu, (int64_t)(m->E_own + L.n_shared) * 2 * L.e_inter * D);
        nb(&L.e_down, (int64_t)(m->E_own + L.n_shared) * D * L.e_inter);
      }
    }
  }
  if (f8) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    cudaFree(tmp8);
    cudaFree(tmps);
  }
  if (rc != DSB_OK) return rc;
  DSB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return dsb_model_finalize(m);
}

extern "C" int dsb_model_finalize(dsb_model* m) {
  if (m == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = m->ctx;
  const dsb_model_config& c = m->cfg;
  if (m->embed == nullptr || m->final_norm == nullptr || m->lm_head == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_model_finalize: embed_tokens, norm or lm_head missing");
  for (int li = 0; li < c.num_hidden_layers; ++li) {
    auto& L = m->layers[li];
    // dense vs MoE by the presence of routed experts (weights.cpp:89-96)
    L.moe = L.has_moe_tensors;
    const bool qkv = L.w_qkv != nullptr || L.qkv8 != nullptr;
    const bool q_ok = c.q_lora_rank > 0 ? (L.qa_norm != nullptr && (L.w_qb != nullptr || L.qb8 != nullptr)) : true;
    if (!L.in_norm || !L.post_norm || !qkv || !q_ok || !L.kva_norm || !L.w_uk_t || !(L.w_o || L.o8))
      return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d attention weights incomplete", li);
    if (L.fp8_weights != L.fp8_scales || !L.kvb8.empty() || !L.kvb8_s.empty())
      return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d has FP8 weights without their scales", li);
    if ((L.w_qkv != nullptr) == (L.qkv8 != nullptr) && L.w_qkv != nullptr)
      return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d mixes bf16 and FP8 q/kv_a projections", li);
    if (L.moe) {
      if (!L.w_router || !(L.e_gu || L.e_gu8) || !(L.e_down || L.e_down8) || c.n_routed_experts <= 0 ||
          c.num_experts_per_tok <= 0)
        return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d MoE weights incomplete", li);
      if (c.scoring_func == DSB_SCORE_SIGMOID && !L.router_bias)
        return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d needs e_score_correction_bias", li);
      if (L.n_shared > 0 && L.shared_seen != 7)
        return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d shared experts incomplete", li);
    } else if (!(L.w_gu || L.gu8) || !(L.w_down || L.down8)) {
      return fail(ctx, DSB_EINVAL, "dsb_model_finalize: layer %d dense MLP incomplete", li);
    }
  }
  m->finalized = true;
  return DSB_OK;
}

extern "C" int dsb_model_weight_bytes(const dsb_model* m, uint64_t* bytes) {
  if (m == nullptr || bytes == nullptr) return DSB_EINVAL;
  *bytes = m->weight_bytes;
  return DSB_OK;
}

// ================================================================= KV cache

static int kvcache_create_impl(dsb_ctx* ctx, const dsb_model* m, int64_t n_blocks, int max_seqs,
                                  int max_blocks_per_seq, dsb_kvcache** out) {
  if (ctx == nullptr || m == nullptr || out == nullptr) return DSB_EINVAL;
  *out = nullptr;
  if (n_blocks <= 0 || n_blocks > INT32_MAX || max_seqs <= 0 || max_blocks_per_seq <= 0)
    return fail(ctx, DSB_EINVAL, "dsb_kvcache_create: bad sizes");
  auto* kv = new dsb_kvcache();
  kv->ctx = ctx;
  kv->n_layers = m->cfg.num_hidden_layers;
  kv->R = m->cfg.kv_lora_rank;
  kv->P = m->cfg.qk_rope_head_dim;
  kv->n_blocks = n_blocks;
  kv->max_seqs = max_seqs;
  kv->max_blocks_per_seq = max_blocks_per_seq;
  const size_t bytes = (size_t)kv->n_layers * n_blocks * 64 * (kv->R + kv->P) * 2;
  cudaError_t e = cudaMalloc(&kv->pool, bytes);
  if (e != cudaSuccess) {
    delete kv;
    return fail(ctx, DSB_ENOMEM, "dsb_kvcache_create: %zu bytes: %s", bytes, cudaGetErrorString(e));
  }
  // zero-filled, so rows past a sequence's length are finite (MLACache::init zero-fills too, mla.cpp:21-22)
  e = cudaMemsetAsync(kv->pool, 0, bytes, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    cudaFree(kv->pool);
    delete kv;
    return fail(ctx, DSB_ECUDA, "dsb_kvcache_create: %s", cudaGetErrorString(e));
  }
  kv->free_pages.reserve((size_t)n_blocks);
  for (int64_t p = n_blocks - 1; p >= 0; --p) kv->free_pages.push_back((int32_t)p);
  kv->seq_pages.resize(max_seqs);
  kv->seq_len.assign(max_seqs, 0);
  kv->seq_live.assign(max_seqs, 0);
  *out = kv;
  return DSB_OK;
}

extern "C" int dsb_kvcache_destroy(dsb_kvcache* kv) {
  if (kv == nullptr) return DSB_OK;
  cudaSetDevice(kv->ctx->device);
  cudaStreamSynchronize(kv->ctx->stream);
  cudaFree(kv->pool);
  delete kv;
  return DSB_OK;
}

static int kvcache_alloc_seq_impl(dsb_kvcache* kv, int* seq_id) {
  if (kv == nullptr || seq_id == nullptr) return DSB_EINVAL;
  for (int s = 0; s < kv->max_seqs; ++s) {
    if (!kv->seq_live[s]) {
      kv->seq_live[s] = 1;
      kv->seq_len[s] = 0;
      kv->seq_pages[s].clear();
      *seq_id = s;
      return DSB_OK;
    }
  }
  return fail(kv->ctx, DSB_ENOMEM, "dsb_kvcache_alloc_seq: all %d sequence slots in use", kv->max_seqs);
}

extern "C" int dsb_kvcache_free_seq(dsb_kvcache* kv, int seq_id) {
  if (kv == nullptr) return DSB_EINVAL;
  if (seq_id < 0 || seq_id >= kv->max_seqs || !kv->seq_live[seq_id])
    return fail(kv->ctx, DSB_EINVAL, "dsb_kvcache_free_seq: %d is not a live sequence", seq_id);
  for (int32_t p : kv->seq_pages[seq_id]) kv->free_pages.push_back(p);
  kv->seq_pages[seq_id].clear();
  kv->seq_len[seq_id] = 0;
  kv->seq_live[seq_id] = 0;
  return DSB_OK;
}

extern "C" int dsb_kvcache_reset(dsb_kvcache* kv) {
  if (kv == nullptr) return DSB_EINVAL;
  for (int s = 0; s < kv->max_seqs; ++s)
    if (kv->seq_live[s]) dsb_kvcache_free_seq(kv, s);
  return DSB_OK;
}

extern "C" int dsb_kvcache_seq_len(const dsb_kvcache* kv, int seq_id, int* len) {
  if (kv == nullptr || len == nullptr || seq_id < 0 || seq_id >= kv->max_seqs || !kv->seq_live[seq_id])
    return DSB_EINVAL;
  *len = kv->seq_len[seq_id];
  return DSB_OK;
}

extern "C" int dsb_kvcache_free_blocks(const dsb_kvcache* kv, int64_t* n) {
  if (kv == nullptr || n == nullptr) return DSB_EINVAL;
  *n = (int64_t)kv->free_pages.size();
  return DSB_OK;
}

namespace dsb {
namespace {

// Rows [r0, r1) of each listed page, in every layer's pool, get N(0, stddev)
// bf16 values.  runs: int32 triples (page, r0, r1).
__global__ void kv_fill_kernel(bf16* __restrict__ pool, int64_t layer_stride, int row_elems,
                               const int32_t* __restrict__ runs, uint64_t seed, float stddev) {
  const int layer = blockIdx.y, run = blockIdx.x;
  const int32_t page = runs[3 * run], r0 = runs[3 * run + 1], r1 = runs[3 * run + 2];
  bf16* base = pool + (int64_t)layer * layer_stride + (int64_t)page * 64 * row_elems;
  const int64_t n = (int64_t)(r1 - r0) * row_elems;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t idx = (int64_t)r0 * row_elems + i;
    const uint64_t hsh = mix64((seed + layer * 0x1000193ull + (uint64_t)page * 0x9e3779b1ull) * 0x9e3779b97f4a7c15ull +
                               (uint64_t)idx);
    const float u1 = ((float)(hsh >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)((hsh >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
    base[idx] = __float2bfloat16_rn(stddev * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
  }
}

}  // namespace
}  // namespace dsb

// Append n_tokens synthetic positions to a sequence: pages as decode would
// take them, every layer's rows filled with N(0, stddev) latents (seeded).
static int kvcache_fill_random_impl(dsb_kvcache* kv, int seq_id, int n_tokens, uint64_t seed, float stddev) {
  if (kv == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = kv->ctx;
  if (seq_id < 0 || seq_id >= kv->max_seqs || !kv->seq_live[seq_id] || n_tokens < 0)
    return fail(ctx, DSB_EINVAL, "dsb_kvcache_fill_random: bad arguments");
  int pos = kv->seq_len[seq_id];
  if (pos + n_tokens > kv->max_blocks_per_seq * 64)
    return fail(ctx, DSB_EINVAL, "dsb_kvcache_fill_random: sequence %d would exceed its page limit", seq_id);
  std::vector<int32_t> runs;
  int left = n_tokens;
  while (left > 0) {
    if (pos % 64 == 0) {
      if (kv->free_pages.empty()) return fail(ctx, DSB_ENOMEM, "dsb_kvcache_fill_random: out of cache pages");
      kv->seq_pages[seq_id].push_back(kv->free_pages.back());
      kv->free_pages.pop_back();
    }
    const int r0 = pos % 64, r1 = std::min(64, r0 + left);
    runs.insert(runs.end(), {kv->seq_pages[seq_id].back(), r0, r1});
    left -= r1 - r0;
    pos += r1 - r0;
  }
  kv->seq_len[seq_id] = pos;
  if (runs.empty()) return DSB_OK;
  int32_t* d_runs = nullptr;
  DSB_CUDA_TRY(ctx, cudaMalloc(&d_runs, runs.size() * 4));
  DSB_CUDA_TRY(ctx, cudaMemcpy(d_runs, runs.data(), runs.size() * 4, cudaMemcpyHostToDevice));
  const int row_elems = kv->R + kv->P;
  const dim3 grid((unsigned)(runs.size() / 3), (unsigned)kv->n_layers);
  kv_fill_kernel<<<grid, 256, 0, ctx->stream>>>(kv->pool, kv->n_blocks * 64 * (int64_t)row_elems, row_elems, d_runs,
                                                seed * 0x2545f4914f6cdd1dull + (uint64_t)seq_id, stddev);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  cudaFree(d_runs);
  if (e != cudaSuccess) return fail(ctx, DSB_ECUDA, "dsb_kvcache_fill_random: %s", cudaGetErrorString(e));
  return DSB_OK;
}

// =============================================================== decode step

namespace dsb {
// defined in mla_decode.cu
int mla_plan_into_aux(dsb_ctx* ctx, const int32_t* seq_lens, int B, int H, int R, int P, dsb_mla_plan* plan);
}  // namespace dsb

namespace {

// FP8 linear of the decode step: x quantised per token and 128 columns into
// (xq, sx), then dsb_linear_fp8 (no group column offsets).
int lin8(dsb_ctx* ctx, const uint8_t* w, const float* ws, int scale_rows, const uint8_t* xq, const float* sx, int K,
         int T, int M, void* y, int64_t ldy, int y_f32, int epi, int G = 1, const int32_t* offs = nullptr,
         int max_tok = 0, const float* row_scale = nullptr, bool offsets_ready = false) {
  dsb_linear_fp8_args a{};
  a.w = w;
  a.ldw = K;
  a.w_scale = ws;
  a.scale_rows = scale_rows;
  a.x = xq;
  a.ldx = K;
  a.x_scale = sx;
  a.ld_xs = K / 128;
  a.tok_offsets = offs;
  a.T = T;
  a.M = M;
  a.K = K;
  a.G = G;
  a.max_tokens_per_group = max_tok;
  a.y = y;
  a.ldy = ldy;
  a.y_f32 = y_f32;
  a.epilogue = epi;
  a.row_scale = row_scale;
  return linear_fp8_ex(ctx, &a, offsets_ready);
}

}  // namespace

namespace {

constexpr int kPrefillMaxTokens = DSB_PREFILL_MAX_TOKENS;

// One pass of B token rows through every layer.  Decode (prefill = false):
// B distinct sequences, one token each; greedy ids (and logits) for every row.
// Prefill: a sequence may appear several times (its tokens in order, appended
// at consecutive positions; each attends to its cache up to its own
// position), and the lm_head runs only on the last row of each distinct
// sequence (in order of first appearance): *n_seq_out of them.
// With `samp`, the id of each lm_head row is sampled (dsb_sample) with the
// draw uniforms_host[row] instead of taken greedily.
int forward_tokens(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids, const int32_t* tokens,
                   int B, bool prefill, float* logits_host, int32_t* greedy_host, int* n_seq_out,
                   const dsb_sampling* samp = nullptr, const float* uniforms_host = nullptr) {
  const char* fn = prefill ? "dsb_prefill" : (samp ? "dsb_decode_step_sampled" : "dsb_decode_step");
  if (ctx == nullptr || m == nullptr || kv == nullptr) return DSB_EINVAL;
  if (!m->finalized) return fail(ctx, DSB_EINVAL, "%s: model not finalized", fn);
  if (seq_ids == nullptr || tokens == nullptr || greedy_host == nullptr || B <= 0 ||
      B > (prefill ? kPrefillMaxTokens : kv->max_seqs))
    return fail(ctx, DSB_EINVAL, "%s: bad arguments (B=%d)", fn, B);
  if (samp != nullptr) {
    if (prefill || uniforms_host == nullptr || !std::isfinite(samp->temperature) || !std::isfinite(samp->top_p))
      return fail(ctx, DSB_EINVAL, "%s: bad sampling arguments", fn);
    for (int b = 0; b < B; ++b)
      if (!(uniforms_host[b] >= 0.0f && uniforms_host[b] <= 1.0f))
        return fail(ctx, DSB_EINVAL, "%s: uniforms[%d] is not in [0, 1]", fn, b);
  }
  const dsb_model_config& c = m->cfg;
  const int D = c.hidden_size, H = c.num_attention_heads, R = c.kv_lora_rank, P = c.qk_rope_head_dim;
  const int nope = c.qk_nope_head_dim, v = c.v_head_dim, V = c.vocab_size, E = c.n_routed_experts;
  const int k = c.num_experts_per_tok, QH = H * (nope + P), MB = kv->max_blocks_per_seq;

  // ---- host: validate, append one position per token, build the step tables
  std::vector<int> seq_order;            // distinct sequences in order of first appearance
  std::vector<int> added(kv->max_seqs, 0), last_row(kv->max_seqs, -1);
  int need_pages = 0;
  for (int b = 0; b < B; ++b) {
    const int s = seq_ids[b];
    if (s < 0 || s >= kv->max_seqs || !kv->seq_live[s])
      return fail(ctx, DSB_EINVAL, "%s: seq_ids[%d]=%d is not a live sequence", fn, b, s);
    if (tokens[b] < 0 || tokens[b] >= V) return fail(ctx, DSB_EINVAL, "%s: token %d out of range", fn, tokens[b]);
    if (added[s] > 0 && !prefill) return fail(ctx, DSB_EINVAL, "dsb_decode_step: sequence %d appears twice", s);
    const int pos = kv->seq_len[s] + added[s];
    if (pos >= MB * 64) return fail(ctx, DSB_EINVAL, "%s: sequence %d is full (%d tokens)", fn, s, pos);
    if (added[s] == 0) seq_order.push_back(s);
    need_pages += (pos % 64 == 0) ? 1 : 0;
    ++added[s];
    last_row[s] = b;
  }
  if ((size_t)need_pages > kv->free_pages.size()) return fail(ctx, DSB_ENOMEM, "%s: out of cache pages", fn);
  const int n_seq = (int)seq_order.size();
  const int LM = prefill ? n_seq : B;  // rows through the lm_head
  const bool ep = m->ep != nullptr;
  int ep_cap = 0, ep_tmax = 0;
  if (ep) {
    int rk, wd, Eg, kg, Dg;
    ep_params(m->ep, &rk, &wd, &Eg, &kg, &Dg, &ep_tmax, nullptr);
    ep_cap = wd * ep_tmax * kg;
    if (B > ep_tmax) return fail(ctx, DSB_EINVAL, "%s: %d rows above the expert group's max_tokens %d", fn, B, ep_tmax);
  }
  // tokens | positions | block table | (prefill) the lm_head rows | (sampling) the draws
  const size_t o_draws = (size_t)B * (2 + MB) + (prefill ? n_seq : 0);
  std::vector<int32_t> host_i(o_draws + (samp ? (size_t)LM : 0), 0);
  if (prefill)
    for (int i = 0; i < n_seq; ++i) host_i[(size_t)B * (2 + MB) + i] = last_row[seq_order[i]];
  if (samp) std::memcpy(host_i.data() + o_draws, uniforms_host, (size_t)LM * 4);
  std::vector<int32_t> lens(B);
  for (int b = 0; b < B; ++b) {
    const int s = seq_ids[b];
    const int pos = kv->seq_len[s];
    if (pos % 64 == 0) {
      kv->seq_pages[s].push_back(kv->free_pages.back());
      kv->free_pages.pop_back();
    }
    kv->seq_len[s] = pos + 1;
    lens[b] = pos + 1;
    host_i[b] = tokens[b];
    host_i[B + b] = pos;
    const auto& pg = kv->seq_pages[s];
    std::memcpy(host_i.data() + 2 * B + (size_t)b * MB, pg.data(), pg.size() * 4);
  }

  // ---- device buffers for this batch size (in the context workspace after the plan)
  int max_I = 0, max_eI = 0, max_ns = 0;
  bool any_moe = false, any_qlora = false;
  for (auto& L : m->layers) {
    max_I = std::max(max_I, L.inter);
    max_eI = std::max(max_eI, L.e_inter);
    max_ns = std::max(max_ns, L.n_shared);
    any_moe |= L.moe;
    any_qlora |= L.w_qa != nullptr;
  }
  const int BK = any_moe ? B * (k + max_ns) : 1;
  // expert rows: permuted picks, or the expert group's receive rows followed by
  // this rank's rows once per shared group
  const int RX = std::max(BK, ep ? ep_cap + max_ns * B : 0);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const int Mq = c.q_lora_rank > 0 ? c.q_lora_rank : QH, LQKV = Mq + R + P;  // fused q|kv_a projection row
  const size_t o_h = take((size_t)B * D * 4), o_xn32 = take((size_t)B * D * 4), o_kva = take((size_t)B * LQKV * 4);
  const size_t o_qa = take(any_qlora ? (size_t)B * c.q_lora_rank * 4 : 4);
  const size_t o_qan = take(any_qlora ? (size_t)B * c.q_lora_rank * 2 : 4);
  const size_t o_lr = take((size_t)B * std::max(E, 1) * 4), o_wts = take((size_t)BK * 4 + 4);
  const size_t o_wperm = take((size_t)BK * 4), o_yperm = take((size_t)RX * D * 4);
  const size_t o_ys = take(ep ? (size_t)max_ns * B * D * 4 : 4);
  const size_t o_logits = take((size_t)LM * V * 4), o_xn = take((size_t)B * D * 2), o_q = take((size_t)B * QH * 2);
  const size_t o_xlm = take(prefill ? (size_t)n_seq * D * 2 : 4);  // (prefill) the lm_head rows of xn
  const size_t o_qrope = take((size_t)B * H * P * 2), o_qlat = take((size_t)B * H * R * 2);
  const size_t o_olat = take((size_t)B * H * R * 2), o_attn = take((size_t)B * H * v * 2);
  const size_t o_mid = take((size_t)B * std::max(max_I, 64) * 2);
  const size_t o_xperm = take((size_t)BK * D * 2), o_midp = take((size_t)RX * std::max(max_eI, 64) * 2);
  const size_t o_ids = take((size_t)BK * 4 + 4), o_cnt = take((size_t)(E + max_ns + 1) * 4);
  const size_t o_off = take((size_t)(E + max_ns + 2) * 4);
  const size_t o_dest = take((size_t)BK * 4), o_src = take((size_t)BK * 4), o_greedy = take((size_t)LM * 4);
  const size_t o_tab = take(host_i.size() * 4);
  // FP8 layers: activations quantised per token and 128 columns
  bool any_fp8 = false;
  for (auto& L : m->layers) any_fp8 |= L.qkv8 || L.qb8 || L.o8 || L.gu8 || L.e_gu8;
  const int64_t q8_rows = any_fp8 ? std::max<int64_t>(RX, B) : 0;
  const int64_t q8_cols = any_fp8 ? std::max({(int64_t)D, (int64_t)H * v, (int64_t)std::max(c.q_lora_rank, 128),
                                              (int64_t)max_I, (int64_t)max_eI}) : 0;
  const size_t o_xq8 = take((size_t)(q8_rows * q8_cols) + 16), o_sx8 = take((size_t)(q8_rows * (q8_cols / 128)) * 4 + 16);
  // the step buffers live in their own context-owned region (ctx->step); the
  // workspace ctx->ws stays free for split-K / split-KV partials
  int rc = ensure_step(ctx, off);
  if (rc != DSB_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(ctx->step);
  auto F = [&](size_t o) { return reinterpret_cast<float*>(base + o); };
  auto Bf = [&](size_t o) { return reinterpret_cast<bf16*>(base + o); };
  auto I32 = [&](size_t o) { return reinterpret_cast<int32_t*>(base + o); };
  float *h = F(o_h), *xn32 = F(o_xn32), *kva = F(o_kva), *qa = F(o_qa), *lr = F(o_lr), *wts = F(o_wts);
  float *wperm = F(o_wperm), *yperm = F(o_yperm), *logits = F(o_logits), *ys = F(o_ys);
  bf16 *xn = Bf(o_xn), *q = Bf(o_q), *qrope = Bf(o_qrope), *qlat = Bf(o_qlat), *olat = Bf(o_olat), *attn = Bf(o_attn);
  bf16 *mid = Bf(o_mid), *xperm = Bf(o_xperm), *midp = Bf(o_midp), *qan = Bf(o_qan);
  int32_t *ids = I32(o_ids), *cnt = I32(o_cnt), *offs = I32(o_off), *dest = I32(o_dest), *src = I32(o_src);
  int32_t *greedy = I32(o_greedy), *tab = I32(o_tab);
  uint8_t* xq8 = base + o_xq8;
  float* sx8 = F(o_sx8);
  // quantise `rows` bf16 rows of K (pitch ld; gathered through src / k when src is set) into xq8 / sx8
  auto q8 = [&](const void* x, int64_t ld, int rows, int K, const int32_t* src = nullptr, int k = 1) {
    return quant_act_1x128(ctx, x, DSB_DTYPE_BF16, ld, src, k, rows, K, xq8, K, sx8, K / 128);
  };
  const int32_t *d_tok = tab, *d_pos = tab + B, *d_bt = tab + 2 * B;
  const int32_t* d_lmrows = tab + (size_t)B * (2 + MB);  // (prefill) lm_head rows
  DSB_CUDA_TRY(ctx, cudaMemcpyAsync(tab, host_i.data(), host_i.size() * 4, cudaMemcpyHostToDevice, ctx->stream));

  dsb_mla_plan plan;
  rc = mla_plan_into_aux(ctx, lens.data(), B, H, R, P, &plan);
  if (rc != DSB_OK) return rc;

  const float scale = 1.0f / std::sqrt((float)(nope + P));  // mla.cpp:88
  const int64_t layer_stride = kv->n_blocks * 64 * (int64_t)(R + P);
#define DSB_STEP(call)          \
  do {                          \
    int rc_ = (call);           \
    if (rc_ != DSB_OK) return rc_; \
  } while (0)

  DSB_STEP(embed(ctx, m->embed, m->embed_bf16, d_tok, B, D, h));
  bool xn_ready = false;  // the previous MoE combine already wrote this layer's input norm into xn
  for (int li = 0; li < c.num_hidden_layers; ++li) {
    const auto& L = m->layers[li];
    bf16* cache = kv->pool + (int64_t)li * layer_stride;
    // the RMSNorm after this layer's MoE block: the next layer's input norm, or the final norm
    const float* next_norm = li + 1 < c.num_hidden_layers ? m->layers[li + 1].in_norm : m->final_norm;
    // post-attention norm, router, routing (and the permutation) in one launch
    // when the router is small enough to be read once per token from L2
    const bool fused_front = L.moe && moe_front_fits(B, D, E, B * (k + L.n_shared));
    // attention block (model.cpp:126-138)
    if (!xn_ready) DSB_STEP(rmsnorm_rows(ctx, h, D, L.in_norm, B, D, c.rms_norm_eps, xn, D, nullptr, 0));
    xn_ready = false;
    // one GEMM for [q | kv_a] (or [q_a | kv_a]) from x, fp32 rows of LQKV
    if (L.qkv8 != nullptr) {
      DSB_STEP(q8(xn, D, B, D));
      DSB_STEP(lin8(ctx, L.qkv8, L.qkv8_s, 1, xq8, sx8, D, B, LQKV, kva, LQKV, 1, DSB_EPI_STORE));
    } else {
      DSB_STEP(linear(ctx, L.w_qkv, D, xn, D, B, LQKV, D, kva, LQKV, 1, DSB_EPI_STORE));
    }
    if (c.q_lora_rank > 0) {
      DSB_STEP(rmsnorm_rows(ctx, kva, LQKV, L.qa_norm, B, c.q_lora_rank, c.rms_norm_eps, qan, c.q_lora_rank,
                            nullptr, 0));
      if (L.qb8 != nullptr) {
        DSB_STEP(q8(qan, c.q_lora_rank, B, c.q_lora_rank));
        DSB_STEP(lin8(ctx, L.qb8, L.qb8_s, 1, xq8, sx8, c.q_lora_rank, B, QH, q, QH, 0, DSB_EPI_STORE));
      } else {
        DSB_STEP(linear(ctx, L.w_qb, c.q_lora_rank, qan, c.q_lora_rank, B, QH, c.q_lora_rank, q, QH, 0,
                        DSB_EPI_STORE));
      }
      DSB_STEP(kv_norm_rope_append(ctx, kva + Mq, LQKV, L.kva_norm, q, nullptr, 0, nullptr, d_pos, d_bt, MB, B, H,
                                   nope, R, P, c.rms_norm_eps, c.rope_theta, cache, qrope));
    } else {
      // q comes as fp32 from the fused GEMM; the append also writes it as bf16 for the absorb GEMM
      DSB_STEP(kv_norm_rope_append(ctx, kva + Mq, LQKV, L.kva_norm, nullptr, kva, LQKV, q, d_pos, d_bt, MB, B, H,
                                   nope, R, P, c.rms_norm_eps, c.rope_theta, cache, qrope));
    }
    // q_lat[:, h] = W_UK[h]^T q_nope[:, h]
    DSB_STEP(linear(ctx, L.w_uk_t, nope, q, QH, B, R, nope, qlat, (int64_t)H * R, 0, DSB_EPI_STORE, H, nope + P, R));
    DSB_STEP(dsb_mla_decode_planned(ctx, &plan, qlat, qrope, cache, kv->n_blocks, d_bt, MB, scale, olat));
    // attn[:, h] = W_UV[h] o_lat[:, h], then h += o_proj(attn)
    DSB_STEP(linear(ctx, L.w_uv, R, olat, (int64_t)H * R, B, v, R, attn, (int64_t)H * v, 0, DSB_EPI_STORE, H, R, v));
    if (L.o8 != nullptr) {
      DSB_STEP(q8(attn, (int64_t)H * v, B, H * v));
      DSB_STEP(lin8(ctx, L.o8, L.o8_s, 1, xq8, sx8, H * v, B, D, h, D, 1, DSB_EPI_ADD));
    } else {
      DSB_STEP(linear(ctx, L.w_o, (int64_t)H * v, attn, (int64_t)H * v, B, D, H * v, h, D, 1, DSB_EPI_ADD));
    }
    // feed-forward block (model.cpp:140-157)
    if (!L.moe) {
      DSB_STEP(rmsnorm_rows(ctx, h, D, L.post_norm, B, D, c.rms_norm_eps, xn, D, nullptr, 0));
      if (L.gu8 != nullptr) {
        DSB_STEP(q8(xn, D, B, D));
        DSB_STEP(lin8(ctx, L.gu8, L.gu8_s, 2, xq8, sx8, D, B, 2 * L.inter, mid, L.inter, 0, DSB_EPI_SILU_GATE));
        DSB_STEP(q8(mid, L.inter, B, L.inter));
        DSB_STEP(lin8(ctx, L.down8, L.down8_s, 1, xq8, sx8, L.inter, B, D, h, D, 1, DSB_EPI_ADD));
      } else {
        DSB_STEP(linear(ctx, L.w_gu, D, xn, D, B, 2 * L.inter, D, mid, L.inter, 0, DSB_EPI_SILU_GATE));
        DSB_STEP(linear(ctx, L.w_down, L.inter, mid, L.inter, B, D, L.inter, h, D, 1, DSB_EPI_ADD));
      }
    } else if (ep) {
      // expert parallel: routed picks go to the experts' ranks and come back;
      // the shared experts run here on this rank's tokens.  The routing
      // kernel's last CTA publishes this rank's pick counts to every rank.
      EpPublishArgs pub;
      DSB_STEP(ep_publish_args(m->ep, B, &pub));
      if (fused_front) {
        DSB_STEP(moe_front(ctx, h, L.post_norm, B, D, c.rms_norm_eps, L.w_router, E, L.router_bias, k, c.scoring_func,
                           c.n_group, c.topk_group, c.norm_topk_prob, c.routed_scaling_factor, 0, xn, lr, ids, wts, 0,
                           nullptr, nullptr, nullptr, nullptr, nullptr, &pub));
      } else {
        DSB_STEP(rmsnorm_rows(ctx, h, D, L.post_norm, B, D, c.rms_norm_eps, xn, D, xn32, D));
        DSB_STEP(router_logits(ctx, xn32, L.w_router, B, D, E, lr));
        DSB_STEP(moe_route(ctx, lr, L.router_bias, B, E, k, c.scoring_func, c.n_group, c.topk_group,
                           c.norm_topk_prob, c.routed_scaling_factor, ids, wts, 0, &pub));
      }
      // the routed and the shared experts in one grouped GEMM pair: the
      // dispatch copies this rank's rows once per shared group after the rows
      // it receives (groups E_own .. E_own + ns - 1, this rank's tokens)
      const int eI = L.e_inter, EL = m->E_own, ns = L.n_shared;
      void* rx = nullptr;
      int32_t* roff = nullptr;
      DSB_STEP(ep_send(m->ep, xn, D, B, ids, &rx, &roff, ns));
      const int rows = ep_cap + ns * B;  // a bound: the groups' offsets hold the real rows
      // the receive kernel writes the offsets right before the bf16 gate|up GEMM;
      // every other expert GEMM here has a launch between (offsets_ready)
      if (L.e_gu8 != nullptr) {
        DSB_STEP(q8(rx, D, rows, D));
        DSB_STEP(lin8(ctx, L.e_gu8, L.e_gu8_s, 2, xq8, sx8, D, rows, 2 * eI, midp, eI, 0, DSB_EPI_SILU_GATE, EL + ns,
                      roff, B, nullptr, true));
        DSB_STEP(q8(midp, eI, rows, eI));
        DSB_STEP(lin8(ctx, L.e_down8, L.e_down8_s, 1, xq8, sx8, eI, rows, D, yperm, D, 1, DSB_EPI_STORE, EL + ns, roff,
                      B, nullptr, true));
      } else {
        DSB_STEP(linear(ctx, L.e_gu, D, rx, D, rows, 2 * eI, D, midp, eI, 0, DSB_EPI_SILU_GATE, EL + ns, 0, 0, roff,
                        B));
        DSB_STEP(linear(ctx, L.e_down, eI, midp, eI, rows, D, eI, yperm, D, 1, DSB_EPI_STORE, EL + ns, 0, 0, roff, B,
                        nullptr, true));
      }
      DSB_STEP(ep_combine(m->ep, yperm, D, B, wts, yperm, ns, h, next_norm, c.rms_norm_eps, xn, roff + EL));
      xn_ready = true;
    } else {
      // each token routes to its top-k experts plus every shared group (weight 1)
      const int kk = k + L.n_shared, G = E + L.n_shared;
      if (fused_front) {
        DSB_STEP(moe_front(ctx, h, L.post_norm, B, D, c.rms_norm_eps, L.w_router, E, L.router_bias, k, c.scoring_func,
                           c.n_group, c.topk_group, c.norm_topk_prob, c.routed_scaling_factor, L.n_shared, xn, lr, ids,
                           wts, 1, cnt, offs, dest, src, wperm));
      } else {
        DSB_STEP(rmsnorm_rows(ctx, h, D, L.post_norm, B, D, c.rms_norm_eps, xn, D, xn32, D));
        DSB_STEP(router_logits(ctx, xn32, L.w_router, B, D, E, lr));
        DSB_STEP(moe_route(ctx, lr, L.router_bias, B, E, k, c.scoring_func, c.n_group, c.topk_group,
                           c.norm_topk_prob, c.routed_scaling_factor, ids, wts, L.n_shared));
        DSB_STEP(moe_permute(ctx, ids, B * kk, G, cnt, offs, dest, src, wts, wperm));
      }
      // (the expert GEMMs' offsets come from the routing kernel, two or more
      // launches back: they may build their schedules before the wait)
      const int eI = L.e_inter;
      if (L.e_gu8 != nullptr) {
        // gather + quantise the permuted rows in one pass, then the FP8 expert GEMMs
        DSB_STEP(q8(xn, D, B * kk, D, src, kk));
        DSB_STEP(lin8(ctx, L.e_gu8, L.e_gu8_s, 2, xq8, sx8, D, B * kk, 2 * eI, midp, eI, 0, DSB_EPI_SILU_GATE, G, offs,
                      B, nullptr, true));
        DSB_STEP(q8(midp, eI, B * kk, eI));
        DSB_STEP(lin8(ctx, L.e_down8, L.e_down8_s, 1, xq8, sx8, eI, B * kk, D, yperm, D, 1, DSB_EPI_ROWSCALE, G, offs,
                      B, wperm, true));
      } else {
        DSB_STEP(gather_rows(ctx, xn, D, src, B * kk, kk, D, xperm));
        // every expert writes the same columns of its own (permuted) token rows
        DSB_STEP(linear(ctx, L.e_gu, D, xperm, D, B * kk, 2 * eI, D, midp, eI, 0, DSB_EPI_SILU_GATE, G, 0, 0, offs,
                        B, nullptr, true));
        DSB_STEP(linear(ctx, L.e_down, eI, midp, eI, B * kk, D, eI, yperm, D, 1, DSB_EPI_ROWSCALE, G, 0, 0, offs, B,
                        wperm, true));
      }
      DSB_STEP(moe_combine(ctx, yperm, dest, B, kk, D, nullptr, h, next_norm, c.rms_norm_eps, xn));
      xn_ready = true;
    }
  }
  // final norm, lm_head, greedy (model.cpp:160-179); a prefill keeps only each
  // sequence's last row
  if (!xn_ready) DSB_STEP(rmsnorm_rows(ctx, h, D, m->final_norm, B, D, c.rms_norm_eps, xn, D, nullptr, 0));
  const bf16* xlm = xn;
  if (prefill) {
    DSB_STEP(gather_rows(ctx, xn, D, d_lmrows, n_seq, 1, D, Bf(o_xlm)));
    xlm = Bf(o_xlm);
  }
  DSB_STEP(linear(ctx, m->lm_head, D, xlm, D, LM, V, D, logits, V, 1, DSB_EPI_STORE));
  if (samp != nullptr)
    DSB_STEP(sample_rows(ctx, logits, V, LM, V, samp->temperature, samp->top_k, samp->top_p,
                         reinterpret_cast<const float*>(tab + o_draws), greedy));
  else
    DSB_STEP(argmax_rows(ctx, logits, V, LM, V, greedy));
#undef DSB_STEP
  DSB_CUDA_TRY(ctx, cudaMemcpyAsync(greedy_host, greedy, (size_t)LM * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (logits_host != nullptr)
    DSB_CUDA_TRY(ctx, cudaMemcpyAsync(logits_host, logits, (size_t)LM * V * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (prefill) {
    ctx->stats.prefill_tokens += (uint64_t)B;
    if (n_seq_out != nullptr) *n_seq_out = n_seq;
  } else {
    ctx->stats.decode_steps++;
  }
  return dsb_sync(ctx);
}

}  // namespace

extern "C" int dsb_decode_step(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids,
                               const int32_t* tokens, int B, float* logits_host, int32_t* greedy_host) {
  return guarded(ctx, "dsb_decode_step", [&] {
    return forward_tokens(ctx, m, kv, seq_ids, tokens, B, false, logits_host, greedy_host, nullptr);
  });
}

extern "C" int dsb_decode_step_sampled(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids,
                                       const int32_t* tokens, int B, const dsb_sampling* sampling,
                                       const float* uniforms_host, float* logits_host, int32_t* ids_host) {
  if (ctx != nullptr && sampling == nullptr) return fail(ctx, DSB_EINVAL, "dsb_decode_step_sampled: no sampling config");
  return guarded(ctx, "dsb_decode_step_sampled", [&] {
    return forward_tokens(ctx, m, kv, seq_ids, tokens, B, false, logits_host, ids_host, nullptr, sampling,
                          uniforms_host);
  });
}

extern "C" int dsb_prefill(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids,
                           const int32_t* tokens, int n_tok, float* logits_host, int32_t* greedy_host, int* n_seq) {
  return guarded(ctx, "dsb_prefill", [&] {
    return forward_tokens(ctx, m, kv, seq_ids, tokens, n_tok, true, logits_host, greedy_host, n_seq);
  });
}

namespace {

// Batched generation on the host over the decode step: ds::rt::generate
// (src/runtime/model.cpp:14-49) for B sequences at once.  Each sequence first
// consumes its prompt token by token (DeepSeekModel::forward,
// src/models/deepseek/model.cpp:104-110), then feeds back its next id; it
// stops after max_new_tokens ids or at eos_id (>= 0; the eos id is kept, as
// the reference does).  Sequences with different prompt lengths are stepped
// together: each call decodes one token for every sequence still running.
// The next id is greedy unless `samp` asks for sampling (temperature, top_k
// or top_p above 0, model.cpp:32-34); then sequence b draws one uniform per
// generated id from its own std::mt19937 seeded with seed + b (seed 0:
// std::random_device), through a fresh std::uniform_real_distribution<float>,
// as the reference's Sampler draws (src/core/sampler.cpp:21, 69-70).
int generate(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids, int B,
             const int32_t* prompt_tokens, const int32_t* prompt_offsets, int max_new_tokens, int32_t eos_id,
             const dsb_sampling* samp, int32_t* out_ids, int32_t* out_counts, const char* fn) {
  if (ctx == nullptr || m == nullptr || kv == nullptr) return DSB_EINVAL;
  if (seq_ids == nullptr || prompt_tokens == nullptr || prompt_offsets == nullptr || out_ids == nullptr ||
      out_counts == nullptr || B <= 0 || max_new_tokens < 0)
    return fail(ctx, DSB_EINVAL, "%s: bad arguments", fn);
  if (m->ep != nullptr)
    return fail(ctx, DSB_EUNSUPPORTED, "%s: expert-parallel models step every rank together; drive "
                                       "dsb_decode_step directly", fn);
  const bool sampling = samp != nullptr && (samp->temperature > 0.0f || samp->top_k > 0 || samp->top_p > 0.0f);
  std::vector<std::mt19937> rng;
  if (sampling) {
    for (int b = 0; b < B; ++b) {
      if (samp->seed != 0) {
        rng.emplace_back(samp->seed + (uint32_t)b);
      } else {
        std::random_device rd;  // only for seed 0, as the reference's Sampler does
        rng.emplace_back(rd());
      }
    }
  }
  std::vector<float> draws;
  for (int b = 0; b < B; ++b) {
    out_counts[b] = 0;
    if (prompt_offsets[b + 1] - prompt_offsets[b] < 1)
      return fail(ctx, DSB_EINVAL, "%s: sequence %d has an empty prompt", fn, b);
  }
  if (max_new_tokens == 0) return DSB_OK;
  std::vector<int> fed(B, 0);           // prompt tokens consumed
  std::vector<int32_t> last(B, 0);      // last generated id
  std::vector<uint8_t> done(B, 0);
  std::vector<int32_t> ids, toks, greedy;
  std::vector<int> rows;
  for (;;) {
    ids.clear();
    toks.clear();
    rows.clear();
    for (int b = 0; b < B; ++b) {
      if (done[b]) continue;
      const int plen = prompt_offsets[b + 1] - prompt_offsets[b];
      ids.push_back(seq_ids[b]);
      toks.push_back(fed[b] < plen ? prompt_tokens[prompt_offsets[b] + fed[b]] : last[b]);
      rows.push_back(b);
    }
    if (rows.empty()) break;
    greedy.resize(rows.size());
    int rc;
    if (sampling) {
      // one draw for each row whose step yields a generated id (prompt rows keep theirs)
      draws.assign(rows.size(), 0.5f);
      for (size_t r = 0; r < rows.size(); ++r) {
        const int b = rows[r];
        if (fed[b] + 1 >= prompt_offsets[b + 1] - prompt_offsets[b]) {
          std::uniform_real_distribution<float> dist(0.0f, 1.0f);
          draws[r] = dist(rng[(size_t)b]);
        }
      }
      rc = forward_tokens(ctx, m, kv, ids.data(), toks.data(), (int)rows.size(), false, nullptr, greedy.data(),
                          nullptr, samp, draws.data());
    } else {
      rc = dsb_decode_step(ctx, m, kv, ids.data(), toks.data(), (int)rows.size(), nullptr, greedy.data());
    }
    if (rc != DSB_OK) return rc;
    for (size_t r = 0; r < rows.size(); ++r) {
      const int b = rows[r];
      const int plen = prompt_offsets[b + 1] - prompt_offsets[b];
      if (fed[b] < plen) ++fed[b];
      if (fed[b] < plen) continue;  // still inside the prompt
      const int32_t nxt = greedy[r];
      out_ids[(size_t)b * max_new_tokens + out_counts[b]] = nxt;
      last[b] = nxt;
      if (++out_counts[b] >= max_new_tokens || (eos_id >= 0 && nxt == eos_id)) done[b] = 1;
    }
  }
  return DSB_OK;
}

}  // namespace

extern "C" int dsb_generate(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids, int B,
                            const int32_t* prompt_tokens, const int32_t* prompt_offsets, int max_new_tokens,
                            int32_t eos_id, int32_t* out_ids, int32_t* out_counts) {
  return guarded(ctx, "dsb_generate", [&] {
    return generate(ctx, m, kv, seq_ids, B, prompt_tokens, prompt_offsets, max_new_tokens, eos_id, nullptr, out_ids,
                    out_counts, "dsb_generate");
  });
}

extern "C" int dsb_generate_sampled(dsb_ctx* ctx, dsb_model* m, dsb_kvcache* kv, const int32_t* seq_ids, int B,
                                    const int32_t* prompt_tokens, const int32_t* prompt_offsets, int max_new_tokens,
                                    int32_t eos_id, const dsb_sampling* sampling, int32_t* out_ids,
                                    int32_t* out_counts) {
  if (ctx != nullptr && sampling == nullptr) return fail(ctx, DSB_EINVAL, "dsb_generate_sampled: no sampling config");
  return guarded(ctx, "dsb_generate_sampled", [&] {  // std::random_device or host allocation may throw
    return generate(ctx, m, kv, seq_ids, B, prompt_tokens, prompt_offsets, max_new_tokens, eos_id, sampling, out_ids,
                    out_counts, "dsb_generate_sampled");
  });
}

dsb_ctx* dsb::model_ctx(const dsb_model* m) { return m->ctx; }
const dsb_model_config* dsb::model_config(const dsb_model* m) { return &m->cfg; }

extern "C" int dsb_model_create(dsb_ctx* ctx, const dsb_model_config* cfg, dsb_model** out) {
  return guarded(ctx, "dsb_model_create", [&] { return model_create_impl(ctx, cfg, out); });
}

extern "C" int dsb_model_set_tensor(dsb_model* m, const char* cname, int dtype, const int64_t* shape, int ndim,
                                    const void* data) {
  return guarded(m ? m->ctx : nullptr, "dsb_model_set_tensor",
                 [&] { return model_set_tensor_impl(m, cname, dtype, shape, ndim, data); });
}

extern "C" int dsb_kvcache_create(dsb_ctx* ctx, const dsb_model* m, int64_t n_blocks, int max_seqs,
                                  int max_blocks_per_seq, dsb_kvcache** out) {
  return guarded(ctx, "dsb_kvcache_create",
                 [&] { return kvcache_create_impl(ctx, m, n_blocks, max_seqs, max_blocks_per_seq, out); });
}

extern "C" int dsb_kvcache_alloc_seq(dsb_kvcache* kv, int* seq_id) {
  return guarded(kv ? kv->ctx : nullptr, "dsb_kvcache_alloc_seq", [&] { return kvcache_alloc_seq_impl(kv, seq_id); });
}

extern "C" int dsb_kvcache_fill_random(dsb_kvcache* kv, int seq_id, int n_tokens, uint64_t seed, float stddev) {
  return guarded(kv ? kv->ctx : nullptr, "dsb_kvcache_fill_random",
                 [&] { return kvcache_fill_random_impl(kv, seq_id, n_tokens, seed, stddev); });
}
