/*
 * CPU oracle for the deepseek_cpp_infer decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library (libdsb.so).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load liboracle.so.
 *
 * Each function restates the reference algorithm in plain C and cites the
 * reference file:line it follows (paths relative to the deepseek_cpp_infer
 * project).  Arithmetic follows the reference's operation order (float
 * accumulation, left to right) so that the primitives match the reference
 * bit for bit; the functions the reference lacks (absorbed MLA over a paged
 * latent cache, the sigmoid+bias grouped router, FP8 e4m3 block scaling,
 * token permutation) are restatements of the published algorithms written in
 * the reference's conventions, and are pinned against the reference's own
 * mathematically equivalent functions by the tests (golden fixtures under
 * tests/golden/ generated from the reference build in oracle/_ref/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ dtypes */

/* bf16 -> f32: the high 16 bits of an IEEE-754 float
 * (src/core/dtype.cpp:8-14). */
ORC_API float orc_bf16_to_f32(uint16_t v) {
  uint32_t u = ((uint32_t)v) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* f32 -> bf16, round to nearest even (NaN kept quiet). */
ORC_API uint16_t orc_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

ORC_API void orc_bf16_to_f32_n(const uint16_t* src, int64_t n, float* dst) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_bf16_to_f32(src[i]);
}

ORC_API void orc_f32_to_bf16_n(const float* src, int64_t n, uint16_t* dst) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_f32_to_bf16(src[i]);
}

/* -------------------------------------------------------------- primitives */

/* dot product with float accumulation (src/core/math.cpp:9-13). */
ORC_API float orc_dot_f32(const float* a, const float* b, int64_t n) {
  float acc = 0.0f;
  for (int64_t i = 0; i < n; ++i) acc += a[i] * b[i];
  return acc;
}

/* y = x * w / sqrt(mean(x^2) + eps)  (src/ops/core/ops.cpp:17-23). */
ORC_API void orc_rmsnorm_f32(const float* x, const float* w, int64_t n, float eps, float* y) {
  float mean2 = 0.0f;
  for (int64_t i = 0; i < n; ++i) mean2 += x[i] * x[i];
  mean2 /= (float)n;
  const float inv = 1.0f / sqrtf(mean2 + eps);
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
}

/* Interleaved-pair RoPE: rotate (x[2k], x[2k+1]) by pos * theta^(-2k/dim)
 * (src/ops/core/rope.cpp:8-23).  Returns -1 for an odd dim, like the
 * reference's throw. */
ORC_API int orc_rope_inplace_f32(float* x, int64_t dim, int64_t pos, float theta) {
  if ((dim % 2) != 0) return -1;
  for (int64_t i = 0; i < dim; i += 2) {
    const int64_t k = i / 2;
    const float inv_freq = powf(theta, -(float)(2.0 * (double)k) / (float)dim);
    const float ang = (float)pos * inv_freq;
    const float c = cosf(ang);
    const float s = sinf(ang);
    const float x0 = x[i];
    const float x1 = x[i + 1];
    x[i] = x0 * c - x1 * s;
    x[i + 1] = x0 * s + x1 * c;
  }
  return 0;
}

/* Stable softmax in place; -1 when the sum is not positive
 * (src/core/math.cpp:15-27). */
ORC_API int orc_softmax_f32(float* x, int64_t n) {
  if (n == 0) return 0;
  float mx = x[0];
  for (int64_t i = 1; i < n; ++i) mx = fmaxf(mx, x[i]);
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    x[i] = expf(x[i] - mx);
    sum += x[i];
  }
  if (!(sum > 0.0f)) return -1;
  const float inv = 1.0f / sum;
  for (int64_t i = 0; i < n; ++i) x[i] *= inv;
  return 0;
}

/* First index of the maximum, strict '>' so ties go to the lowest index
 * (src/core/math.cpp:29-40). */
ORC_API int64_t orc_argmax_f32(const float* x, int64_t n) {
  if (n == 0) return 0;
  int64_t best = 0;
  float bv = x[0];
  for (int64_t i = 1; i < n; ++i) {
    if (x[i] > bv) {
      bv = x[i];
      best = i;
    }
  }
  return best;
}

/* Row-major matvec y[o] = sum_i x[i] * W[o, i], float accumulation
 * (src/models/deepseek/ops.cpp:49-63). */
ORC_API void orc_linear_f32(const float* w, const float* x, int64_t in, float* y, int64_t out) {
  for (int64_t o = 0; o < out; ++o) {
    const float* row = w + o * in;
    float acc = 0.0f;
    for (int64_t i = 0; i < in; ++i) acc += x[i] * row[i];
    y[o] = acc;
  }
}

static float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* down(silu(gate x) * up x)  (src/models/deepseek/ops.cpp:97-108). */
ORC_API void orc_dense_mlp_f32(const float* w_gate, const float* w_up, const float* w_down, const float* x,
                               int64_t hidden, int64_t inter, float* out) {
  float* g = (float*)malloc(sizeof(float) * (size_t)inter);
  float* u = (float*)malloc(sizeof(float) * (size_t)inter);
  orc_linear_f32(w_gate, x, hidden, g, inter);
  orc_linear_f32(w_up, x, hidden, u, inter);
  for (int64_t i = 0; i < inter; ++i) g[i] = orc_silu(g[i]) * u[i];
  orc_linear_f32(w_down, g, inter, out, hidden);
  free(g);
  free(u);
}

/* ------------------------------------------------- absorbed MLA, paged cache */

/*
 * Latent attention for one head (src/models/deepseek/mla.cpp:104-115):
 * scores[t] = dot_f32(q, row_t, D) * scale, softmax_f32, then
 * out[i] = sum_t scores[t] * row_t[i] for i < R, float accumulation in token
 * order.  rows holds len rows of D = R + P values [c | kr].
 */
static int orc_attend_latent(const float* q, const float* rows, int len, int D, int R, float scale, float* scores,
                             float* out) {
  for (int t = 0; t < len; ++t) scores[t] = orc_dot_f32(q, rows + (int64_t)t * D, D) * scale;
  const int rc = orc_softmax_f32(scores, len);
  for (int i = 0; i < R; ++i) out[i] = 0.0f;
  for (int t = 0; t < len; ++t) {
    const float* c = rows + (int64_t)t * D;
    for (int i = 0; i < R; ++i) out[i] += scores[t] * c[i];
  }
  return rc;
}

/*
 * Absorbed MLA decode attention over a paged latent cache.
 *
 * Per sequence b and head h the reference computes (src/models/deepseek/mla.cpp:86-116)
 *   s_t = dot(q_h, k_{t,h}) * scale, p = softmax(s), o_h = sum_t p_t v_{t,h}
 * with k_{t,h} = [W_UK[h] c_t ; rope(kr_t)] and v_{t,h} = W_UV[h] c_t.  With
 * q_lat[h] = W_UK[h]^T q_nope[h] the score is dot([q_lat ; q_rope], [c_t ; kr_t]),
 * and o_h = W_UV[h] (sum_t p_t c_t): this function returns the latent output
 * o_lat[b, h, :] = sum_t p_t c_t (R values).  The cache row of token t of
 * sequence b is block_table[b * max_blocks + t / block_size] * block_size +
 * t % block_size; each row holds [c (R) | kr (P)] in bf16.
 * Returns 0, or -1 when a softmax sum is not positive.
 */
ORC_API int orc_mla_decode_paged(const uint16_t* q_lat, const uint16_t* q_rope, const uint16_t* cache,
                                 const int32_t* block_table, const int32_t* seq_lens, int B, int H, int R, int P,
                                 int block_size, int max_blocks, float scale, float* out) {
  const int D = R + P;
  float* q = (float*)malloc(sizeof(float) * (size_t)D);
  int rc = 0;
  for (int b = 0; b < B; ++b) {
    const int len = seq_lens[b];
    float* scores = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
    float* rows = (float*)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1) * (size_t)D);
    for (int t = 0; t < len; ++t) {
      const int64_t page = block_table[(int64_t)b * max_blocks + t / block_size];
      const int64_t row = page * block_size + t % block_size;
      orc_bf16_to_f32_n(cache + row * D, D, rows + (int64_t)t * D);
    }
    for (int h = 0; h < H; ++h) {
      orc_bf16_to_f32_n(q_lat + ((int64_t)b * H + h) * R, R, q);
      orc_bf16_to_f32_n(q_rope + ((int64_t)b * H + h) * P, P, q + R);
      if (orc_attend_latent(q, rows, len, D, R, scale, scores, out + ((int64_t)b * H + h) * R) != 0) rc = -1;
    }
    free(rows);
    free(scores);
  }
  free(q);
  return rc;
}

/*
 * One MLA layer (no q-LoRA) decoded for T consecutive positions 0..T-1 of one
 * sequence, written with absorbed weights over a latent cache.  It follows
 * mla_decode_step (src/models/deepseek/mla.cpp:41-119) step for step:
 *   q = W_q x, kv_a = W_kva x (mla.cpp:58-72), c = rmsnorm(kv_a[:R]) (mla.cpp:74-77),
 *   kr = rope(kv_a[R:], pos) (mla.cpp:82-84), q_rope = rope(q_h[nope:], pos) (mla.cpp:97),
 *   attention (mla.cpp:104-116) and o_proj (mla.cpp:118),
 * but with k_nope/v never materialised: q_lat[h] = W_UK[h]^T q_nope[h],
 * o_h = W_UV[h] sum_t p_t c_t, where kv_b rows [h*(nope+v), h*(nope+v)+nope)
 * are W_UK[h] and the following v rows are W_UV[h] (mla.cpp:99-102).
 * The latent cache is kept in fp32 here; the test pins this restatement to
 * the reference's non-absorbed mla_decode_step.
 */
ORC_API void orc_act_fp8_roundtrip(float* x, int64_t T, int64_t K);

static int mla_layer_seq(int D, int H, int nope, int rope, int v, int R, float eps, float theta, const float* w_q,
                         const float* w_kva, const float* w_kva_norm, const float* w_kvb, const float* w_o,
                         const float* hidden, int T, float* out, int fp8_o);

ORC_API int orc_mla_layer_seq_f32(int D, int H, int nope, int rope, int v, int R, float eps, float theta,
                                  const float* w_q, const float* w_kva, const float* w_kva_norm, const float* w_kvb,
                                  const float* w_o, const float* hidden, int T, float* out) {
  return mla_layer_seq(D, H, nope, rope, v, R, eps, theta, w_q, w_kva, w_kva_norm, w_kvb, w_o, hidden, T, out, 0);
}

/* The same layer for a block-scaled FP8 checkpoint: the o_proj input (the
 * heads' outputs) goes through orc_act_fp8_roundtrip first, as the FP8 GEMM
 * quantises its activations; the weights are the dequantised ones. */
ORC_API int orc_mla_layer_seq_fp8act_f32(int D, int H, int nope, int rope, int v, int R, float eps, float theta,
                                         const float* w_q, const float* w_kva, const float* w_kva_norm,
                                         const float* w_kvb, const float* w_o, const float* hidden, int T,
                                         float* out) {
  return mla_layer_seq(D, H, nope, rope, v, R, eps, theta, w_q, w_kva, w_kva_norm, w_kvb, w_o, hidden, T, out, 1);
}

static int mla_layer_seq(int D, int H, int nope, int rope, int v, int R, float eps, float theta, const float* w_q,
                         const float* w_kva, const float* w_kva_norm, const float* w_kvb, const float* w_o,
                         const float* hidden, int T, float* out, int fp8_o) {
  const int qh = nope + rope;
  const float scale = 1.0f / sqrtf((float)qh);
  float* q = (float*)calloc((size_t)H * qh, sizeof(float));
  float* kva = (float*)calloc((size_t)(R + rope), sizeof(float));
  float* lat = (float*)calloc((size_t)T * (R + rope), sizeof(float)); /* cache rows [c | kr] */
  float* qfull = (float*)calloc((size_t)(R + rope), sizeof(float));
  float* scores = (float*)calloc((size_t)T, sizeof(float));
  float* olat = (float*)calloc((size_t)R, sizeof(float));
  float* attn = (float*)calloc((size_t)H * v, sizeof(float));
  int rc = 0;
  for (int pos = 0; pos < T; ++pos) {
    const float* x = hidden + (int64_t)pos * D;
    orc_linear_f32(w_q, x, D, q, (int64_t)H * qh);
    orc_linear_f32(w_kva, x, D, kva, R + rope);
    float* row = lat + (int64_t)pos * (R + rope);
    orc_rmsnorm_f32(kva, w_kva_norm, R, eps, row);
    memcpy(row + R, kva + R, sizeof(float) * (size_t)rope);
    if (rope > 0) orc_rope_inplace_f32(row + R, rope, pos, theta);
    for (int h = 0; h < H; ++h) {
      const float* qn = q + (int64_t)h * qh;
      const float* wuk = w_kvb + (int64_t)h * (nope + v) * R; /* [nope, R] */
      const float* wuv = wuk + (int64_t)nope * R;              /* [v, R] */
      /* q_lat = W_UK^T q_nope */
      for (int r = 0; r < R; ++r) {
        float acc = 0.0f;
        for (int i = 0; i < nope; ++i) acc += qn[i] * wuk[(int64_t)i * R + r];
        qfull[r] = acc;
      }
      memcpy(qfull + R, qn + nope, sizeof(float) * (size_t)rope);
      if (rope > 0) orc_rope_inplace_f32(qfull + R, rope, pos, theta);
      if (orc_attend_latent(qfull, lat, pos + 1, R + rope, R, scale, scores, olat) != 0) rc = -1;
      orc_linear_f32(wuv, olat, R, attn + (int64_t)h * v, v);
    }
    if (fp8_o) orc_act_fp8_roundtrip(attn, 1, (int64_t)H * v);
    orc_linear_f32(w_o, attn, (int64_t)H * v, out + (int64_t)pos * D, D);
  }
  free(q);
  free(kva);
  free(lat);
  free(qfull);
  free(scores);
  free(olat);
  free(attn);
  return rc;
}

/* ------------------------------------------ fused norm + rope + cache append */

/*
 * For each of B tokens: c = rmsnorm(kv_a[b, :R]) * w (mla.cpp:74-77),
 * kr = rope(kv_a[b, R:R+P], pos[b]) (mla.cpp:82-84), written as bf16 into the
 * paged cache row of (seq b, position pos[b]); and q_rope[b, h] =
 * rope(q[b, h, nope:nope+P], pos[b]) (mla.cpp:97) for every head.
 * kv_a, q are fp32 here; q row stride is H*(nope+P).
 */
ORC_API int orc_kv_norm_rope_append(const float* kv_a, const float* w_norm, const float* q, const int32_t* positions,
                                    const int32_t* block_table, int B, int H, int nope, int R, int P,
                                    int block_size, int max_blocks, float eps, float theta, uint16_t* cache,
                                    float* q_rope_out) {
  float* tmp = (float*)malloc(sizeof(float) * (size_t)(R + P));
  for (int b = 0; b < B; ++b) {
    const int pos = positions[b];
    const float* src = kv_a + (int64_t)b * (R + P);
    orc_rmsnorm_f32(src, w_norm, R, eps, tmp);
    memcpy(tmp + R, src + R, sizeof(float) * (size_t)P);
    if (P > 0 && orc_rope_inplace_f32(tmp + R, P, pos, theta) != 0) {
      free(tmp);
      return -1;
    }
    const int64_t page = block_table[(int64_t)b * max_blocks + pos / block_size];
    const int64_t row = page * block_size + pos % block_size;
    orc_f32_to_bf16_n(tmp, R + P, cache + row * (R + P));
    for (int h = 0; h < H; ++h) {
      float* dst = q_rope_out + ((int64_t)b * H + h) * P;
      memcpy(dst, q + ((int64_t)b * H + h) * (nope + P) + nope, sizeof(float) * (size_t)P);
      if (P > 0) orc_rope_inplace_f32(dst, P, pos, theta);
    }
  }
  free(tmp);
  return 0;
}

/* ------------------------------------------------------------------ router */

/*
 * Top-k selection by strict '>' insertion with ties going to the lower index,
 * as in routing_kernels.cu:21-30 (the CPU partial_sort at ops.cpp:37-45 picks
 * the same set; its order among equal scores is unspecified).
 */
static void orc_topk(const float* s, int n, int k, int32_t* ids, float* vals) {
  for (int j = 0; j < k; ++j) {
    ids[j] = -1;
    vals[j] = -INFINITY;
  }
  for (int i = 0; i < n; ++i) {
    const float v = s[i];
    for (int j = 0; j < k; ++j) {
      if (ids[j] < 0 || v > vals[j]) {
        for (int m = k - 1; m > j; --m) {
          ids[m] = ids[m - 1];
          vals[m] = vals[m - 1];
        }
        ids[j] = i;
        vals[j] = v;
        break;
      }
    }
  }
}

/*
 * Softmax-greedy router (src/models/deepseek/ops.cpp:110-131): softmax over
 * the E gate logits, top-k, optional renormalisation of the k probabilities
 * (sum > 0), then each weight times routed_scaling_factor (ops.cpp:137).
 * logits [T, E] fp32 -> ids [T, k] int32, weights [T, k] fp32.
 */
ORC_API int orc_route_softmax_greedy(const float* logits, int T, int E, int k, int norm_topk, float routed_scale,
                                     int32_t* ids, float* weights) {
  float* s = (float*)malloc(sizeof(float) * (size_t)E);
  float* v = (float*)malloc(sizeof(float) * (size_t)k);
  int rc = 0;
  for (int t = 0; t < T; ++t) {
    memcpy(s, logits + (int64_t)t * E, sizeof(float) * (size_t)E);
    if (orc_softmax_f32(s, E) != 0) rc = -1;
    orc_topk(s, E, k, ids + (int64_t)t * k, v);
    if (norm_topk) {
      float sum = 0.0f;
      for (int j = 0; j < k; ++j) sum += v[j];
      if (sum > 0.0f)
        for (int j = 0; j < k; ++j) v[j] /= sum;
    }
    for (int j = 0; j < k; ++j) weights[(int64_t)t * k + j] = v[j] * routed_scale;
  }
  free(s);
  free(v);
  return rc;
}

/*
 * The expert half of moe_step (src/models/deepseek/ops.cpp:128-145) for one
 * token whose experts are already chosen: for each pick i in order
 * out += (w[i] * routed_scale) * mlp_{ids[i]}(x), then out += shared(x).
 * Expert weights: gate/up [E, I, D], down [E, D, I]; shared gate/up [Is, D],
 * down [D, Is] (s_gate NULL = no shared experts).
 */
ORC_API void orc_moe_mix_f32(const float* e_gate, const float* e_up, const float* e_down, const float* s_gate,
                             const float* s_up, const float* s_down, int shared_inter, int D, int I, int k,
                             const int32_t* ids, const float* w, float routed_scale, const float* x, float* out) {
  float* tmp = (float*)malloc(sizeof(float) * (size_t)D);
  for (int j = 0; j < D; ++j) out[j] = 0.0f;
  for (int i = 0; i < k; ++i) {
    const int64_t e = ids[i];
    orc_dense_mlp_f32(e_gate + e * I * D, e_up + e * I * D, e_down + e * D * I, x, D, I, tmp);
    const float scale = w[i] * routed_scale;
    for (int j = 0; j < D; ++j) out[j] += scale * tmp[j];
  }
  if (s_gate != NULL) {
    orc_dense_mlp_f32(s_gate, s_up, s_down, x, D, shared_inter, tmp);
    for (int j = 0; j < D; ++j) out[j] += tmp[j];
  }
  free(tmp);
}

/*
 * One token through a softmax-greedy MoE block, step for step as moe_step
 * (src/models/deepseek/ops.cpp:110-146): gate logits -> route -> for each
 * chosen expert out += (p * routed_scale) * mlp_e(x) in selection order ->
 * out += shared(x).  Expert weights: gate/up [E, I, D], down [E, D, I];
 * shared gate/up [Is, D], down [D, Is] (s_gate NULL = no shared experts).
 */
ORC_API int orc_moe_softmax_f32(const float* w_gate, const float* e_gate, const float* e_up, const float* e_down,
                                const float* s_gate, const float* s_up, const float* s_down, int shared_inter, int D,
                                int E, int k, int I, int norm_topk, float routed_scale, const float* x, float* out) {
  float* logits = (float*)malloc(sizeof(float) * (size_t)E);
  int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)k);
  float* w = (float*)malloc(sizeof(float) * (size_t)k);
  orc_linear_f32(w_gate, x, D, logits, E);
  const int rc = orc_route_softmax_greedy(logits, 1, E, k, norm_topk, 1.0f, ids, w);
  orc_moe_mix_f32(e_gate, e_up, e_down, s_gate, s_up, s_down, shared_inter, D, I, k, ids, w, routed_scale, x, out);
  free(logits);
  free(ids);
  free(w);
  return rc;
}

/*
 * Sigmoid + bias grouped router (no reference code; the published DeepSeek-V3
 * "noaux_tc" method, written in the conventions of ops.cpp:110-146):
 *   s = sigmoid(logit); s' = s + bias
 *   group score = sum of the top-2 s' inside each of n_group equal groups
 *   keep the topk_group best groups (ties -> lower group id)
 *   top-k of s' over experts in kept groups (ties -> lower expert id)
 *   weight = s (without bias) of the chosen experts, divided by their sum
 *   when norm_topk (V3 uses it), then times routed_scale.
 */
ORC_API int orc_route_sigmoid_grouped(const float* logits, const float* bias, int T, int E, int n_group,
                                      int topk_group, int k, int norm_topk, float routed_scale, int32_t* ids,
                                      float* weights) {
  if (n_group <= 0 || E % n_group != 0) return -1;
  const int per = E / n_group;
  float* s = (float*)malloc(sizeof(float) * (size_t)E);
  float* sb = (float*)malloc(sizeof(float) * (size_t)E);
  float* gs = (float*)malloc(sizeof(float) * (size_t)n_group);
  int32_t* gid = (int32_t*)malloc(sizeof(int32_t) * (size_t)n_group);
  float* gv = (float*)malloc(sizeof(float) * (size_t)n_group);
  float* masked = (float*)malloc(sizeof(float) * (size_t)E);
  float* v = (float*)malloc(sizeof(float) * (size_t)k);
  for (int t = 0; t < T; ++t) {
    const float* lg = logits + (int64_t)t * E;
    for (int e = 0; e < E; ++e) {
      s[e] = 1.0f / (1.0f + expf(-lg[e]));
      sb[e] = s[e] + bias[e];
    }
    for (int g = 0; g < n_group; ++g) {
      int32_t i2[2];
      float v2[2];
      orc_topk(sb + g * per, per, per >= 2 ? 2 : 1, i2, v2);
      gs[g] = per >= 2 ? v2[0] + v2[1] : v2[0];
    }
    orc_topk(gs, n_group, topk_group, gid, gv);
    for (int e = 0; e < E; ++e) masked[e] = -INFINITY;
    for (int j = 0; j < topk_group; ++j) {
      const int g = gid[j];
      for (int e = g * per; e < (g + 1) * per; ++e) masked[e] = sb[e];
    }
    int32_t* out_ids = ids + (int64_t)t * k;
    orc_topk(masked, E, k, out_ids, v);
    float sum = 0.0f;
    for (int j = 0; j < k; ++j) {
      v[j] = s[out_ids[j]];
      sum += v[j];
    }
    for (int j = 0; j < k; ++j) {
      float w = v[j];
      if (norm_topk && sum > 0.0f) w /= sum;
      weights[(int64_t)t * k + j] = w * routed_scale;
    }
  }
  free(s);
  free(sb);
  free(gs);
  free(gid);
  free(gv);
  free(masked);
  free(v);
  return 0;
}

/*
 * Token permutation with histogram offsets.  For the T*k (token, slot) pairs
 * in token-major order: counts[e] = pairs routed to e, offsets = exclusive
 * prefix sum, and the pair with flat index i = t*k + j lands at position
 * dest[i] = offsets[e] + (number of earlier pairs routed to e), so that
 * src_pair[dest[i]] = i.  The order inside an expert is the stable order of
 * the flat index, which the CUDA path reproduces exactly.
 */
ORC_API void orc_moe_permute(const int32_t* ids, int T, int k, int E, int32_t* counts, int32_t* offsets,
                             int32_t* dest, int32_t* src_pair) {
  for (int e = 0; e < E; ++e) counts[e] = 0;
  for (int64_t i = 0; i < (int64_t)T * k; ++i) counts[ids[i]]++;
  int32_t acc = 0;
  for (int e = 0; e < E; ++e) {
    offsets[e] = acc;
    acc += counts[e];
  }
  offsets[E] = acc;
  int32_t* fill = (int32_t*)calloc((size_t)E, sizeof(int32_t));
  for (int64_t i = 0; i < (int64_t)T * k; ++i) {
    const int e = ids[i];
    const int32_t d = offsets[e] + fill[e]++;
    dest[i] = d;
    src_pair[d] = (int32_t)i;
  }
  free(fill);
}

/* --------------------------------------------------------------------- FP8 */

/* e4m3 (1-4-3, bias 7, no inf, S.1111.111 = NaN) decoded by its bit definition. */
ORC_API float orc_e4m3_to_f32(uint8_t v) {
  const int sign = (v >> 7) & 1;
  const int exp = (v >> 3) & 0xF;
  const int man = v & 0x7;
  float mag;
  if (exp == 0xF && man == 0x7) return NAN;
  if (exp == 0)
    mag = ldexpf((float)man, -9); /* subnormal: man/8 * 2^-6 */
  else
    mag = ldexpf(1.0f + (float)man / 8.0f, exp - 7);
  return sign ? -mag : mag;
}

/* f32 -> e4m3, round to nearest even, saturating to +-448 (no inf in e4m3). */
ORC_API uint8_t orc_f32_to_e4m3(float f) {
  if (isnan(f)) return 0x7F;
  const uint8_t sign = signbit(f) ? 0x80 : 0x00;
  float a = fabsf(f);
  if (a >= 448.0f) return sign | 0x7E;
  /* exhaustive nearest search over the 127 non-negative finite codes keeps the
   * rounding rule obvious: nearest value, ties to the even code. */
  uint8_t best = 0;
  float bd = INFINITY;
  for (int c = 0; c <= 0x7E; ++c) {
    const float d = fabsf(orc_e4m3_to_f32((uint8_t)c) - a);
    if (d < bd || (d == bd && (c & 1) == 0)) {
      bd = d;
      best = (uint8_t)c;
    }
  }
  return sign | best;
}

/* Per-token 1x128 activation quantisation: scale = amax / 448 over each
 * 128-column group (1 when the group is all zero), q = e4m3(x / scale). */
ORC_API void orc_quant_act_1x128(const float* x, int64_t T, int64_t K, uint8_t* q, float* scales) {
  const int64_t G = (K + 127) / 128;
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t g = 0; g < G; ++g) {
      const int64_t c0 = g * 128, c1 = c0 + 128 < K ? c0 + 128 : K;
      float amax = 0.0f;
      for (int64_t c = c0; c < c1; ++c) amax = fmaxf(amax, fabsf(x[t * K + c]));
      const float sc = amax > 0.0f ? amax / 448.0f : 1.0f;
      scales[t * G + g] = sc;
      for (int64_t c = c0; c < c1; ++c) q[t * K + c] = orc_f32_to_e4m3(x[t * K + c] / sc);
    }
  }
}

/* An activation as a block-scaled FP8 GEMM sees it: each value rounded to
 * the bf16 activation buffer, quantised per token and 128 columns
 * (orc_quant_act_1x128) and dequantised (e4m3 * scale), in place. */
ORC_API void orc_act_fp8_roundtrip(float* x, int64_t T, int64_t K) {
  const int64_t G = (K + 127) / 128;
  uint8_t* q = (uint8_t*)malloc((size_t)(T * K));
  float* sc = (float*)malloc(sizeof(float) * (size_t)(T * G));
  uint16_t b;
  for (int64_t i = 0; i < T * K; ++i) {
    orc_f32_to_bf16_n(x + i, 1, &b);
    orc_bf16_to_f32_n(&b, 1, x + i);
  }
  orc_quant_act_1x128(x, T, K, q, sc);
  for (int64_t t = 0; t < T; ++t)
    for (int64_t c = 0; c < K; ++c) x[t * K + c] = orc_e4m3_to_f32(q[t * K + c]) * sc[t * G + c / 128];
  free(q);
  free(sc);
}

/* Weight quantisation per 128x128 block: scale = amax / 448 over the block
 * (1 when it is all zero), q = e4m3(w / scale); scales [ceil(M/128), ceil(K/128)]. */
ORC_API void orc_quant_weight_128x128(const float* w, int64_t M, int64_t K, uint8_t* q, float* scales) {
  const int64_t GM = (M + 127) / 128, GK = (K + 127) / 128;
  for (int64_t bm = 0; bm < GM; ++bm) {
    for (int64_t bk = 0; bk < GK; ++bk) {
      const int64_t r1 = (bm + 1) * 128 < M ? (bm + 1) * 128 : M, c1 = (bk + 1) * 128 < K ? (bk + 1) * 128 : K;
      float amax = 0.0f;
      for (int64_t r = bm * 128; r < r1; ++r)
        for (int64_t c = bk * 128; c < c1; ++c) amax = fmaxf(amax, fabsf(w[r * K + c]));
      const float sc = amax > 0.0f ? amax / 448.0f : 1.0f;
      scales[bm * GK + bk] = sc;
      for (int64_t r = bm * 128; r < r1; ++r)
        for (int64_t c = bk * 128; c < c1; ++c) q[r * K + c] = orc_f32_to_e4m3(w[r * K + c] / sc);
    }
  }
}

/*
 * y[t, o] = sum_k (e4m3(w[o,k]) * sw[o/128][k/128]) * (e4m3(x[t,k]) * sx[t][k/128]),
 * accumulated in double and rounded to float; equals ds::rt::linear
 * (ops.cpp:49-63) applied to the dequantised weights and activations.
 */
ORC_API void orc_fp8_linear(const uint8_t* w, const float* sw, const uint8_t* x, const float* sx, int64_t T,
                            int64_t O, int64_t K, float* y) {
  const int64_t GK = (K + 127) / 128;
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t o = 0; o < O; ++o) {
      double acc = 0.0;
      for (int64_t kk = 0; kk < K; ++kk) {
        const double wv = (double)orc_e4m3_to_f32(w[o * K + kk]) * sw[(o / 128) * GK + kk / 128];
        const double xv = (double)orc_e4m3_to_f32(x[t * K + kk]) * sx[t * GK + kk / 128];
        acc += wv * xv;
      }
      y[t * O + o] = (float)acc;
    }
  }
}

/* ---------------------------------------------------------------- sampling */

typedef struct {
  int32_t id;
  float x; /* logit / t */
  float p;
} orc_item;

/* Descending x, ties to the lower id: the order the CUDA sampler scans a
 * filtered row in, one of the orders std::nth_element / std::sort can leave
 * (p is non-decreasing in x, so this is also a descending-p order). */
static int orc_item_desc(const void* a, const void* b) {
  const orc_item* u = (const orc_item*)a;
  const orc_item* v = (const orc_item*)b;
  if (u->x > v->x) return -1;
  if (u->x < v->x) return 1;
  return (u->id > v->id) - (u->id < v->id);
}

/* ds::core::Sampler::sample (src/core/sampler.cpp:23-77) for one row, with
 * the uniform draw r in [0, 1) given instead of drawn.  Steps and float
 * arithmetic as the reference: x = logit / t (t <= 0 reads as 1); top-k
 * (0 < top_k < V) keeps the top_k largest x; softmax over the kept items in
 * their current order (math.cpp:15-27); top-p (0 < top_p < 1) sorts by p,
 * accumulates until cum >= top_p (that item kept, at least one) and divides
 * by the kept sum; the draw returns the first item in order with r <= cum,
 * else the last.  Orders the reference leaves unspecified (nth_element's
 * arrangement, std::sort among equal p) are fixed to descending x with ties
 * to the lower id; with no cut active the items stay in id order.
 * margin: distance of r from the nearer end of the chosen item's cumulative
 * interval; cut_margin: |cum - top_p| where the top-p cut stopped (1 when no
 * top-p cut).  Either may be NULL.  Returns the id, or -1 when V <= 0 or the
 * softmax sum is not positive (the reference throws). */
ORC_API int32_t orc_sample(const float* logits, int64_t V, float temperature, int32_t top_k, float top_p, float r,
                           double* margin, double* cut_margin) {
  if (V <= 0) return -1;
  orc_item* it = (orc_item*)malloc((size_t)V * sizeof *it);
  if (it == NULL) return -1;
  const float t = temperature <= 0.0f ? 1.0f : temperature;
  for (int64_t i = 0; i < V; ++i) {
    it[i].id = (int32_t)i;
    it[i].x = logits[i] / t;
    it[i].p = 0.0f;
  }
  int64_t n = V;
  const int sorted = top_k > 0 && top_k < V;
  if (sorted) {
    qsort(it, (size_t)V, sizeof *it, orc_item_desc);
    n = top_k;
  }
  float mx = it[0].x;
  for (int64_t i = 1; i < n; ++i) mx = (mx < it[i].x) ? it[i].x : mx; /* std::max */
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    it[i].p = expf(it[i].x - mx);
    sum += it[i].p;
  }
  if (!(sum > 0.0f)) {
    free(it);
    return -1;
  }
  const float inv = 1.0f / sum;
  for (int64_t i = 0; i < n; ++i) it[i].p *= inv;
  double cm = 1.0;
  if (top_p > 0.0f && top_p < 1.0f) {
    if (!sorted) qsort(it, (size_t)n, sizeof *it, orc_item_desc);
    float cum = 0.0f;
    int64_t keep = 0;
    for (; keep < n; ++keep) {
      cum += it[keep].p;
      if (cum >= top_p) {
        ++keep;
        break;
      }
    }
    cm = fabs((double)cum - (double)top_p);
    if (keep < 1) keep = 1;
    if (keep > n) keep = n;
    n = keep;
    float s = 0.0f;
    for (int64_t i = 0; i < n; ++i) s += it[i].p;
    for (int64_t i = 0; i < n; ++i) it[i].p /= s;
  }
  float cum = 0.0f;
  int32_t id = it[n - 1].id;
  double mg = -1.0;
  for (int64_t i = 0; i < n; ++i) {
    const float prev = cum;
    cum += it[i].p;
    if (r <= cum) {
      id = it[i].id;
      const double a = (double)r - (double)prev, b = (double)cum - (double)r;
      mg = a < b ? a : b;
      break;
    }
  }
  if (mg < 0.0) mg = (double)r - (double)cum;
  if (margin) *margin = mg;
  if (cut_margin) *cut_margin = cm;
  free(it);
  return id;
}
