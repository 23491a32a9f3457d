// Memory-bound and routing kernels of the decode step, sm_100a.
//
// Each kernel replaces a reference CPU function or SIMT kernel and keeps its
// arithmetic order where that decides the result: products are rounded in the
// reference's order with __fmul_rn/__fadd_rn (no FMA contraction), softmax /
// RMSNorm use IEEE division and square root, ties go to the lowest index.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"
#include "ep_common.cuh"
#include "rows.cuh"

namespace dsb {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum of one float per thread (blockDim.x multiple of 32, <= 1024).
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.0f;
  for (int i = 0; i < nw; ++i) r += red[i];
  return r;
}

// ------------------------------------------------------------------ RMSNorm

// y = x * (1 / sqrt(mean(x^2) + eps)) * w per row (src/ops/core/ops.cpp:17-23,
// ds_rmsnorm_kernel elementwise_kernels.cu:13-28), written as bf16 and/or fp32.
// 1 / sqrt(mean(x^2) + eps) of one row, by the whole block; the summation
// order depends only on blockDim.x, so every kernel that normalises a row
// with the same block size gets the same bits.
__device__ float row_inv_rms(const float* xr, int n, bool vec, float eps, float* red) {
  float ss = 0.0f;
  if (vec) {  // 16-byte rows
    for (int i4 = threadIdx.x; i4 < n / 4; i4 += blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(xr)[i4];
      ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
      ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
      ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
      ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
  }
  const float mean2 = __fdiv_rn(block_sum(ss, red), (float)n);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean2, eps)));
}

__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ w, int n,
                                    float eps, __nv_bfloat16* __restrict__ yb, int64_t ldyb, float* __restrict__ yf,
                                    int64_t ldyf) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ float red[32];
  const float* xr = x + blockIdx.x * ldx;
  const float inv = row_inv_rms(xr, n, (n % 4) == 0 && (ldx % 4) == 0, eps, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
    if (yb) yb[blockIdx.x * ldyb + i] = __float2bfloat16_rn(v);
    if (yf) yf[blockIdx.x * ldyf + i] = v;
  }
}

// -------------------------------------------------- norm + RoPE + cache append

// Interleaved-pair rotation of (x0, x1) by the angle whose cosine / sine are
// c / s (src/ops/core/rope.cpp:8-23; pair k of a dim-wide rope vector turns by
// pos * theta^(-2k/dim)).
__device__ __forceinline__ void rotate_pair(float& x0, float& x1, float c, float s) {
  const float a = x0, b = x1;
  x0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  x1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// Per token b: c = rmsnorm(kv_a[b, :R]) * w and kr = rope(kv_a[b, R:]) go to
// the token's paged-cache row (mla.cpp:74-84), and every head's rope query
// q[b, h, nope:] is rotated into q_rope[b, h] (mla.cpp:97).
__global__ void kv_norm_rope_append_kernel(const float* __restrict__ kv_a, int64_t ld_kv, const float* __restrict__ w_norm,
                                           const __nv_bfloat16* __restrict__ q, const float* __restrict__ qf,
                                           int64_t ld_qf, __nv_bfloat16* __restrict__ q_out,
                                           const int32_t* __restrict__ pos, const int32_t* __restrict__ block_table,
                                           int max_blocks, int H, int nope, int R, int P, float eps, float theta,
                                           __nv_bfloat16* __restrict__ cache, __nv_bfloat16* __restrict__ q_rope) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ float red[32];
  __shared__ float cs[2][64];  // cos / sin of each rope pair at this token's position (P <= 128)
  // CTA (b, 0) appends the latent row; with gridDim.y > 1 the query's heads
  // are split over CTAs (b, 1..), which run beside it
  const int b = blockIdx.x, part = blockIdx.y, qparts = gridDim.y > 1 ? gridDim.y - 1 : 1;
  const int p = pos[b];
  const float* kv = kv_a + (int64_t)b * ld_kv;
  for (int k = threadIdx.x; k < P / 2; k += blockDim.x) {
    const float inv_freq = powf(theta, __fdiv_rn(-(float)(2 * k), (float)P));  // rope.cpp:8-23
    const float ang = __fmul_rn((float)p, inv_freq);
    cs[0][k] = cosf(ang);
    cs[1][k] = sinf(ang);
  }
  __syncthreads();
  if (part == 0) {
    float ss = 0.0f;
    for (int i = threadIdx.x; i < R; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(kv[i], kv[i]));
    const float mean2 = __fdiv_rn(block_sum(ss, red), (float)R);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean2, eps)));
    const int64_t page = block_table[(int64_t)b * max_blocks + p / 64];
    __nv_bfloat16* row = cache + (page * 64 + p % 64) * (int64_t)(R + P);
    for (int i = threadIdx.x; i < R; i += blockDim.x) row[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(kv[i], inv), w_norm[i]));
    for (int k = threadIdx.x; k < P / 2; k += blockDim.x) {
      float x0 = kv[R + 2 * k], x1 = kv[R + 2 * k + 1];
      rotate_pair(x0, x1, cs[0][k], cs[1][k]);
      row[R + 2 * k] = __float2bfloat16_rn(x0);
      row[R + 2 * k + 1] = __float2bfloat16_rn(x1);
    }
  }
  if (gridDim.y > 1 && part == 0) return;
  const int qp = gridDim.y > 1 ? part - 1 : 0;
  const int h0 = qp * H / qparts, h1 = (qp + 1) * H / qparts;  // this CTA's query heads
  const int qh = nope + P;
  if (qf != nullptr) {
    // fp32 query: its nope parts go out as the bf16 query of the absorb GEMM
    for (int idx = h0 * nope + (int)threadIdx.x; idx < h1 * nope; idx += blockDim.x) {
      const int h = idx / nope, i = idx % nope;
      q_out[(int64_t)b * H * qh + (int64_t)h * qh + i] = __float2bfloat16_rn(qf[(int64_t)b * ld_qf + h * qh + i]);
    }
  }
  for (int idx = h0 * (P / 2) + (int)threadIdx.x; idx < h1 * (P / 2); idx += blockDim.x) {
    const int h = idx / (P / 2), k = idx % (P / 2);
    float x0, x1;
    if (qf != nullptr) {
      const float* src = qf + (int64_t)b * ld_qf + (int64_t)h * qh + nope + 2 * k;
      x0 = src[0];
      x1 = src[1];
    } else {
      const __nv_bfloat16* src = q + (int64_t)b * H * qh + (int64_t)h * qh + nope + 2 * k;
      x0 = __bfloat162float(src[0]);
      x1 = __bfloat162float(src[1]);
    }
    rotate_pair(x0, x1, cs[0][k], cs[1][k]);
    __nv_bfloat16* dst = q_rope + ((int64_t)b * H + h) * P + 2 * k;
    dst[0] = __float2bfloat16_rn(x0);
    dst[1] = __float2bfloat16_rn(x1);
  }
}

// -------------------------------------------------------------------- router

// logits[t, e] = x[t] . W_gate[e] in fp32 (the reference's gate linear,
// ops.cpp:115-117); one warp per (token, expert).
// One warp's dot product of a normalised row with a router row (D a multiple
// of 4): each lane takes every 32nd float4 in one explicit FMA chain, then
// the warp sums the lanes, so the bits do not depend on where x lives.
__device__ __forceinline__ float router_dot(const float* xr, const float* __restrict__ wr, int D, int lane) {
  float acc = 0.0f;
#pragma unroll 16  // loads in flight: one warp per expert leaves little else to hide their latency
  for (int i = lane * 4; i < D; i += 128) {
    const float4 a = *reinterpret_cast<const float4*>(xr + i);
    const float4 b = __ldg(reinterpret_cast<const float4*>(wr + i));
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
  }
  return warp_sum(acc);
}

__global__ void router_logits_kernel(const float* __restrict__ x, const float* __restrict__ w, int T, int D, int E,
                                     float* __restrict__ logits) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= T * E) return;
  const int t = gw / E, e = gw % E;
  const float acc = router_dot(x + (int64_t)t * D, w + (int64_t)e * D, D, lane);
  if (lane == 0) logits[(int64_t)t * E + e] = acc;
}

// Large batches: a 32-token x 64-expert tile per CTA with both operands staged
// through shared memory in 64-wide slices of D; each thread accumulates 2 x 4
// logits in fp32 (sequential over D within a thread).
constexpr int kRtT = 32, kRtE = 64, kRtD = 64;

__global__ void __launch_bounds__(256) router_logits_tiled_kernel(const float* __restrict__ x,
                                                                   const float* __restrict__ w, int T, int D, int E,
                                                                   float* __restrict__ logits) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ float xs[kRtT][kRtD + 1];
  __shared__ float ws[kRtE][kRtD + 1];
  const int t0 = blockIdx.y * kRtT, e0 = blockIdx.x * kRtE;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads: experts tx+16j, tokens ty+16i
  float acc[2][4] = {};
  for (int d0 = 0; d0 < D; d0 += kRtD) {
    for (int i = threadIdx.x; i < kRtT * kRtD; i += 256) {
      const int rr = i / kRtD, cc = i % kRtD;
      xs[rr][cc] = (t0 + rr < T && d0 + cc < D) ? x[(int64_t)(t0 + rr) * D + d0 + cc] : 0.0f;
    }
    for (int i = threadIdx.x; i < kRtE * kRtD; i += 256) {
      const int rr = i / kRtD, cc = i % kRtD;
      ws[rr][cc] = (e0 + rr < E && d0 + cc < D) ? w[(int64_t)(e0 + rr) * D + d0 + cc] : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < kRtD; ++c) {
      const float a0 = xs[ty][c], a1 = xs[ty + 16][c];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float bv = ws[tx + 16 * j][c];
        acc[0][j] = fmaf(a0, bv, acc[0][j]);
        acc[1][j] = fmaf(a1, bv, acc[1][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = t0 + ty + 16 * i, e = e0 + tx + 16 * j;
      if (t < T && e < E) logits[(int64_t)t * E + e] = acc[i][j];
    }
}

constexpr int kMaxExpertsPerLane = 8;  // E <= 256

// Warp-wide arg-max over per-lane candidates: the largest value, ties to the
// lowest index (the strict '>' scan of routing_kernels.cu:21-30).
__device__ __forceinline__ void warp_argmax(float& v, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
}

// One warp per token.  scoring 0: softmax over the E logits, top-k, optional
// renormalisation, times routed_scale (ops.cpp:110-131,137).  scoring 1:
// sigmoid + bias grouped selection (DeepSeek-V3): groups ranked by the sum of
// their top-2 biased scores, the top topk_group groups kept, top-k experts of
// the kept groups by biased score, weights = unbiased sigmoid scores of the
// chosen experts, normalised when norm_topk, times routed_scale.
// One warp routes one token: lg its E logits (global or shared memory); the
// k picks and weights, then n_extra always-on groups, go to ids_row / w_row.
__device__ __forceinline__ void route_token(const float* lg, const float* __restrict__ bias, int E, int k, int scoring,
                                            int n_group, int topk_group, int norm_topk, float routed_scale,
                                            int32_t* ids_row, float* w_row, int n_extra, int lane) {
  float sel[kMaxExpertsPerLane], val[kMaxExpertsPerLane];  // selection key, weight source
#pragma unroll
  for (int j = 0; j < kMaxExpertsPerLane; ++j) {
    const int e = lane + 32 * j;
    sel[j] = -INFINITY;
    val[j] = 0.0f;
    if (e < E) {
      const float l = lg[e];
      if (scoring == 0) {
        sel[j] = l;  // softmax is monotone: rank by logit, weigh by probability
        val[j] = l;
      } else {
        const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-l)));
        sel[j] = __fadd_rn(s, bias[e]);
        val[j] = s;
      }
    }
  }
  if (scoring == 0) {
    // probabilities: p = exp(l - max) / sum (softmax_f32, math.cpp:15-27)
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j) mx = fmaxf(mx, sel[j]);
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j) {
      const int e = lane + 32 * j;
      val[j] = e < E ? expf(__fsub_rn(val[j], mx)) : 0.0f;
      sum = __fadd_rn(sum, val[j]);
    }
    sum = warp_sum(sum);
    const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j) val[j] = __fmul_rn(val[j], inv);
  } else {
    // group ranking: E/n_group consecutive experts per group
    const int per = E / n_group;
    // group score for every group, computed by lane g (n_group <= 32)
    float gscore = -INFINITY;
    {
      // each lane gathers the biased scores of group `lane` from the owners
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int i = 0; i < per; ++i) {
        // expert lane*per + i lives at lane (e % 32), slot (e / 32)
        float v = -INFINITY;
        // every lane must take part in each shuffle: loop over the slot index
#pragma unroll
        for (int j = 0; j < kMaxExpertsPerLane; ++j) {
          const int e = lane * per + i;
          const float cand = __shfl_sync(0xffffffffu, sel[j], e & 31);
          if ((e >> 5) == j && lane < n_group) v = cand;
        }
        if (lane < n_group) {
          if (v > b1) {
            b2 = b1;
            b1 = v;
          } else if (v > b2) {
            b2 = v;
          }
        }
      }
      if (lane < n_group) gscore = per >= 2 ? __fadd_rn(b1, b2) : b1;
    }
    // keep the best topk_group groups (ties -> lower group id)
    unsigned keep = 0;
    for (int r = 0; r < topk_group; ++r) {
      float v = (lane < n_group && !((keep >> lane) & 1u)) ? gscore : -INFINITY;
      int gi = lane < n_group ? lane : 1 << 30;
      if ((keep >> lane) & 1u) gi = 1 << 30;
      warp_argmax(v, gi);
      keep |= 1u << gi;
    }
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((keep >> (e / per)) & 1u)) sel[j] = -INFINITY;
    }
  }
  // top-k by selection key, ties to the lower expert id
  // k <= 8 picks, kept in registers (every index a compile-time constant)
  float wsel[8];
  int isel[8];
  float wsum = 0.0f;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r >= k) break;
    float v = -INFINITY;
    int idx = 1 << 30;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (sel[j] > v || (sel[j] == v && e < idx))) {
        v = sel[j];
        idx = e;
      }
    }
    warp_argmax(v, idx);
    // owner lane removes the winner and publishes its weight source
    float wv = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j)
      if (lane + 32 * j == idx) {
        wv = val[j];
        sel[j] = -INFINITY;
      }
    wv = __shfl_sync(0xffffffffu, wv, idx & 31);
    wsel[r] = wv;
    isel[r] = idx;
    wsum = __fadd_rn(wsum, wv);
  }
  if (lane == 0) {
    // the k routed picks, then n_extra always-on groups
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (r >= k) break;
      float wv = wsel[r];
      if (norm_topk && wsum > 0.0f) wv = __fdiv_rn(wv, wsum);
      ids_row[r] = isel[r];
      w_row[r] = __fmul_rn(wv, routed_scale);
    }
    for (int j = 0; j < n_extra; ++j) {
      ids_row[k + j] = E + j;
      w_row[k + j] = 1.0f;
    }
  }
}

// With pub.enabled (expert parallel, n_extra = 0), the last CTA to finish
// writes every pick's slot and this rank's pick counts for the dispatch
// (ep_count_warp) once every token is routed.
__global__ void route_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int T, int E, int k,
                             int scoring, int n_group, int topk_group, int norm_topk, float routed_scale,
                             int32_t* __restrict__ ids, float* __restrict__ weights, int n_extra, EpPublishArgs pub,
                             int* __restrict__ ticket, int* __restrict__ status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int kk = k + n_extra;
  if (t < T)
    route_token(logits + (int64_t)t * E, bias, E, k, scoring, n_group, topk_group, norm_topk, routed_scale,
                ids + (int64_t)t * kk, weights + (int64_t)t * kk, n_extra, lane);
  if (!pub.enabled) return;
  __shared__ int last;
  __shared__ int32_t cnt[256];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
    if (last) *ticket = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if ((threadIdx.x >> 5) == 0) ep_count_warp(ids, T * k, pub, status, cnt, lane);
}

// Deterministic permutation of the N = T*k (token, slot) pairs by expert: the
// pair with flat index i goes to dest[i] = offsets[e] + (number of earlier
// pairs routed to e); src_pair is the inverse.  One warp walks the pairs in
// order, 32 at a time, ranking equal experts with match.any.
// ids: the N expert ids, and weights (when w_perm is wanted) their routing
// weights, both in shared memory; cnt is [E] ints of shared memory.
__device__ void permute_warp(const int32_t* ids, int N, int E, int32_t* __restrict__ counts,
                             int32_t* __restrict__ offsets, int32_t* __restrict__ dest, int32_t* __restrict__ src_pair,
                             const float* weights, float* __restrict__ w_perm, int* __restrict__ status, int32_t* cnt,
                             int lane) {
  for (int e = lane; e < E; e += 32) cnt[e] = 0;
  __syncwarp();
  for (int c = 0; c < N; c += 32) {
    const int i = c + lane;
    int e = i < N ? ids[i] : -1 - lane;  // unique negative keys for idle lanes
    if (i < N && (unsigned)e >= (unsigned)E) {  // out-of-range id: flagged, entry dropped
      atomicExch(status, kStatusBadInput);
      e = -1 - lane;
    }
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(grp & ((1u << lane) - 1u));
    const int base = e >= 0 ? cnt[e] : 0;
    __syncwarp();
    if (i < N) dest[i] = base + rank;
    if (e >= 0 && rank == 0) cnt[e] = base + __popc(grp);
    __syncwarp();
  }
  // exclusive prefix sum of the counts
  int carry = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int v = e < E ? cnt[e] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (e < E) {
      counts[e] = v;
      offsets[e] = carry + incl - v;
    }
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) offsets[E] = carry;
  __syncwarp();
#pragma unroll 4
  for (int i = lane; i < N; i += 32) {
    const int e = ids[i];
    if ((unsigned)e >= (unsigned)E) continue;
    const int d = offsets[e] + dest[i];
    dest[i] = d;
    src_pair[d] = i;
    if (w_perm != nullptr) w_perm[d] = weights[i];
  }
}

__global__ void permute_kernel(const int32_t* __restrict__ ids, int N, int E, int32_t* __restrict__ counts,
                               int32_t* __restrict__ offsets, int32_t* __restrict__ dest,
                               int32_t* __restrict__ src_pair, const float* __restrict__ weights,
                               float* __restrict__ w_perm, int* __restrict__ status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  extern __shared__ int32_t cnt[];  // [E] counts, then the N ids and their weights
  int32_t* sids = cnt + E;
  float* swts = reinterpret_cast<float*>(sids + N);
#pragma unroll 8
  for (int i = threadIdx.x; i < N; i += 32) {
    sids[i] = ids[i];
    if (w_perm != nullptr) swts[i] = weights[i];
  }
  __syncwarp();
  permute_warp(sids, N, E, counts, offsets, dest, src_pair, swts, w_perm, status, cnt, threadIdx.x);
}

// The MoE front of a decode step in one launch: post-attention RMSNorm,
// router logits, routing and (single GPU) the permutation by expert.  CTA
// (b, t) normalises token t's row (the bf16 row for the experts is written by
// b == 0) and computes the router logits of experts [8b, 8b+8), one warp per
// expert.  The last of token t's CTAs to finish (a ticket) routes the
// token; with the permutation, the last token to be routed permutes all
// pairs.  Row norms, logits, routes and the permutation are bit-identical to
// rmsnorm_rows + router_logits + route + permute (the same device functions,
// the same block size).  tickets: T + 1 zeroed ints, re-zeroed here.
constexpr int kFrontExperts = 8;  // one expert per warp: more CTAs share the router matrix

__global__ void __launch_bounds__(256) moe_front_kernel(
    const float* __restrict__ h, const float* __restrict__ w_norm, int D, float eps, const float* __restrict__ w_router,
    int E, const float* __restrict__ bias, int k, int scoring, int n_group, int topk_group, int norm_topk,
    float routed_scale, int n_extra, __nv_bfloat16* __restrict__ xn, float* __restrict__ logits,
    int32_t* __restrict__ ids, float* __restrict__ weights, int permute, int32_t* __restrict__ counts,
    int32_t* __restrict__ offsets, int32_t* __restrict__ dest, int32_t* __restrict__ src_pair,
    float* __restrict__ w_perm, int* __restrict__ tickets, int* __restrict__ status, EpPublishArgs pub) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  extern __shared__ float xs[];  // [D] normalised row, [E] logits, [E + n_extra] permute counts
  __shared__ float red[32];
  __shared__ int last;
  const int b = blockIdx.x, t = blockIdx.y, EB = gridDim.x, T = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* hr = h + (int64_t)t * D;
  const float inv = row_inv_rms(hr, D, true, eps, red);
  // (the element formula of rmsnorm_rows, four columns per thread and step)
#pragma unroll 2
  for (int i4 = threadIdx.x; i4 < D / 4; i4 += blockDim.x) {
    const float4 hv = reinterpret_cast<const float4*>(hr)[i4];
    const float4 wv = __ldg(reinterpret_cast<const float4*>(w_norm) + i4);
    float4 v;
    v.x = __fmul_rn(__fmul_rn(hv.x, inv), wv.x);
    v.y = __fmul_rn(__fmul_rn(hv.y, inv), wv.y);
    v.z = __fmul_rn(__fmul_rn(hv.z, inv), wv.z);
    v.w = __fmul_rn(__fmul_rn(hv.w, inv), wv.w);
    reinterpret_cast<float4*>(xs)[i4] = v;
    if (b == 0) {
      __nv_bfloat162 p2[2] = {__floats2bfloat162_rn(v.x, v.y), __floats2bfloat162_rn(v.z, v.w)};
      reinterpret_cast<uint2*>(xn + (int64_t)t * D)[i4] = *reinterpret_cast<const uint2*>(p2);
    }
  }
  __syncthreads();
  const int e1 = min(E, (b + 1) * kFrontExperts);
  for (int e = b * kFrontExperts + warp; e < e1; e += blockDim.x >> 5) {
    const float acc = router_dot(xs, w_router + (int64_t)e * D, D, lane);
    if (lane == 0) logits[(int64_t)t * E + e] = acc;
  }
  // the last CTA of this token routes it
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(&tickets[t], 1) == EB - 1;
    if (last) tickets[t] = 0;  // every CTA of the token has taken its ticket
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float* lg = xs + D;
  for (int e = threadIdx.x; e < E; e += blockDim.x) lg[e] = __ldcg(logits + (int64_t)t * E + e);
  __syncthreads();
  const int kk = k + n_extra;
  if (warp == 0)
    route_token(lg, bias, E, k, scoring, n_group, topk_group, norm_topk, routed_scale, ids + (int64_t)t * kk,
                weights + (int64_t)t * kk, n_extra, lane);
  if (!permute && !pub.enabled) return;
  // the last token to be routed permutes every pair (or, expert parallel,
  // writes the picks' slots and this rank's pick counts for the dispatch)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(&tickets[T], 1) == T - 1;
    if (last) tickets[T] = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  int32_t* cnt = reinterpret_cast<int32_t*>(lg + E);  // [E + n_extra]
  if (!permute) {
    if (warp == 0) ep_count_warp(ids, T * k, pub, status, cnt, lane);
    return;
  }
  int32_t* sids = cnt + E + n_extra;                   // [T * kk] ids, then their weights
  float* swts = reinterpret_cast<float*>(sids + T * kk);
  for (int i = threadIdx.x; i < T * kk; i += blockDim.x) {
    sids[i] = __ldcg(ids + i);
    swts[i] = __ldcg(weights + i);
  }
  __syncthreads();
  if (warp == 0)
    permute_warp(sids, T * kk, E + n_extra, counts, offsets, dest, src_pair, swts, w_perm, status, cnt, lane);
}

// out[p] = x[src_pair[p] / k] (bf16 rows, 16-byte vectors).
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int32_t* __restrict__ src,
                                   int k, int D, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int p = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(x + (int64_t)(src[p] / k) * ldx);
  uint4* d = reinterpret_cast<uint4*>(out + (int64_t)p * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) d[i] = s[i];
}

// Multi-block permute for large T*k, with the same result as permute_kernel:
// entries of one expert keep their input order.  Entries are cut into chunks
// of kPermChunk; pass 1 counts each chunk's experts, pass 2 turns the counts
// into per-chunk start positions (expert offset + entries of that expert in
// earlier chunks), pass 3 walks each chunk in order with one warp and ranks
// equal experts with match_any.
constexpr int kPermChunk = 1024;
constexpr int kPermSingleWarpMax = 4096;

__global__ void permute_count_kernel(const int32_t* __restrict__ ids, int N, int E, int32_t* __restrict__ hist,
                                     int* __restrict__ status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  extern __shared__ int32_t h[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int base = blockIdx.x * kPermChunk;
  for (int i = threadIdx.x; i < kPermChunk && base + i < N; i += blockDim.x) {
    const int e = ids[base + i];
    if ((unsigned)e < (unsigned)E) atomicAdd(&h[e], 1);
    else atomicExch(status, kStatusBadInput);  // out-of-range id: flagged, entry dropped
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(int64_t)blockIdx.x * E + e] = h[e];
}

__global__ void permute_scan_kernel(int32_t* __restrict__ hist, int chunks, int E, int32_t* __restrict__ counts,
                                    int32_t* __restrict__ offsets) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  extern __shared__ int32_t tot[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int v = 0;
    for (int c = 0; c < chunks; ++c) v += hist[(int64_t)c * E + e];
    tot[e] = v;
    counts[e] = v;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // exclusive scan of the totals over experts, 32 at a time
    const int lane = threadIdx.x;
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int v = e < E ? tot[e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (e < E) tot[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) offsets[E] = carry;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = tot[e];
    offsets[e] = run;
    for (int c = 0; c < chunks; ++c) {
      const int v = hist[(int64_t)c * E + e];
      hist[(int64_t)c * E + e] = run;
      run += v;
    }
  }
}

__global__ void permute_scatter_kernel(const int32_t* __restrict__ ids, int N, int E, const int32_t* __restrict__ hist,
                                       int32_t* __restrict__ dest, int32_t* __restrict__ src_pair,
                                       const float* __restrict__ weights, float* __restrict__ w_perm) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  extern __shared__ int32_t cur[];
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) cur[e] = hist[(int64_t)blockIdx.x * E + e];
  __syncwarp();
  const int base = blockIdx.x * kPermChunk;
  const int end = min(N, base + kPermChunk);
  for (int c = base; c < end; c += 32) {
    const int i = c + lane;
    int e = i < end ? ids[i] : -1 - lane;
    if ((unsigned)e >= (unsigned)E) e = -1 - lane;
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(grp & ((1u << lane) - 1u));
    const int pos = e >= 0 ? cur[e] + rank : 0;
    __syncwarp();
    if (e >= 0) {
      dest[i] = pos;
      src_pair[pos] = i;
      if (w_perm != nullptr) w_perm[pos] = weights[i];
    }
    if (e >= 0 && rank == 0) cur[e] += __popc(grp);
    __syncwarp();
  }
}

// h[t] += (y[dest[t*k]] + ... + y[dest[t*k+k-1]]) + shared[t]: the order of
// moe_step's accumulation (ops.cpp:133-145) followed by the residual add
// (model.cpp:209).
constexpr int kMaxCombinePicks = 32;  // k + shared groups per token

__global__ void moe_combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ dest, int k, int D,
                                   const float* __restrict__ shared, float* __restrict__ h,
                                   const float* __restrict__ w_next, float eps, __nv_bfloat16* __restrict__ xn_next) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ float red[32];
  __shared__ const float4* rows[kMaxCombinePicks];  // the token's pick rows, looked up once
  const int t = blockIdx.x;
  if ((int)threadIdx.x < k) rows[threadIdx.x] = reinterpret_cast<const float4*>(y + (int64_t)dest[(int64_t)t * k + threadIdx.x] * D);
  __syncthreads();
  auto pick = [&](int j, int i4) { return rows[j][i4]; };
  combine_row(pick, k, D, shared ? shared + (int64_t)t * D : nullptr, shared ? 1 : 0, 0, h + (int64_t)t * D, w_next,
              eps, xn_next ? xn_next + (int64_t)t * D : nullptr, red);
}

// Greedy id per row: first index of the maximum (argmax_f32, math.cpp:29-40).
__global__ void argmax_rows_kernel(const float* __restrict__ logits, int64_t ld, int V, int32_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* row = logits + blockIdx.x * ld;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = row[i];
    if (x > v || (x == v && i < idx)) {  // NaN never wins, like the reference's '>'
      v = x;
      idx = i;
    }
  }
  warp_argmax(v, idx);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = v;
    si[w] = idx;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    v = l < nw ? sv[l] : -INFINITY;
    idx = l < nw ? si[l] : 0x7fffffff;
    warp_argmax(v, idx);
    if (l == 0) out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
  }
}

// h[b] = embedding row of token[b] as fp32 (embedding_lookup_f32,
// src/hf/weight_ops.cpp:37-65).
__global__ void embed_kernel(const void* __restrict__ table, int bf16, const int32_t* __restrict__ tokens, int D,
                             float* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int b = blockIdx.x;
  const int64_t row = tokens[b];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    h[(int64_t)b * D + i] = bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(table)[row * D + i])
                                 : static_cast<const float*>(table)[row * D + i];
  }
}

int launched(dsb_ctx* ctx) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ctx, DSB_ECUDA, "kernel launch: %s", cudaGetErrorString(e));
  ctx->stats.kernel_launches++;
  return DSB_OK;
}

}  // namespace

int rmsnorm_rows(dsb_ctx* ctx, const float* x, int64_t ldx, const float* w, int rows, int n, float eps,
                 void* y_bf16, int64_t ldyb, float* y_f32, int64_t ldyf) {
  launch_pdl(rmsnorm_rows_kernel, rows, 256, 0, ctx->stream, x, ldx, w, n, eps, static_cast<__nv_bfloat16*>(y_bf16), ldyb,
                                                     y_f32, ldyf);
  return launched(ctx);
}

int kv_norm_rope_append(dsb_ctx* ctx, const float* kv_a, int64_t ld_kv, const float* w_norm, const void* q,
                        const float* qf, int64_t ld_qf, void* q_out, const int32_t* pos, const int32_t* block_table,
                        int max_blocks, int B, int H, int nope, int R, int P, float eps, float theta, void* cache,
                        void* q_rope) {
  // the latent row in CTA (b, 0), the query's heads over 1..8 more CTAs per token
  const int qparts = std::min(8, std::max(1, H / 8));
  launch_pdl(kv_norm_rope_append_kernel, dim3((unsigned)B, (unsigned)(1 + qparts)), 256, 0, ctx->stream, kv_a, ld_kv,
             w_norm,
             static_cast<const __nv_bfloat16*>(q), qf, ld_qf, static_cast<__nv_bfloat16*>(q_out), pos, block_table,
             max_blocks, H, nope, R, P, eps, theta, static_cast<__nv_bfloat16*>(cache),
             static_cast<__nv_bfloat16*>(q_rope));
  return launched(ctx);
}

int router_logits(dsb_ctx* ctx, const float* x, const float* w, int T, int D, int E, float* logits) {
  const int warps = T * E;
  if (T > 64) {
    const dim3 grid((E + kRtE - 1) / kRtE, (T + kRtT - 1) / kRtT);
    launch_pdl(router_logits_tiled_kernel, grid, 256, 0, ctx->stream, x, w, T, D, E, logits);
    return launched(ctx);
  }
  launch_pdl(router_logits_kernel, (warps + 7) / 8, 256, 0, ctx->stream, x, w, T, D, E, logits);
  return launched(ctx);
}

bool moe_front_fits(int T, int D, int E, int N) {
  // every CTA of a token re-reads nothing but its 16 router rows; the whole
  // router matrix is read once per token from L2, so the fused front is for
  // decode batches with a small router (the single-warp permutation bounds N)
  return T >= 1 && (D % 4) == 0 && E <= 256 && N <= kPermSingleWarpMax &&
         (double)T * E * D * 4.0 <= 32.0 * (1 << 20);
}

int moe_front(dsb_ctx* ctx, const float* h, const float* w_norm, int T, int D, float eps, const float* w_router,
              int E, const float* bias, int k, int scoring, int n_group, int topk_group, int norm_topk,
              float routed_scale, int n_extra, void* xn, float* logits, int32_t* ids, float* weights, int permute,
              int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* src_pair, float* w_perm,
              const EpPublishArgs* pub) {
  EpPublishArgs none{};
  if (pub != nullptr && (permute || n_extra != 0))
    return fail(ctx, DSB_EINVAL, "moe_front: publishing expert-parallel counts needs permute = 0 and no extra groups");
  int rc = ensure_counters(ctx, kTicketFront + T + 1);
  if (rc != DSB_OK) return rc;
  const size_t smem = (size_t)(D + E + E + n_extra + 2 * T * (k + n_extra)) * sizeof(float);
  if (smem > 48 * 1024) {
    static std::atomic<bool> attr_set[kMaxDevices];
    if (int rc2 = smem_attr_once(ctx, moe_front_kernel, 200 * 1024, attr_set); rc2 != DSB_OK) return rc2;
  }
  const dim3 grid((E + kFrontExperts - 1) / kFrontExperts, T);
  launch_pdl(moe_front_kernel, grid, 256, smem, ctx->stream, h, w_norm, D, eps, w_router, E, bias, k, scoring, n_group,
             topk_group, norm_topk, routed_scale, n_extra, static_cast<__nv_bfloat16*>(xn), logits, ids, weights,
             permute, counts, offsets, dest, src_pair, w_perm, ctx->counters + kTicketFront, ctx->d_status,
             pub != nullptr ? *pub : none);
  return launched(ctx);
}

int moe_route(dsb_ctx* ctx, const float* logits, const float* bias, int T, int E, int k, int scoring, int n_group,
              int topk_group, int norm_topk, float routed_scale, int32_t* ids, float* weights, int n_extra,
              const EpPublishArgs* pub) {
  EpPublishArgs none{};
  if (pub != nullptr && n_extra != 0)
    return fail(ctx, DSB_EINVAL, "moe_route: publishing expert-parallel counts needs no extra groups");
  int rc = ensure_counters(ctx, kTicketRoute + 1);
  if (rc != DSB_OK) return rc;
  launch_pdl(route_kernel, (T + 7) / 8, 256, 0, ctx->stream, logits, bias, T, E, k, scoring, n_group, topk_group,
             norm_topk, routed_scale, ids, weights, n_extra, pub != nullptr ? *pub : none,
             ctx->counters + kTicketRoute, ctx->d_status);
  return launched(ctx);
}

int moe_permute(dsb_ctx* ctx, const int32_t* ids, int N, int E, int32_t* counts, int32_t* offsets, int32_t* dest,
                int32_t* src_pair, const float* weights, float* w_perm) {
  if (N <= kPermSingleWarpMax) {
    launch_pdl(permute_kernel, 1, 32, (E + 2 * N) * sizeof(int32_t), ctx->stream, ids, N, E, counts, offsets, dest, src_pair, weights,
                                                                 w_perm, ctx->d_status);
    return launched(ctx);
  }
  // large batches: per-chunk histograms, one scan, stable per-chunk scatter
  const int chunks = (N + kPermChunk - 1) / kPermChunk;
  int rc = ensure_buffer(ctx, &ctx->perm, &ctx->perm_bytes, (size_t)chunks * E * sizeof(int32_t), 64 << 10,
                         "permute histogram");
  if (rc != DSB_OK) return rc;
  int32_t* hist = static_cast<int32_t*>(ctx->perm);
  const size_t sh = (size_t)E * sizeof(int32_t);
  launch_pdl(permute_count_kernel, chunks, 256, sh, ctx->stream, ids, N, E, hist, ctx->d_status);
  rc = launched(ctx);
  if (rc != DSB_OK) return rc;
  launch_pdl(permute_scan_kernel, 1, 1024, sh, ctx->stream, hist, chunks, E, counts, offsets);
  rc = launched(ctx);
  if (rc != DSB_OK) return rc;
  launch_pdl(permute_scatter_kernel, chunks, 32, sh, ctx->stream, ids, N, E, hist, dest, src_pair, weights, w_perm);
  return launched(ctx);
}

int gather_rows(dsb_ctx* ctx, const void* x, int64_t ldx, const int32_t* src_pair, int n_pairs, int k, int D,
                void* out) {
  launch_pdl(gather_rows_kernel, n_pairs, 128, 0, ctx->stream, static_cast<const __nv_bfloat16*>(x), ldx, src_pair, k, D,
                                                       static_cast<__nv_bfloat16*>(out));
  return launched(ctx);
}

int moe_combine(dsb_ctx* ctx, const float* y, const int32_t* dest, int T, int k, int D, const float* shared,
                float* h, const float* w_next, float eps, void* xn_next) {
  if (k > kMaxCombinePicks || (D % 4) != 0)
    return fail(ctx, DSB_EINVAL, "moe_combine: k=%d (at most %d) or D=%d (a multiple of 4)", k, kMaxCombinePicks, D);
  launch_pdl(moe_combine_kernel, T, combine_threads(D), 0, ctx->stream, y, dest, k, D, shared, h, w_next, eps,
             static_cast<__nv_bfloat16*>(xn_next));
  return launched(ctx);
}

int argmax_rows(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, int32_t* out) {
  launch_pdl(argmax_rows_kernel, B, 1024, 0, ctx->stream, logits, ld, V, out);
  return launched(ctx);
}

int embed(dsb_ctx* ctx, const void* table, int bf16, const int32_t* tokens, int B, int D, float* h) {
  launch_pdl(embed_kernel, B, 256, 0, ctx->stream, table, bf16, tokens, D, h);
  return launched(ctx);
}

}  // namespace dsb

// ------------------------------------------------------------------ C ABI

extern "C" int dsb_rmsnorm(dsb_ctx* ctx, const float* x, int64_t ldx, const float* w, int rows, int n, float eps,
                           void* y_bf16, int64_t ldy_bf16, float* y_f32, int64_t ldy_f32) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (x == nullptr || w == nullptr || rows <= 0 || n <= 0 || (y_bf16 == nullptr && y_f32 == nullptr))
    return dsb::fail(ctx, DSB_EINVAL, "dsb_rmsnorm: bad arguments");
  return dsb::rmsnorm_rows(ctx, x, ldx, w, rows, n, eps, y_bf16, ldy_bf16, y_f32, ldy_f32);
}

extern "C" int dsb_kv_norm_rope_append(dsb_ctx* ctx, const float* kv_a, const float* w_norm, const void* q,
                                       const int32_t* positions, const int32_t* block_table, int max_blocks, int B,
                                       int H, int nope, int R, int P, float eps, float theta, void* cache,
                                       void* q_rope) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (kv_a == nullptr || w_norm == nullptr || q == nullptr || positions == nullptr || block_table == nullptr ||
      cache == nullptr || q_rope == nullptr || B <= 0 || H <= 0 || R <= 0 || P <= 0 || (P % 2) != 0 || P > 128)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_kv_norm_rope_append: bad arguments");
  return dsb::kv_norm_rope_append(ctx, kv_a, R + P, w_norm, q, nullptr, 0, nullptr, positions, block_table,
                                  max_blocks, B, H, nope, R, P, eps, theta, cache, q_rope);
}

extern "C" int dsb_router_logits(dsb_ctx* ctx, const float* x, const float* w, int T, int D, int E, float* logits) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (x == nullptr || w == nullptr || logits == nullptr || T <= 0 || E <= 0 || D <= 0 || (D % 4) != 0)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_router_logits: bad arguments (D must be a multiple of 4)");
  return dsb::router_logits(ctx, x, w, T, D, E, logits);
}

extern "C" int dsb_moe_route(dsb_ctx* ctx, const float* logits, const float* bias, int T, int E, int k, int scoring,
                             int n_group, int topk_group, int norm_topk, float routed_scale, int32_t* ids,
                             float* weights) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (logits == nullptr || ids == nullptr || weights == nullptr || T <= 0 || E <= 0 || E > 256 || k < 1 || k > 8 ||
      k > E)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_moe_route: bad arguments (E <= 256, 1 <= k <= 8)");
  if (scoring == DSB_SCORE_SIGMOID) {
    if (bias == nullptr || n_group < 1 || n_group > 32 || E % n_group != 0 || topk_group < 1 ||
        topk_group > n_group || k > topk_group * (E / n_group))
      return dsb::fail(ctx, DSB_EINVAL, "dsb_moe_route: bad grouped-router arguments");
  } else if (scoring != DSB_SCORE_SOFTMAX) {
    return dsb::fail(ctx, DSB_EINVAL, "dsb_moe_route: unknown scoring %d", scoring);
  }
  return dsb::moe_route(ctx, logits, bias, T, E, k, scoring, n_group, topk_group, norm_topk, routed_scale, ids,
                        weights, 0);
}

extern "C" int dsb_moe_permute(dsb_ctx* ctx, const int32_t* ids, int T, int k, int E, int32_t* counts,
                               int32_t* offsets, int32_t* dest, int32_t* src_pair, const float* weights,
                               float* w_perm) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (ids == nullptr || counts == nullptr || offsets == nullptr || dest == nullptr || src_pair == nullptr || T <= 0 ||
      k <= 0 || E <= 0 || E > 4096)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_moe_permute: bad arguments");
  if ((weights == nullptr) != (w_perm == nullptr))
    return dsb::fail(ctx, DSB_EINVAL, "dsb_moe_permute: weights and w_perm go together");
  return dsb::moe_permute(ctx, ids, T * k, E, counts, offsets, dest, src_pair, weights, w_perm);
}

extern "C" int dsb_gather_rows(dsb_ctx* ctx, const void* x, int64_t ldx, const int32_t* src_pair, int n_pairs, int k,
                               int D, void* out) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (x == nullptr || src_pair == nullptr || out == nullptr || n_pairs <= 0 || k <= 0 || D <= 0 || (D % 8) ||
      (ldx % 8))
    return dsb::fail(ctx, DSB_EINVAL, "dsb_gather_rows: bad arguments (D, ldx multiples of 8)");
  return dsb::gather_rows(ctx, x, ldx, src_pair, n_pairs, k, D, out);
}

extern "C" int dsb_moe_combine(dsb_ctx* ctx, const float* y, const int32_t* dest, int T, int k, int D,
                               const float* shared, float* h) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (y == nullptr || dest == nullptr || h == nullptr || T <= 0 || k <= 0 || D <= 0)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_moe_combine: bad arguments");
  return dsb::moe_combine(ctx, y, dest, T, k, D, shared, h);
}

extern "C" int dsb_argmax(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, int32_t* out) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (logits == nullptr || out == nullptr || B <= 0 || V <= 0 || ld < V)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_argmax: bad arguments");
  return dsb::argmax_rows(ctx, logits, ld, B, V, out);
}

extern "C" int dsb_embed(dsb_ctx* ctx, const void* table, int table_bf16, const int32_t* tokens, int B, int D,
                         float* h) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (table == nullptr || tokens == nullptr || h == nullptr || B <= 0 || D <= 0)
    return dsb::fail(ctx, DSB_EINVAL, "dsb_embed: bad arguments");
  return dsb::embed(ctx, table, table_bf16, tokens, B, D, h);
}
