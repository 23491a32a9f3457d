// Stochastic sampling of token ids on the device: ds::core::Sampler::sample
// (src/core/sampler.cpp:23-77) for B logits rows at once, one CTA per row.
//
// Per row, as the reference does it:
//   x_i = logit_i / t                                   (t <= 0 reads as 1)
//   top-k (0 < k < V): keep the k largest x            (sampler.cpp:35-40)
//   p = softmax over the kept items                     (sampler.cpp:42-47)
//   top-p (0 < top_p < 1): in descending-p order keep the shortest prefix whose
//     mass reaches top_p, the item that reaches it included, and renormalise
//     (sampler.cpp:49-67)
//   return the first item, in scan order, at which the cumulative mass
//   reaches the caller's uniform draw u in [0, 1)      (sampler.cpp:69-76)
// Scan order: with no filter active the items stay in id order, as in the
// reference.  With a filter the reference's order comes from std::nth_element
// and std::sort and is unspecified; here it is descending x with ties to the
// lower id, one of the orders those can produce.  Ties at the top-k boundary
// keep the lower ids.
//
// Nothing is sorted.  Each cut is a radix select over order-preserving 32-bit
// keys of x (three passes of 11/11/10 bits, histograms in shared memory),
// weighted by counts (the top-k cut) or by probability mass (the top-p cut
// and the draw).  Masses are fixed point, q = round(p * 2^40) in uint64, so
// the shared-memory atomic sums do not depend on the order the atomics land
// in: a row's result is deterministic.  Rank among equal keys is kept in id
// order by giving each warp a contiguous segment of the row that it walks in
// 32-element steps (ballot + popc).  The row is re-read (from L2) on every
// pass: at most 14 passes for the filtered case, 3 and a one-warp walk
// unfiltered.

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

namespace dsb {
namespace {

using u64 = unsigned long long;

constexpr int kThreads = 1024, kWarps = kThreads / 32, kBins = 2048;
constexpr double kFix = 1099511627776.0;  // 2^40: fixed-point unit of probability mass

__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleSmem {
  u64 hist[kBins];
  u64 wval[kWarps];    // per-warp partial sums / counts
  u64 wbase[kWarps];   // their exclusive prefix
  float fred[kWarps];
  u64 sel_excl, target;
  int sel_bin, sel_warp;
  int out_id;
};

// The cuts of one row, as each warp sees its own segment.
struct RowView {
  const float* row;
  int seg0, seg1;  // this warp's items [seg0, seg1)
  float t;
  bool fk, fp;     // top-k / top-p cut active
  uint32_t Kk, Kp;
  int need_k, need_p;  // how many items with the cut's key survive it (lowest ids first)
  int base_k, base_p;
};

// f(i, x, key, in, keep) for every lane of every 32-item step of this warp's
// segment, in id order; keep = the item survives the active cuts.  All 32
// lanes take part (ballots); lanes past the segment get in = keep = false.
template <class F>
__device__ __forceinline__ void walk(const RowView& r, F f) {
  const uint32_t lane = threadIdx.x & 31, lt = (1u << lane) - 1u;
  int run_k = r.base_k, run_p = r.base_p;
  for (int i0 = r.seg0; i0 < r.seg1; i0 += 32) {
    const int i = i0 + (int)lane;
    const bool in = i < r.seg1;
    const float x = in ? __fdiv_rn(r.row[i], r.t) : -INFINITY;
    const uint32_t key = fkey(x);
    bool keep = in;
    if (r.fk) {
      const bool eq = in && key == r.Kk;
      const uint32_t b = __ballot_sync(0xffffffffu, eq);
      const int rank = run_k + __popc(b & lt);
      run_k += __popc(b);
      keep = in && (key > r.Kk || (eq && rank < r.need_k));
    }
    if (r.fp) {
      const bool eq = keep && key == r.Kp;
      const uint32_t b = __ballot_sync(0xffffffffu, eq);
      const int rank = run_p + __popc(b & lt);
      run_p += __popc(b);
      keep = keep && (key > r.Kp || (eq && rank < r.need_p));
    }
    f(i, x, key, in, keep);
  }
}

__device__ __forceinline__ u64 warp_incl_scan(u64 v) {
  const uint32_t lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const u64 y = __shfl_up_sync(0xffffffffu, v, o);
    if ((int)lane >= o) v += y;
  }
  return v;
}

// Exclusive prefix over the block's threads (in thread order); also returns the total.
__device__ u64 block_excl_scan(SampleSmem& s, u64 v, u64* total) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const u64 incl = warp_incl_scan(v);
  if (lane == 31) s.wval[w] = incl;
  __syncthreads();
  if (w == 0) {
    const u64 t = s.wval[lane];
    const u64 ti = warp_incl_scan(t);
    s.wbase[lane] = ti - t;
    if (lane == 31) s.target = ti;  // block total (s.target is free here)
  }
  __syncthreads();
  const u64 r = s.wbase[w] + incl - v;
  *total = s.target;
  __syncthreads();
  return r;
}

// Per-warp values -> each warp's exclusive prefix in s.wbase and the total.
__device__ u64 warps_excl_scan(SampleSmem& s, u64 mine) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s.wval[w] = mine;
  __syncthreads();
  if (w == 0) {
    const u64 t = s.wval[lane];
    const u64 ti = warp_incl_scan(t);
    s.wbase[lane] = ti - t;
    if (lane == 31) s.target = ti;
  }
  __syncthreads();
  const u64 total = s.target;
  __syncthreads();
  return total;
}

// Deterministic block reductions (fixed shuffle tree, then warp 0 over the warps).
__device__ float block_max(SampleSmem& s, float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s.fred[w] = v;
  __syncthreads();
  v = s.fred[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  return v;
}

__device__ float block_sum(SampleSmem& s, float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s.fred[w] = v;
  __syncthreads();
  v = s.fred[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  return v;
}

struct Selected {
  uint32_t key;  // key of the item at which the cumulative weight reaches the target
  u64 rem;       // target minus the weight of the candidates with a larger key (>= 1)
  u64 total;     // weight of all candidates
};

// Among the candidates (keep == true), taken in descending key order, find
// the item at which the cumulative weight first reaches the target: `target`
// itself, or with frac >= 0 max(1, ceil(frac * total)).  weight(x, key) is
// the candidate's weight (1 for counts, its fixed-point mass otherwise).
template <class Wt>
__device__ Selected radix_select(SampleSmem& s, const RowView& r, Wt weight, u64 target, double frac) {
  uint32_t prefix = 0;
  int have = 0;
  u64 rem = target, total = 0;
  for (int pass = 0; pass < 3; ++pass) {
    const int bits = pass < 2 ? 11 : 10, nb = 1 << bits, shift = 32 - have - bits;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) s.hist[b] = 0;
    __syncthreads();
    walk(r, [&](int, float x, uint32_t key, bool, bool keep) {
      if (keep && (have == 0 || (key >> (32 - have)) == prefix))
        atomicAdd(&s.hist[(key >> shift) & (uint32_t)(nb - 1)], weight(x, key));
    });
    __syncthreads();
    // descending bins: thread t holds bins nb-1-2t and nb-2-2t
    const int j0 = 2 * (int)threadIdx.x, b0 = nb - 1 - j0, b1 = nb - 2 - j0;
    const u64 h0 = b0 >= 0 ? s.hist[b0] : 0, h1 = b1 >= 0 ? s.hist[b1] : 0;
    u64 group = 0;
    const u64 excl = block_excl_scan(s, h0 + h1, &group);
    if (pass == 0) {
      total = group;
      if (frac >= 0.0) {
        const double c = ceil(frac * (double)total);
        rem = c < 1.0 ? 1ull : (c > (double)total ? total : (u64)c);
      }
    }
    if (threadIdx.x == 0) {
      s.sel_bin = 0;
      s.sel_excl = 0;
    }
    __syncthreads();
    if (b0 >= 0 && excl < rem && rem <= excl + h0) {
      s.sel_bin = b0;
      s.sel_excl = excl;
    } else if (b1 >= 0 && excl + h0 < rem && rem <= excl + h0 + h1) {
      s.sel_bin = b1;
      s.sel_excl = excl + h0;
    }
    __syncthreads();
    prefix = (prefix << bits) | (uint32_t)s.sel_bin;
    have += bits;
    rem -= s.sel_excl;
    __syncthreads();
  }
  return {prefix, rem, total};
}

// Items of this warp's segment that are candidates with key == K, counted per
// warp; returns each warp's exclusive prefix (items before its segment).
__device__ int eq_base(SampleSmem& s, const RowView& r, uint32_t K) {
  int n = 0;
  walk(r, [&](int, float, uint32_t key, bool, bool keep) {
    n += __popc(__ballot_sync(0xffffffffu, keep && key == K));
  });
  warps_excl_scan(s, (u64)n);
  return (int)s.wbase[threadIdx.x >> 5];
}

__global__ void __launch_bounds__(kThreads) sample_rows_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                               float t, int top_k, float top_p,
                                                               const float* __restrict__ uniforms,
                                                               int32_t* __restrict__ out) {
  pdl_wait();
  __shared__ SampleSmem s;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = ((V + kThreads - 1) / kThreads) * 32;  // warp segment, a multiple of 32
  RowView r{};
  r.row = logits + (int64_t)blockIdx.x * ld;
  r.seg0 = min(V, w * S);
  r.seg1 = min(V, r.seg0 + S);
  r.t = t;
  const float u = uniforms[blockIdx.x];
  if (threadIdx.x == 0) s.out_id = 0;

  // max of x: the top-k survivors always include it, so it is the softmax's max
  float mx = -INFINITY;
  walk(r, [&](int, float x, uint32_t, bool in, bool) {
    if (in) mx = fmaxf(mx, x);
  });
  mx = block_max(s, mx);

  const bool fk = top_k > 0 && top_k < V, fp = top_p > 0.0f && top_p < 1.0f;
  if (fk) {
    const Selected c = radix_select(s, r, [](float, uint32_t) { return 1ull; }, (u64)top_k, -1.0);
    r.Kk = c.key;
    r.need_k = (int)c.rem;
    r.base_k = eq_base(s, r, c.key);  // r.fk is still off: counts every item with the key
    r.fk = true;
  }

  // softmax over the survivors: p = exp(x - max) * (1 / sum)   (math.cpp:15-27)
  float sum = 0.0f;
  walk(r, [&](int, float x, uint32_t, bool, bool keep) {
    if (keep) sum += expf(x - mx);
  });
  sum = block_sum(s, sum);
  const float inv = 1.0f / sum;
  auto mass = [&](float x, uint32_t) -> u64 { return __double2ull_rn((double)(expf(x - mx) * inv) * kFix); };

  if (!fk && !fp) {
    // id order: per-warp mass, then the warp holding the draw walks its segment
    u64 m = 0;
    walk(r, [&](int, float x, uint32_t key, bool in, bool) {
      if (in) m += mass(x, key);
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
    const u64 total = warps_excl_scan(s, m);
    const double c = ceil((double)u * (double)total);
    const u64 R = c < 1.0 ? 1ull : (c > (double)total ? total : (u64)c);
    if (threadIdx.x == 0) s.sel_warp = -1;
    __syncthreads();
    if (lane == 0 && s.wbase[w] < R && R <= s.wbase[w] + s.wval[w]) s.sel_warp = w;
    __syncthreads();
    if (w == s.sel_warp) {
      u64 run = s.wbase[w];
      bool found = false;
      walk(r, [&](int i, float x, uint32_t key, bool in, bool) {
        const u64 q = in ? mass(x, key) : 0ull;
        const u64 incl = run + warp_incl_scan(q);
        const uint32_t hit = __ballot_sync(0xffffffffu, in && !found && incl >= R);
        if (hit != 0u && !found) {
          if ((int)lane == __ffs(hit) - 1) s.out_id = i;
          found = true;
        }
        run = __shfl_sync(0xffffffffu, incl, 31);
      });
    }
    __syncthreads();
  } else {
    if (fp) {
      const Selected c = radix_select(s, r, mass, 0, (double)top_p);
      const u64 q = mass(key_to_float(c.key), c.key);
      r.Kp = c.key;
      r.need_p = q > 0 ? (int)((c.rem + q - 1) / q) : 0;
      r.base_p = eq_base(s, r, c.key);  // r.fp still off: survivors of the top-k cut with the key
      r.fp = true;
    }
    // the draw: the item at which the survivors' mass, in descending order, reaches u * total
    const Selected d = radix_select(s, r, mass, 0, (double)u);
    const u64 qd = mass(key_to_float(d.key), d.key);
    const int m = qd > 0 ? (int)((d.rem + qd - 1) / qd) : 1;  // the m-th survivor with this key, in id order
    const int base = eq_base(s, r, d.key);
    const int n = (int)s.wval[w];  // this warp's count, left by eq_base
    if (threadIdx.x == 0) s.sel_warp = -1;
    __syncthreads();
    if (lane == 0 && base < m && m <= base + n) s.sel_warp = w;
    __syncthreads();
    if (w == s.sel_warp) {
      int run = base;
      walk(r, [&](int i, float, uint32_t key, bool, bool keep) {
        const uint32_t b = __ballot_sync(0xffffffffu, keep && key == d.key);
        const int c = __popc(b);
        if (run < m && m <= run + c) {
          // the (m - run)-th set lane of b
          uint32_t bb = b;
          for (int j = 1; j < m - run; ++j) bb &= bb - 1u;
          if ((int)lane == __ffs(bb) - 1) s.out_id = i;
        }
        run += c;
      });
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = s.out_id;
}

}  // namespace

int sample_rows(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, float temperature, int top_k, float top_p,
                const float* uniforms, int32_t* out) {
  const float t = temperature <= 0.0f ? 1.0f : temperature;
  DSB_CUDA_TRY(ctx, launch_pdl(sample_rows_kernel, B, kThreads, 0, ctx->stream, logits, ld, V, t, top_k, top_p,
                               uniforms, out));
  ctx->stats.kernel_launches++;
  return DSB_OK;
}

}  // namespace dsb

extern "C" int dsb_sample(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, float temperature, int top_k,
                          float top_p, const float* uniforms, int32_t* out_ids) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (logits == nullptr || uniforms == nullptr || out_ids == nullptr || B <= 0 || V <= 0 || ld < V ||
      !(temperature == temperature) || !(top_p == top_p))
    return dsb::fail(ctx, DSB_EINVAL, "dsb_sample: bad arguments");
  return dsb::sample_rows(ctx, logits, ld, B, V, temperature, top_k, top_p, uniforms, out_ids);
}
