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
// keys of x (four passes of 8 bits), weighted by counts (the top-k cut) or
// by probability mass (the top-p cut and the draw), all in 32-bit shared
// counters (a mass in two: its high and low 16 bits).  Masses are fixed point,
// q = round(p * 2^40) in uint64, so the shared-memory atomic sums do not
// depend on the order the atomics land in: a row's result is deterministic.
// The histogram has one column per lane (256 bins x 32 lanes x 2, 64 KB), so
// lanes of a warp never collide on an address even when their keys share a
// bin.  Rank among equal keys is kept in id order by giving each warp a
// contiguous segment of the row that it walks 32 items at a time (ballot +
// popc), four loads ahead; ranks are only computed when a cut splits a run
// of equal keys, and every other pass loads float4s in no particular order.  The row is re-read from L2 on every pass (at most 17 with
// both cuts, 3 with none).  A top-k cut of at most 1024 items, or a top-p
// nucleus of at most 1024, is instead gathered into shared memory, sorted,
// and drawn from there in the reference's float order (5 passes for top-k,
// 8 for top-p).

#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

namespace dsb {
namespace {

using u64 = unsigned long long;

constexpr int kThreads = 1024, kWarps = kThreads / 32, kBins = 256, kAhead = 4, kAheadVec = 2, kCompactMax = 1024;
constexpr size_t kHistBytes = (size_t)kBins * 32 * sizeof(unsigned long long);  // dynamic shared memory
constexpr double kFix = 1099511627776.0;  // 2^40: fixed-point unit of probability mass

__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleSmem {
  u64 bins[kBins];     // a pass's histogram, lane columns summed
  u64 wval[kWarps];    // per-warp partial sums / counts
  u64 wbase[kWarps];   // their exclusive prefix
  float fred[kWarps];
  u64 sel_excl, sel_h, target;
  int sel_bin, sel_warp;
  int out_id;
  int ncomp;
};

__device__ __forceinline__ u64* hist_cols() {
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  return reinterpret_cast<u64*>(dyn_smem);  // [kBins][32]
}

// The cuts of one row, as each warp sees its own segment.
struct RowView {
  const float* row;
  int seg0, seg1;  // this warp's items [seg0, seg1)
  float t;
  bool vec;        // row 16-byte aligned: unordered walks load float4
  bool fk, fp;     // top-k / top-p cut active
  uint32_t Kk, Kp;
  int need_k, need_p;  // how many items with the cut's key survive it (lowest ids first)
  int base_k, base_p;
};

// Ordered walk: f(i, x, key, in, keep) for every lane of every 32-item step
// of this warp's segment, in id order; keep = the item survives the active
// cuts.  All 32 lanes take part (ballots); lanes past the segment get
// in = keep = false.
template <class F>
__device__ __forceinline__ void walk_ordered(const RowView& r, F f) {
  const uint32_t lane = threadIdx.x & 31, lt = (1u << lane) - 1u;
  int run_k = r.base_k, run_p = r.base_p;
  for (int i0 = r.seg0; i0 < r.seg1; i0 += 32 * kAhead) {
    float v[kAhead];
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
      const int i = i0 + j * 32 + (int)lane;
      v[j] = i < r.seg1 ? __ldg(r.row + i) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
      const int i = i0 + j * 32 + (int)lane;
      const bool in = i < r.seg1;
      const float x = in ? (r.t == 1.0f ? v[j] : __fdiv_rn(v[j], r.t)) : -INFINITY;
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
}

__device__ __forceinline__ bool ranked(const RowView& r) {
  return (r.fk && r.need_k != 0x7fffffff) || (r.fp && r.need_p != 0x7fffffff);
}

// Unordered walk: f for every item of the segment, in no particular order
// (each lane takes four consecutive items per 128-item step, loaded as one
// float4, kAheadVec steps ahead).  Every lane makes the same number of calls, so
// f may use warp votes, but not id order.  Falls back to the ordered walk
// when a cut must rank equal keys or the row is not 16-byte aligned.
template <class F>
__device__ __forceinline__ void walk(const RowView& r, F f) {
  if (!r.vec || ranked(r)) {
    walk_ordered(r, f);
    return;
  }
  const int lane = threadIdx.x & 31;
  for (int i0 = r.seg0; i0 < r.seg1; i0 += 128 * kAheadVec) {
    float4 v[kAheadVec];
#pragma unroll
    for (int j = 0; j < kAheadVec; ++j) {
      const int i = i0 + j * 128 + 4 * lane;
      if (i + 3 < r.seg1) {
        v[j] = __ldg(reinterpret_cast<const float4*>(r.row + i));
      } else {
        v[j].x = i < r.seg1 ? __ldg(r.row + i) : 0.0f;
        v[j].y = i + 1 < r.seg1 ? __ldg(r.row + i + 1) : 0.0f;
        v[j].z = i + 2 < r.seg1 ? __ldg(r.row + i + 2) : 0.0f;
        v[j].w = 0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < kAheadVec; ++j) {
      const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = i0 + j * 128 + 4 * lane + c;
        const bool in = i < r.seg1;
        const float x = in ? (r.t == 1.0f ? e[c] : __fdiv_rn(e[c], r.t)) : -INFINITY;
        const uint32_t key = fkey(x);
        const bool keep = in && (!r.fk || key >= r.Kk) && (!r.fp || key >= r.Kp);
        f(i, x, key, in, keep);
      }
    }
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
  u64 eq;        // weight of the candidates with this key
};

// Among the candidates (keep == true), taken in descending key order, find
// the item at which the cumulative weight first reaches the target: `target`
// itself, or with frac >= 0 max(1, ceil(frac * total)).  weight(x, key) is
// the candidate's weight (1 for counts, its fixed-point mass otherwise).
// COUNT: every weight is 1, one 32-bit counter per cell.  Otherwise a
// weight q (< 2^41) goes into two 32-bit counters, q >> 16 and q & 0xffff:
// the high parts of a cell sum to at most the row's mass / 2^16 (~2^24), the
// low parts to at most V/32 items x 2^16, below 2^32 for V <= 2^21.
template <bool COUNT, class Wt>
__device__ Selected radix_select(SampleSmem& s, const RowView& r, Wt weight, u64 target, double frac) {
  unsigned* Hh = reinterpret_cast<unsigned*>(hist_cols());  // [kBins][32] counts or high parts
  unsigned* Hl = Hh + kBins * 32;                            // [kBins][32] low parts
  const uint32_t lane = threadIdx.x & 31;
  uint32_t prefix = 0;
  u64 rem = target;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int c = threadIdx.x; c < kBins * 32 * (COUNT ? 1 : 2); c += blockDim.x) Hh[c] = 0u;
    __syncthreads();
    walk(r, [&](int, float x, uint32_t key, bool, bool keep) {
      if (keep && (pass == 0 || (key >> (shift + 8)) == prefix)) {
        const uint32_t cell = ((key >> shift) & 255u) * 32 + lane;
        if (COUNT) {
          atomicAdd(&Hh[cell], 1u);
        } else {
          const u64 w = weight(x, key);
          atomicAdd(&Hh[cell], (unsigned)(w >> 16));
          atomicAdd(&Hl[cell], (unsigned)(w & 0xffffu));
        }
      }
    });
    __syncthreads();
    {  // bin totals: 4 threads per bin, 8 lane columns each
      const int bin = threadIdx.x >> 2, q = threadIdx.x & 3;
      u64 t = 0;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int cell = bin * 32 + q * 8 + c;
        t += COUNT ? (u64)Hh[cell] : ((u64)Hh[cell] << 16) + (u64)Hl[cell];
      }
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      if (q == 0) s.bins[bin] = t;
    }
    __syncthreads();
    // descending bins: thread t < 256 holds bin 255 - t
    const int b0 = kBins - 1 - (int)threadIdx.x;
    const u64 h0 = b0 >= 0 ? s.bins[b0] : 0;
    u64 group = 0;
    const u64 excl = block_excl_scan(s, h0, &group);
    if (pass == 0 && frac >= 0.0) {
      const double c = ceil(frac * (double)group);
      rem = c < 1.0 ? 1ull : (c > (double)group ? group : (u64)c);
    }
    if (threadIdx.x == 0) {
      s.sel_bin = 0;
      s.sel_excl = 0;
      s.sel_h = 0;
    }
    __syncthreads();
    if (b0 >= 0 && excl < rem && rem <= excl + h0) {
      s.sel_bin = b0;
      s.sel_excl = excl;
      s.sel_h = h0;
    }
    __syncthreads();
    prefix = (prefix << 8) | (uint32_t)s.sel_bin;
    rem -= s.sel_excl;
    __syncthreads();
  }
  return {prefix, rem, s.sel_h};
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

// Gather the survivors of the active cuts (at most kCompactMax) into shared
// memory, sorted by descending x, ties to the lower id: e[j] = exp(x_j - mx)
// (mx = the first item's x when mx is NaN) and idv[j] for j < n.  Returns n,
// or -1 (in every thread) when there are more survivors than kCompactMax.
__device__ int gather_sorted(SampleSmem& s, const RowView& r, float mx, float*& e, int*& idv) {
  u64* A = hist_cols();  // [kCompactMax] (key << 32) | ~id, sorted ascending
  e = reinterpret_cast<float*>(A + kCompactMax);
  idv = reinterpret_cast<int*>(e + kCompactMax);
  for (int j = threadIdx.x; j < kCompactMax; j += blockDim.x) A[j] = 0;  // pads sort first (smallest)
  if (threadIdx.x == 0) s.ncomp = 0;
  __syncthreads();
  walk(r, [&](int i, float, uint32_t key, bool, bool keep) {
    if (keep) {
      const int slot = atomicAdd(&s.ncomp, 1);
      if (slot < kCompactMax) A[slot] = ((u64)key << 32) | (u64)(~(uint32_t)i);
    }
  });
  __syncthreads();
  const int total = s.ncomp;
  if (total > kCompactMax) return -1;
  int N = 2;
  while (N < total) N <<= 1;
  // the first N slots hold every survivor (the pads are zero)
  for (int kk = 2; kk <= N; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const u64 a = A[i], b = A[ixj];
          if (((i & kk) == 0) ? (a > b) : (a < b)) {
            A[i] = b;
            A[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const float m0 = mx == mx ? mx : key_to_float((uint32_t)(A[N - 1] >> 32));
  for (int j = threadIdx.x; j < total; j += blockDim.x) {
    const u64 c = A[N - 1 - j];
    e[j] = expf(key_to_float((uint32_t)(c >> 32)) - m0);
    idv[j] = (int)(~(uint32_t)c);
  }
  __syncthreads();
  return total;
}

// The draw over a gathered list in the reference's float order
// (sampler.cpp:42-76): the running sums left to right, p = e * inv.
// top_k mode (inv < 0): the softmax over the list (inv = 1 / sum e), then the
// top-p cut when fp, renormalised by division; nucleus mode (inv >= 0): the
// list is the top-p nucleus of a softmax whose 1 / sum is inv, renormalised
// by the list's sum.  Thread 0's result.
__device__ int draw_sorted(const float* e, const int* idv, int n, float inv, bool fp, float top_p, float u) {
  if (threadIdx.x != 0 || n <= 0) return 0;
  const bool topk = inv < 0.0f;
  if (topk) {
    float sum = 0.0f;
    for (int j = 0; j < n; ++j) sum += e[j];
    inv = 1.0f / sum;
  }
  int keep = n;
  if (topk && fp) {
    float cum = 0.0f;
    keep = 0;
    for (; keep < n; ++keep) {
      cum += e[keep] * inv;
      if (cum >= top_p) {
        ++keep;
        break;
      }
    }
    keep = max(1, min(keep, n));
  }
  const bool renorm = fp;  // a top-p cut was taken: divide by the kept sum
  float s2 = 0.0f;
  if (renorm)
    for (int j = 0; j < keep; ++j) s2 += e[j] * inv;
  int id = idv[keep - 1];
  float cum = 0.0f;
  for (int j = 0; j < keep; ++j) {
    const float pj = renorm ? (e[j] * inv) / s2 : e[j] * inv;
    cum += pj;
    if (u <= cum) {
      id = idv[j];
      break;
    }
  }
  return id;
}

__global__ void __launch_bounds__(kThreads) sample_rows_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                               float t, int top_k, float top_p,
                                                               const float* __restrict__ uniforms,
                                                               int32_t* __restrict__ out, int vec) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ SampleSmem s;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = ((V + kWarps * 128 - 1) / (kWarps * 128)) * 128;  // warp segment, a multiple of 128
  RowView r{};
  r.row = logits + (int64_t)blockIdx.x * ld;
  r.seg0 = min(V, w * S);
  r.seg1 = min(V, r.seg0 + S);
  r.t = t;
  r.vec = vec != 0;
  const float u = uniforms[blockIdx.x];
  if (threadIdx.x == 0) s.out_id = 0;

  const bool fk = top_k > 0 && top_k < V, fp = top_p > 0.0f && top_p < 1.0f;
  const bool small_k = fk && top_k <= kCompactMax;  // finished on the gathered survivors
  // max of x: the top-k survivors always include it, so it is the softmax's max
  float mx = -INFINITY;
  if (!small_k) {
    walk(r, [&](int, float x, uint32_t, bool in, bool) {
      if (in) mx = fmaxf(mx, x);
    });
    mx = block_max(s, mx);
  }
  if (fk) {
    const Selected c = radix_select<true>(s, r, [](float, uint32_t) { return 1ull; }, (u64)top_k, -1.0);
    r.Kk = c.key;
    if (c.rem < c.eq) {  // the cut splits a run of equal keys: rank them by id
      r.need_k = (int)c.rem;
      r.base_k = eq_base(s, r, c.key);  // r.fk is still off: counts every item with the key
    } else {
      r.need_k = 0x7fffffff;
    }
    r.fk = true;
    if (small_k) {
      float* e;
      int* idv;
      const int n = gather_sorted(s, r, NAN, e, idv);  // exactly top_k survivors
      const int id = draw_sorted(e, idv, n, -1.0f, fp, top_p, u);
      if (threadIdx.x == 0) out[blockIdx.x] = id;
      return;
    }
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
      walk_ordered(r, [&](int i, float x, uint32_t key, bool in, bool) {
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
      const Selected c = radix_select<false>(s, r, mass, 0, (double)top_p);
      const u64 q = mass(key_to_float(c.key), c.key);
      r.Kp = c.key;
      const u64 m = q > 0 ? (c.rem + q - 1) / q : 0;  // items with the key that the cut keeps
      if (m * q < c.eq) {  // the cut splits a run of equal keys: rank them by id
        r.need_p = (int)m;
        r.base_p = eq_base(s, r, c.key);  // r.fp still off: survivors of the top-k cut with the key
      } else {
        r.need_p = 0x7fffffff;
      }
      r.fp = true;
      // a nucleus of at most kCompactMax items is drawn from in shared memory
      float* e;
      int* idv;
      const int n = gather_sorted(s, r, mx, e, idv);
      if (n > 0) {
        const int id = draw_sorted(e, idv, n, inv, true, top_p, u);
        if (threadIdx.x == 0) out[blockIdx.x] = id;
        return;
      }
    }
    // the draw: the item at which the survivors' mass, in descending order, reaches u * total
    const Selected d = radix_select<false>(s, r, mass, 0, (double)u);
    const u64 qd = mass(key_to_float(d.key), d.key);
    const int m = qd > 0 ? (int)((d.rem + qd - 1) / qd) : 1;  // the m-th survivor with this key, in id order
    if (m == 1) {
      // the first survivor with the key: each warp's first, then the lowest
      int first = 0x7fffffff;
      walk(r, [&](int i, float, uint32_t key, bool, bool keep) {
        if (keep && key == d.key) first = min(first, i);
      });
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
      if (lane == 0) s.wval[w] = (u64)(uint32_t)first;
      __syncthreads();
      if (threadIdx.x == 0) {
        int best = 0x7fffffff;
        for (int j = 0; j < kWarps; ++j) best = min(best, (int)(uint32_t)s.wval[j]);
        s.out_id = best == 0x7fffffff ? 0 : best;
      }
      __syncthreads();
      if (threadIdx.x == 0) out[blockIdx.x] = s.out_id;
      return;
    }
    const int base = eq_base(s, r, d.key);
    const int n = (int)s.wval[w];  // this warp's count, left by eq_base
    if (threadIdx.x == 0) s.sel_warp = -1;
    __syncthreads();
    if (lane == 0 && base < m && m <= base + n) s.sel_warp = w;
    __syncthreads();
    if (w == s.sel_warp) {
      int run = base;
      walk_ordered(r, [&](int i, float, uint32_t key, bool, bool keep) {
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
  static std::atomic<bool> attr_set[kMaxDevices];
  if (int rc = smem_attr_once(ctx, sample_rows_kernel, kHistBytes, attr_set); rc != DSB_OK) return rc;
  const int vec = ((uintptr_t)logits % 16 == 0 && ld % 4 == 0) ? 1 : 0;
  DSB_CUDA_TRY(ctx, launch_pdl(sample_rows_kernel, B, kThreads, kHistBytes, ctx->stream, logits, ld, V, t, top_k,
                               top_p, uniforms, out, vec));
  ctx->stats.kernel_launches++;
  return DSB_OK;
}

}  // namespace dsb

extern "C" int dsb_sample(dsb_ctx* ctx, const float* logits, int64_t ld, int B, int V, float temperature, int top_k,
                          float top_p, const float* uniforms, int32_t* out_ids) {
  if (ctx == nullptr) return DSB_EINVAL;
  if (logits == nullptr || uniforms == nullptr || out_ids == nullptr || B <= 0 || V <= 0 || V > (1 << 21) || ld < V ||
      !(temperature == temperature) || !(top_p == top_p))
    return dsb::fail(ctx, DSB_EINVAL, "dsb_sample: bad arguments");
  return dsb::sample_rows(ctx, logits, ld, B, V, temperature, top_k, top_p, uniforms, out_ids);
}
