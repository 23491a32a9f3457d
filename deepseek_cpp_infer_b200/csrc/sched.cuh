// Work schedule of a persistent (grouped) GEMM launch, shared by the bf16
// and FP8 GEMM kernels.
//
// A unit is one (group, 128-row weight tile, token tile) with at least one
// token; groups without tokens contribute none, so the units of a MoE expert
// GEMM are only those of the experts this step routed to.  With `grid` CTAs
// the first R = floor(N / grid) rounds of units run whole; the remaining
// `tail` units (the partial last round) are each split along K into S parts,
// S = min(grid / tail, max_splits), so the last round fills the SMs instead
// of leaving most of them idle.  Split units are reduced by whichever of
// their CTAs finishes last (in split order).  Work item i of the launch is
// taken by CTA i % grid.
//
// The unit counts depend on the token offsets that the previous kernel
// writes, so each CTA builds the table in shared memory once (one warp), and
// every role of the CTA walks the same sequence from it.

#pragma once

#include <stdint.h>

namespace dsb {

constexpr int kSchedMaxGroups = 512;

struct SchedShape {
  int full;    // work items that are whole units (R * grid)
  int splits;  // parts of each tail unit
  int items;   // work items of the launch
};

__host__ __device__ inline SchedShape sched_shape(int n_units, int grid, int max_splits) {
  const int rounds = n_units / grid, tail = n_units - rounds * grid;
  int s = 1;
  if (tail > 0) {
    s = grid / tail;
    if (s > max_splits) s = max_splits;
    if (s < 1) s = 1;
  }
  return {rounds * grid, s, rounds * grid + tail * s};
}

struct SchedTable {
  SchedShape shape;
  int G;
  int first_unit[kSchedMaxGroups + 1];  // units of the groups before g
  int tok0[kSchedMaxGroups];            // first token row of group g
  int count[kSchedMaxGroups];           // token rows of group g
};

// Built by one warp (all 32 lanes).  Dense launches (tok_offsets null) give
// every group the token rows [0, T).
__device__ __forceinline__ void sched_build(SchedTable* tb, const int32_t* tok_offsets, int G, int T, int NT,
                                            int m_tiles, int max_splits, uint32_t lane) {
  int carry = 0;
  for (int g0 = 0; g0 < G; g0 += 32) {
    const int g = g0 + (int)lane;
    int t0 = 0, n = 0;
    if (g < G) {
      if (tok_offsets != nullptr) {  // clamped to [0, T]: rows outside are never touched
        t0 = min(max(tok_offsets[g], 0), T);
        n = min(max(tok_offsets[g + 1], t0), T) - t0;
      } else {
        n = T;
      }
    }
    const int units = ((n + NT - 1) / NT) * m_tiles;
    int incl = units;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if ((int)lane >= o) incl += v;
    }
    if (g < G) {
      tb->first_unit[g] = carry + incl - units;
      tb->tok0[g] = t0;
      tb->count[g] = n;
    }
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    tb->first_unit[G] = carry;
    tb->G = G;
    tb->shape = sched_shape(carry, (int)gridDim.x, max_splits);
  }
}

// The work items of this CTA, in order.
struct SchedIter {
  const SchedTable* tb;
  int m_tiles, NT, KB;
  int item = -1;
  int g = 0, mt = 0, nt = 0;  // group, weight tile, token tile
  int tok0 = 0, tok1 = 0;     // token rows of the group
  int split = 0, nsplit = 1;  // part of the unit (tail units only)
  int tail_j = -1;            // index of a split unit among the tail units
  int kb0 = 0, kb1 = 0;       // K blocks of this item

  __device__ bool next() {
    item = item < 0 ? (int)blockIdx.x : item + (int)gridDim.x;
    const SchedShape sh = tb->shape;
    if (item >= sh.items) return false;
    int unit;
    if (item < sh.full) {
      unit = item;
      split = 0;
      nsplit = 1;
      tail_j = -1;
    } else {
      const int v = item - sh.full;
      tail_j = v / sh.splits;
      split = v - tail_j * sh.splits;
      nsplit = sh.splits;
      unit = sh.full + tail_j;
    }
    // the last group whose first unit is <= unit (groups without units share
    // their successor's first unit and are passed over)
    int lo = 0, hi = tb->G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tb->first_unit[mid] <= unit) lo = mid;
      else hi = mid - 1;
    }
    g = lo;
    const int local = unit - tb->first_unit[g];
    mt = local % m_tiles;
    nt = local / m_tiles;
    tok0 = tb->tok0[g];
    tok1 = tok0 + tb->count[g];
    kb0 = (int)((int64_t)split * KB / nsplit);
    kb1 = (int)((int64_t)(split + 1) * KB / nsplit);
    return true;
  }
};

}  // namespace dsb
