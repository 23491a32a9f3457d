// Expert-parallel pieces shared by the exchange kernels (ep.cu) and the
// routing kernels (ops.cu): the window layout, the peers' window pointers,
// and the stable slot of every pick with this rank's pick counts.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "dsb_ptx.cuh"

namespace dsb {

constexpr int kMaxWorld = 8;
constexpr int kMaxShared = 4;  // shared-expert groups whose rows can follow the received ones

struct EpPeers {
  uint8_t* win[kMaxWorld];  // every rank's window, mapped here (win[rank] = own)
};

struct EpLayout {
  int world, rank, E_local, D, k, T_max, cap;
  size_t off_counts, off_flags, off_meta, off_recv, off_inbox, off_stage, off_smeta, bytes;
  uint64_t wait_ns;  // bound of every flag wait (the context's limit at launch)
};

// What a routing kernel needs to prepare this rank's side of one exchange.
struct EpPublishArgs {
  EpLayout L;
  EpPeers peers;
  int32_t* slot;   // [T * k] out: rank of each pick among this rank's picks of its expert
  int32_t* cnt;    // [E] out: this rank's picks of each expert
  uint32_t epoch;  // the exchange's epoch (odd)
  int E;           // experts over all ranks
  int enabled;     // 0: nothing to prepare
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp (lane = 0..31): the stable slot of every pick among this rank's
// picks of the same expert, and this rank's per-expert pick counts, both into
// this rank's own memory (a.slot, a.cnt; the dispatch sends them).  ids: the
// n_picks expert ids (global memory, complete when the warp starts); cnt:
// [E] ints of shared memory.  An out-of-range id is flagged in *status and
// not counted.
__device__ __forceinline__ void ep_count_warp(const int32_t* ids, int n_picks, const EpPublishArgs& a, int* status,
                                              int32_t* cnt, int lane) {
  for (int e = lane; e < a.E; e += 32) cnt[e] = 0;
  __syncwarp();
  for (int c = 0; c < n_picks; c += 32) {
    const int i = c + lane;
    int e = i < n_picks ? __ldcg(ids + i) : -1 - lane;
    if (i < n_picks && (unsigned)e >= (unsigned)a.E) {
      atomicExch(status, kStatusBadInput);
      e = -1 - lane;
    }
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int r = __popc(grp & ((1u << lane) - 1u));
    const int base = e >= 0 ? cnt[e] : 0;
    __syncwarp();
    if (i < n_picks) a.slot[i] = e >= 0 ? base + r : -1;
    if (e >= 0 && r == 0) cnt[e] = base + __popc(grp);
    __syncwarp();
  }
  for (int e = lane; e < a.E; e += 32) a.cnt[e] = cnt[e];
}

}  // namespace dsb
