// Expert parallelism over peer memory: token dispatch to the ranks that own
// the picked experts, and the return of the expert outputs, as kernels that
// write straight into the other GPUs' memory over NVLink (CUDA IPC windows),
// with no collective library on the data path.
//
// Expert e lives on rank e / E_local.  Every rank keeps its own tokens (data
// parallel attention) and exchanges, per MoE layer, in two rendezvous:
//   1. rows     each pick's bf16 token row goes, with no wait, to a staging
//               slot of the owner's window fixed by (source rank, local
//               expert, rank of the pick among the source's picks of that
//               expert), and the source's [world][E_local] counts to every
//               window; the owner waits for every source's rows flag and lays
//               the rows out grouped by local expert, sources in rank order,
//               picks of one source in pick order (so an expert sees the same
//               row order as the single-GPU permutation restricted to it)
//   2. return   each received row's expert output goes back into the home
//               rank's inbox slot of that pick; the home rank sums
//               w[t,j] * out[t,j] in pick order, then its shared experts
//               (moe_step's order, src/models/deepseek/ops.cpp:133-145).
// Every step publishes with a flag holding the call's epoch; a receiver waits
// (bounded) until all sources show the epoch.  The windows are reused across
// calls, which is safe because each rank's next dispatch needs every peer's
// return of the previous call, and the owner reads its staging slots and
// counts before it returns.
//
// Window layout (identical on every rank):
//   counts [world src][world dst][E_local] int32
//   flags  [3][world src] uint32 (row 1: rows, row 2: return; row 0 unused)
//   meta   [cap] int32  (source rank << 24 | source pick index) per received row
//   recv   [cap + kMaxShared * T_max][D] bf16 received rows, cap = world * T_max * k,
//          followed (when asked) by this rank's own rows once per shared expert
//   inbox  [T_max * k][D] fp32 returned outputs of this rank's picks
//   stage  [world src][E_local][T_max][D] bf16 rows as the sources sent them
//   smeta  [world src][E_local][T_max] int32 their source pick indices
// Replaces nothing in the reference (single GPU, B = 1); the exchange model
// is a host permutation: token -> rank = expert / (E / world).

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"
#include "ep_common.cuh"
#include "rows.cuh"

namespace dsb {
namespace {

EpLayout make_layout(int world, int rank, int E_local, int D, int k, int T_max) {
  EpLayout L{};
  L.world = world;
  L.rank = rank;
  L.E_local = E_local;
  L.D = D;
  L.k = k;
  L.T_max = T_max;
  L.cap = world * T_max * k;
  auto a = [](size_t v) { return (v + 255) & ~size_t(255); };
  size_t o = 0;
  L.off_counts = o;
  o += a((size_t)world * world * E_local * 4);
  L.off_flags = o;
  o += a((size_t)3 * world * 4);
  L.off_meta = o;
  o += a((size_t)L.cap * 4);
  L.off_recv = o;
  o += a((size_t)(L.cap + kMaxShared * T_max) * D * 2);
  L.off_inbox = o;
  o += a((size_t)T_max * k * D * 4);
  L.off_stage = o;
  o += a((size_t)world * E_local * T_max * D * 2);
  L.off_smeta = o;
  o += a((size_t)world * E_local * T_max * 4);
  L.bytes = o;
  return L;
}

// Bounded wait until flags[s] == epoch for every source s (one thread); gives
// up after limit_ns of %globaltimer.
__device__ bool wait_flags(const uint32_t* flags, int world, uint32_t epoch, uint64_t limit_ns) {
  uint64_t t0 = 0;
  for (uint32_t it = 1;; ++it) {
    bool all = true;
    for (int s = 0; s < world; ++s) all &= ld_acquire_sys(flags + s) == epoch;
    if (all) return true;
    if ((it & 255u) == 0) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > limit_ns) return false;
    }
  }
}

// 1. One warp: the slot of every pick and this rank's pick counts
// (ep_count_warp).  The routing kernels do the same in their last CTA when
// given publish arguments, so this launch is only for dsb_ep_dispatch called
// directly.
__global__ void ep_count_kernel(const int32_t* __restrict__ ids, int n_picks, EpPublishArgs pub, int* status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ int32_t cnt[256];
  ep_count_warp(ids, n_picks, pub, status, cnt, threadIdx.x);
}

// 2. Rows to their owners, with no wait: pick i's row goes to the staging
// slot [this rank][local expert][slot[i]] of the owner's window (a source's
// picks of one expert are at most its T <= T_max tokens), its pick index to
// the slot's meta; CTA 0 also writes this rank's counts into every window's
// count matrix [src][dst][E_local].  The last CTA to finish raises the rows
// flag in every window.
__global__ void ep_dispatch_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int32_t* __restrict__ ids,
                                   const int32_t* __restrict__ slot, const int32_t* __restrict__ cnt, int n_picks,
                                   EpLayout L, EpPeers peers, int* __restrict__ ticket, uint32_t epoch) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int W = L.world, EL = L.E_local;
  if (blockIdx.x == 0) {
    for (int idx = threadIdx.x; idx < W * EL; idx += blockDim.x) {
      const int dst = idx / EL, el = idx % EL;
      reinterpret_cast<int32_t*>(peers.win[dst] + L.off_counts)[(L.rank * W + dst) * EL + el] = cnt[idx];
    }
  }
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int vec_per_row = L.D / 8;  // 16-byte vectors of bf16
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < n_picks; i += gridDim.x * warps) {
    const int e = ids[i], s = slot[i];
    if (s < 0 || s >= L.T_max) continue;
    const int dst = e / EL, el = e % EL;
    const size_t srow = ((size_t)L.rank * EL + el) * L.T_max + s;
    uint8_t* pw = peers.win[dst];
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(i / L.k) * ldx);
    uint4* out = reinterpret_cast<uint4*>(pw + L.off_stage + srow * L.D * 2);
    for (int v = lane; v < vec_per_row; v += 32) out[v] = src[v];
    if (lane == 0) reinterpret_cast<int32_t*>(pw + L.off_smeta)[srow] = i;
  }
  // the CTA's stores, ordered by the barrier, then one system-scope fence
  // before its ticket (cumulative: it covers every store the barrier ordered
  // before it, the pattern of a cooperative grid barrier)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int prev = atomicAdd(ticket, 1);
    if (prev == (int)gridDim.x - 1) {
      *ticket = 0;
      __threadfence_system();
      for (int p = 0; p < W; ++p)
        st_release_sys(reinterpret_cast<uint32_t*>(peers.win[p] + L.off_flags) + 1 * W + L.rank, epoch);
    }
  }
}

// 2'. The owner's side: wait (bounded) until every source has raised the rows
// flag, then lay the staged rows out for the grouped expert GEMMs - local
// experts in order, within one the sources in rank order, within a source
// its picks in pick order (the single-GPU permutation restricted to this
// rank) - with their (source << 24 | pick) meta for the return, the receive
// offsets (CTA 0), and with shared experts this rank's own T rows once per
// shared group after them (groups E_local .. E_local + n_shared - 1).
// Counts are clamped to the staging capacity and the rows to the receive
// capacity, so a corrupt count cannot move a copy out of its buffer.
__global__ void ep_recv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int T, int n_shared, EpLayout L,
                               EpPeers peers, int32_t* __restrict__ recv_offsets, uint32_t epoch, int* status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ int32_t base_s[257];  // [el][src] first receive row of each staged block, then n_recv
  __shared__ int ok_s;
  uint8_t* win = peers.win[L.rank];
  const int W = L.world, EL = L.E_local, nb = W * EL;
  if (threadIdx.x == 0) {
    ok_s = wait_flags(reinterpret_cast<const uint32_t*>(win + L.off_flags) + 1 * W, W, epoch, L.wait_ns) ? 1 : 0;
    if (!ok_s) atomicCAS(status, 0, kStatusTimeout);
  }
  __syncthreads();
  if (!ok_s) return;
  // block b = el * W + s holds min(counts[s][rank][el], T_max) rows; one warp scans
  const int32_t* counts = reinterpret_cast<const int32_t*>(win + L.off_counts);
  if (threadIdx.x < 32) {
    int run = 0;
    for (int c = 0; c < nb; c += 32) {
      const int b = c + (int)threadIdx.x;
      int n = 0;
      if (b < nb) n = min(max(__ldcv(counts + ((b % W) * W + L.rank) * EL + b / W), 0), L.T_max);
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if ((int)threadIdx.x >= o) incl += v;
      }
      if (b < nb) base_s[b] = min(run + incl - n, L.cap);
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (threadIdx.x == 0) base_s[nb] = min(run, L.cap);
  }
  __syncthreads();
  const int n_recv = base_s[nb];
  if (blockIdx.x == 0) {
    for (int el = threadIdx.x; el <= EL + n_shared; el += blockDim.x)
      recv_offsets[el] = el <= EL ? (el < EL ? base_s[el * W] : n_recv) : n_recv + (el - EL) * T;
  }
  uint8_t* recv = win + L.off_recv;
  const int32_t* smeta = reinterpret_cast<const int32_t*>(win + L.off_smeta);
  int32_t* meta = reinterpret_cast<int32_t*>(win + L.off_meta);
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int vec_per_row = L.D / 8;
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < n_recv; r += gridDim.x * warps) {
    // the block holding row r: the last b with base_s[b] <= r
    int lo = 0, hi = nb - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (base_s[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int el = lo / W, s = lo % W, j = r - base_s[lo];
    const size_t srow = ((size_t)s * EL + el) * L.T_max + j;
    const uint4* src = reinterpret_cast<const uint4*>(win + L.off_stage + srow * L.D * 2);
    uint4* out = reinterpret_cast<uint4*>(recv + (size_t)r * L.D * 2);
    for (int v = lane; v < vec_per_row; v += 32) out[v] = __ldcv(src + v);
    if (lane == 0) meta[r] = (s << 24) | __ldcv(smeta + srow);
  }
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < n_shared * T; i += gridDim.x * warps) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(i % T) * ldx);
    uint4* out = reinterpret_cast<uint4*>(recv + (size_t)(n_recv + i) * L.D * 2);
    for (int v = lane; v < vec_per_row; v += 32) out[v] = src[v];
  }
}

// 3. Wait until every source has raised `phase` here (one thread): phase 1,
// its rows have landed; phase 2, its returns have.  Used for phase 2 by a
// rank with no tokens, whose combine has nothing else to wait on (the rows
// wait is the receive kernel's).
__global__ void ep_wait_kernel(EpLayout L, EpPeers peers, int phase, uint32_t epoch, int* status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(peers.win[L.rank] + L.off_flags) + phase * L.world;
  if (!wait_flags(flags, L.world, epoch, L.wait_ns)) atomicCAS(status, 0, kStatusTimeout);
}

// 4. Expert outputs (fp32 [cap][D], rows in receive order) back to the home
// ranks' inboxes; the last CTA raises the return flag in every window.  After
// an earlier wait of this exchange ran out (status set), the receive offsets
// and meta may be stale: no row is stored, but the flag is still raised so
// that the peers' waits end with the status they already report.
__global__ void ep_return_kernel(const float* __restrict__ y, int64_t ldy, const int32_t* __restrict__ recv_offsets,
                                 EpLayout L, EpPeers peers, int* __restrict__ ticket, uint32_t epoch,
                                 const int* __restrict__ status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const int n_recv = *reinterpret_cast<const volatile int*>(status) != 0 ? 0 : recv_offsets[L.E_local];
  const int32_t* meta = reinterpret_cast<const int32_t*>(peers.win[L.rank] + L.off_meta);
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int vec_per_row = L.D / 4;  // 16-byte vectors of fp32
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < n_recv; r += gridDim.x * warps) {
    const int m = __ldcv(meta + r);
    const int home = m >> 24, pick = m & 0xFFFFFF;
    const uint4* src = reinterpret_cast<const uint4*>(y + (int64_t)r * ldy);
    uint4* out = reinterpret_cast<uint4*>(peers.win[home] + L.off_inbox + (size_t)pick * L.D * 4);
    for (int v = lane; v < vec_per_row; v += 32) out[v] = src[v];
  }
  // as in the dispatch: the barrier, then one system-scope fence per CTA
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int prev = atomicAdd(ticket, 1);
    if (prev == (int)gridDim.x - 1) {
      *ticket = 0;
      __threadfence_system();
      for (int p = 0; p < L.world; ++p)
        st_release_sys(reinterpret_cast<uint32_t*>(peers.win[p] + L.off_flags) + 2 * L.world + L.rank, epoch);
    }
  }
}

// 5. h[t] += sum_j w[t,j] * inbox[t*k+j] (pick order) + sum_s shared[s*T + t].
__global__ void ep_combine_kernel(const float* __restrict__ weights, int T, EpLayout L, EpPeers peers,
                                  const float* __restrict__ shared, const int32_t* __restrict__ shared_row0,
                                  int n_shared, float* __restrict__ h,
                                  const float* __restrict__ w_next, float eps, __nv_bfloat16* __restrict__ xn_next,
                                  uint32_t epoch, int* status) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  __shared__ int ok_s;
  const uint8_t* win = peers.win[L.rank];
  if (threadIdx.x == 0) {
    ok_s = wait_flags(reinterpret_cast<const uint32_t*>(win + L.off_flags) + 2 * L.world, L.world, epoch, L.wait_ns)
               ? 1
               : 0;
    if (!ok_s) atomicCAS(status, 0, kStatusTimeout);
  }
  __syncthreads();
  if (!ok_s) return;
  const float* inbox = reinterpret_cast<const float*>(win + L.off_inbox);
  const int t = blockIdx.x, k = L.k, D = L.D;
  __shared__ float red[32];
  __shared__ float wsm[32];  // the token's routing weights (k <= 32, checked at create), looked up once
  if ((int)threadIdx.x < k) wsm[threadIdx.x] = weights[(size_t)t * k + threadIdx.x];
  __syncthreads();
  // the weighted outputs w * out, the single-GPU combine's pre-weighted rows
  auto pick = [&](int j, int i4) {
    const float4 v = __ldcv(reinterpret_cast<const float4*>(inbox + ((size_t)t * k + j) * D) + i4);
    const float wj = wsm[j];
    return make_float4(__fmul_rn(v.x, wj), __fmul_rn(v.y, wj), __fmul_rn(v.z, wj), __fmul_rn(v.w, wj));
  };
  // shared outputs: [n_shared][T][D], at row shared_row0[0] of `shared` when given
  if (shared_row0 != nullptr) shared += (size_t)shared_row0[0] * D;
  combine_row(pick, k, D, n_shared > 0 ? shared + (size_t)t * D : nullptr, n_shared, (int64_t)T * D, h + (size_t)t * D,
              w_next, eps,
              xn_next ? xn_next + (size_t)t * D : nullptr, red);
}

}  // namespace
}  // namespace dsb

struct dsb_ep {
  dsb_ctx* ctx = nullptr;
  dsb::EpLayout L{};
  int E = 0;
  uint8_t* win = nullptr;
  dsb::EpPeers peers{};
  bool connected = false;
  bool opened[dsb::kMaxWorld] = {};
  uint32_t epoch = 0;
  int published_T = -1;           // tokens of the dispatch whose counts went out last
  int32_t* d_slot = nullptr;      // [T_max * k]
  int32_t* d_cnt = nullptr;       // [E] this rank's picks of each expert
  int32_t* d_recv_off = nullptr;  // [E_local + 1]
  int* d_ticket = nullptr;        // [2]: dispatch, return
};

using namespace dsb;

int dsb::ep_params(const dsb_ep* ep, int* rank, int* world, int* n_experts, int* top_k, int* hidden, int* max_tokens,
                   int* E_local) {
  if (rank) *rank = ep->L.rank;
  if (world) *world = ep->L.world;
  if (n_experts) *n_experts = ep->E;
  if (top_k) *top_k = ep->L.k;
  if (hidden) *hidden = ep->L.D;
  if (max_tokens) *max_tokens = ep->L.T_max;
  if (E_local) *E_local = ep->L.E_local;
  return DSB_OK;
}

static int ep_create_impl(dsb_ctx* ctx, int rank, int world, int n_experts, int hidden, int top_k,
                             int max_tokens, dsb_ep** out) {
  if (ctx == nullptr || out == nullptr) return DSB_EINVAL;
  *out = nullptr;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || n_experts <= 0 || n_experts % world ||
      n_experts > 256 || hidden <= 0 || hidden % 8 || top_k <= 0 || top_k > 32 || max_tokens <= 0 ||
      (int64_t)world * max_tokens * top_k >= (1 << 24))
    return fail(ctx, DSB_EINVAL,
                "dsb_ep_create: bad sizes (world <= 8, E <= 256 and divisible by world, top_k <= 32)");
  auto* ep = new dsb_ep();
  ep->ctx = ctx;
  ep->E = n_experts;
  ep->L = make_layout(world, rank, n_experts / world, hidden, top_k, max_tokens);
  cudaError_t e = cudaMalloc(&ep->win, ep->L.bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->win, 0, ep->L.bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ep->d_slot, (size_t)max_tokens * top_k * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ep->d_cnt, (size_t)n_experts * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ep->d_recv_off, (size_t)(ep->L.E_local + 1 + kMaxShared) * 4);
  // zero ranges until the first dispatch (a timed-out exchange leaves them as they were)
  if (e == cudaSuccess) e = cudaMemset(ep->d_recv_off, 0, (size_t)(ep->L.E_local + 1 + kMaxShared) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&ep->d_ticket, 2 * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ep->d_ticket, 0, 2 * sizeof(int));
  if (e != cudaSuccess) {
    cudaFree(ep->win);
    cudaFree(ep->d_slot);
    cudaFree(ep->d_cnt);
    cudaFree(ep->d_recv_off);
    cudaFree(ep->d_ticket);
    delete ep;
    return fail(ctx, DSB_ENOMEM, "dsb_ep_create: %s", cudaGetErrorString(e));
  }
  ep->peers.win[rank] = ep->win;
  *out = ep;
  return DSB_OK;
}

extern "C" int dsb_ep_window_handle(dsb_ep* ep, void* handle) {
  if (ep == nullptr || handle == nullptr) return DSB_EINVAL;
  cudaIpcMemHandle_t h;
  DSB_CUDA_TRY(ep->ctx, cudaIpcGetMemHandle(&h, ep->win));
  std::memcpy(handle, &h, sizeof(h));
  return DSB_OK;
}

extern "C" int dsb_ep_connect(dsb_ep* ep, const void* handles) {
  if (ep == nullptr || handles == nullptr) return DSB_EINVAL;
  const auto* hs = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < ep->L.world; ++p) {
    if (p == ep->L.rank) continue;
    void* ptr = nullptr;
    DSB_CUDA_TRY(ep->ctx, cudaIpcOpenMemHandle(&ptr, hs[p], cudaIpcMemLazyEnablePeerAccess));
    ep->peers.win[p] = static_cast<uint8_t*>(ptr);
    ep->opened[p] = true;
  }
  ep->connected = true;
  return DSB_OK;
}

extern "C" int dsb_ep_window_ptr(dsb_ep* ep, void** ptr) {
  if (ep == nullptr || ptr == nullptr) return DSB_EINVAL;
  *ptr = ep->win;
  return DSB_OK;
}

extern "C" int dsb_ep_connect_local(dsb_ep* ep, void* const* windows) {
  if (ep == nullptr) return DSB_EINVAL;
  if (windows == nullptr) return fail(ep->ctx, DSB_EINVAL, "dsb_ep_connect_local: null window list");
  if (ep->connected) return fail(ep->ctx, DSB_EINVAL, "dsb_ep_connect_local: already connected");
  for (int p = 0; p < ep->L.world; ++p) {
    if (p == ep->L.rank) continue;
    if (windows[p] == nullptr || (reinterpret_cast<uintptr_t>(windows[p]) & 255u))
      return fail(ep->ctx, DSB_EINVAL, "dsb_ep_connect_local: window %d null or not 256-byte aligned", p);
  }
  for (int p = 0; p < ep->L.world; ++p)
    if (p != ep->L.rank) ep->peers.win[p] = static_cast<uint8_t*>(windows[p]);
  ep->connected = true;
  return DSB_OK;
}

extern "C" int dsb_ep_destroy(dsb_ep* ep) {
  if (ep == nullptr) return DSB_OK;
  cudaStreamSynchronize(ep->ctx->stream);
  for (int p = 0; p < ep->L.world; ++p)
    if (ep->opened[p]) cudaIpcCloseMemHandle(ep->peers.win[p]);
  cudaFree(ep->win);
  cudaFree(ep->d_slot);
  cudaFree(ep->d_cnt);
  cudaFree(ep->d_recv_off);
  cudaFree(ep->d_ticket);
  delete ep;
  return DSB_OK;
}

extern "C" int dsb_ep_info(const dsb_ep* ep, int* E_local, int* recv_capacity, uint64_t* window_bytes) {
  if (ep == nullptr) return DSB_EINVAL;
  if (E_local) *E_local = ep->L.E_local;
  if (recv_capacity) *recv_capacity = ep->L.cap;
  if (window_bytes) *window_bytes = ep->L.bytes;
  return DSB_OK;
}

int dsb::ep_publish_args(dsb_ep* ep, int T, EpPublishArgs* out) {
  if (ep == nullptr || out == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = ep->ctx;
  if (!ep->connected && ep->L.world > 1) return fail(ctx, DSB_EINVAL, "dsb_ep_dispatch: dsb_ep_connect first");
  if (T < 0 || T > ep->L.T_max) return fail(ctx, DSB_EINVAL, "dsb_ep_dispatch: bad arguments (T <= max_tokens)");
  ep->L.wait_ns = ctx->wait_limit_ns;
  const uint32_t epoch = ++ep->epoch * 2 - 1;  // odd: dispatch, even: the return of the same call
  ep->published_T = T;
  out->L = ep->L;
  out->peers = ep->peers;
  out->slot = ep->d_slot;
  out->cnt = ep->d_cnt;
  out->epoch = epoch;
  out->E = ep->E;
  out->enabled = 1;
  return DSB_OK;
}

int dsb::ep_publish(dsb_ep* ep, int T, const int32_t* ids) {
  if (ep == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = ep->ctx;
  if (ids == nullptr) return fail(ctx, DSB_EINVAL, "dsb_ep_dispatch: null ids");
  EpPublishArgs pub;
  int rc = ep_publish_args(ep, T, &pub);
  if (rc != DSB_OK) return rc;
  launch_pdl(ep_count_kernel, 1, 32, 0, ctx->stream, ids, T * ep->L.k, pub, ctx->d_status);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches += 1;
  return DSB_OK;
}

int dsb::ep_send(dsb_ep* ep, const void* x, int64_t ldx, int T, const int32_t* ids, void** recv_x,
                 int32_t** recv_offsets, int n_shared) {
  if (ep == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = ep->ctx;
  if (x == nullptr || ids == nullptr || T != ep->published_T || ldx < ep->L.D || (ldx % 8) ||
      (reinterpret_cast<uintptr_t>(x) & 15u) || n_shared < 0 || n_shared > kMaxShared)
    return fail(ctx, DSB_EINVAL, "dsb_ep_dispatch: bad arguments (the published T, 16-byte aligned rows)");
  const uint32_t epoch = ep->epoch * 2 - 1;
  const int n = T * ep->L.k;
  const int blocks = std::max(1, std::min(ctx->sm_count, (n + 7) / 8));
  launch_pdl(ep_dispatch_kernel, blocks, 256, 0, ctx->stream, static_cast<const __nv_bfloat16*>(x), ldx, ids,
             ep->d_slot, ep->d_cnt, n, ep->L, ep->peers, ep->d_ticket, epoch);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  // at most cap received rows plus the shared copies, one per warp
  const int rblocks = std::max(1, std::min(ctx->sm_count, (ep->L.cap + n_shared * T + 7) / 8));
  launch_pdl(ep_recv_kernel, rblocks, 256, 0, ctx->stream, static_cast<const __nv_bfloat16*>(x), ldx, T, n_shared,
             ep->L, ep->peers, ep->d_recv_off, epoch, ctx->d_status);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches += 2;
  if (recv_x) *recv_x = ep->win + ep->L.off_recv;
  if (recv_offsets) *recv_offsets = ep->d_recv_off;
  return DSB_OK;
}

extern "C" int dsb_ep_dispatch(dsb_ep* ep, const void* x, int64_t ldx, int T, const int32_t* ids, void** recv_x,
                               int32_t** recv_offsets) {
  if (ep == nullptr) return DSB_EINVAL;
  if (x == nullptr || ldx < ep->L.D || (ldx % 8) || (reinterpret_cast<uintptr_t>(x) & 15u))
    return fail(ep->ctx, DSB_EINVAL, "dsb_ep_dispatch: bad arguments (T <= max_tokens, 16-byte aligned rows)");
  int rc = dsb::ep_publish(ep, T, ids);
  if (rc != DSB_OK) return rc;
  return dsb::ep_send(ep, x, ldx, T, ids, recv_x, recv_offsets, 0);
}

extern "C" int dsb_ep_combine(dsb_ep* ep, const float* y, int64_t ldy, int T, const float* weights,
                              const float* shared, int n_shared, float* h) {
  return dsb::ep_combine(ep, y, ldy, T, weights, shared, n_shared, h, nullptr, 0.0f, nullptr, nullptr);
}

int dsb::ep_combine(dsb_ep* ep, const float* y, int64_t ldy, int T, const float* weights, const float* shared,
                    int n_shared, float* h, const float* w_next, float eps, void* xn_next,
                    const int32_t* shared_row0) {
  if (ep == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = ep->ctx;
  if (y == nullptr || weights == nullptr || h == nullptr || T < 0 || T > ep->L.T_max || ldy < ep->L.D ||
      (ldy % 4) || (reinterpret_cast<uintptr_t>(y) & 15u) || n_shared < 0 || (n_shared > 0 && shared == nullptr))
    return fail(ctx, DSB_EINVAL, "dsb_ep_combine: bad arguments");
  if (ep->epoch == 0) return fail(ctx, DSB_EINVAL, "dsb_ep_combine: no dispatch to return");
  ep->L.wait_ns = ctx->wait_limit_ns;
  const uint32_t epoch = ep->epoch * 2;
  // at most cap rows come back, one per warp
  const int ret_blocks = std::max(1, std::min(ctx->sm_count, (ep->L.cap + 7) / 8));
  launch_pdl(ep_return_kernel, ret_blocks, 256, 0, ctx->stream, y, ldy, ep->d_recv_off, ep->L, ep->peers,
             ep->d_ticket + 1, epoch, ctx->d_status);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  if (T > 0) {
    launch_pdl(ep_combine_kernel, T, combine_threads(ep->L.D), 0, ctx->stream, weights, T, ep->L, ep->peers, shared,
               shared_row0, n_shared, h, w_next,
               eps, static_cast<__nv_bfloat16*>(xn_next), epoch,
                                                  ctx->d_status);
    DSB_CUDA_TRY(ctx, cudaGetLastError());
  } else {
    // no tokens here, but the next dispatch may only start once every peer has returned
    launch_pdl(ep_wait_kernel, 1, 1, 0, ctx->stream, ep->L, ep->peers, 2, epoch, ctx->d_status);
    DSB_CUDA_TRY(ctx, cudaGetLastError());
  }
  ctx->stats.kernel_launches += 2;
  return DSB_OK;
}

extern "C" int dsb_ep_create(dsb_ctx* ctx, int rank, int world, int n_experts, int hidden, int top_k,
                             int max_tokens, dsb_ep** out) {
  return dsb::guarded(ctx, "dsb_ep_create",
                      [&] { return ep_create_impl(ctx, rank, world, n_experts, hidden, top_k, max_tokens, out); });
}
