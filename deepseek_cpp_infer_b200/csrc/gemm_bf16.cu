// Grouped bf16 linear layer on tcgen05, weights as the 128-row A operand
// ("swap AB"): for group g, token rows t and output features n
//     y[t, g*y_group_col + n] = sum_k x[t, g*x_group_col + k] * W[g*M + n, k]
// A work tile is a 128-feature slice of one group's weights (and a K split);
// its tokens are the N side of the MMA (16..256 columns), so at decode the
// weight stream is the roofline and the token count only sets the TMEM width.
//
// Persistent kernel: one CTA per SM walks the tiles blockIdx.x, +gridDim.x, ...
// The TMA ring streams across tile boundaries without draining, and the TMEM
// accumulator is double-buffered so the epilogue of one tile overlaps the
// MMAs of the next.
//
// Replaces cublasSgemv / cublasGemmEx in gemv_row_major_mixed
// (src/models/deepseek/cuda_backend.cpp:459-498), the GEMV chains of
// dense_mlp_to_slot / moe_to_slot (cuda_backend.cpp:820-883) and the
// ds_silu_mul_kernel / ds_scale_add_kernel elementwise passes
// (src/ops/cuda/elementwise_kernels.cu:35-45), which become epilogues.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2-5
// epilogue (warp w reads TMEM lanes 32*(w%4)..+31 = weight rows of the tile).
// Split-K (dense groups with <= 256 tokens only): every split writes an fp32
// partial, the last split to finish (atomic ticket) sums the partials in split
// order - deterministic - and runs the epilogue.  A dense launch whose units
// all fit one round runs the splits of a unit as one thread-block cluster
// instead (plain store / add outputs): each CTA keeps its partial in its own
// shared memory, and after a cluster barrier each sums its share of the
// tile's 32-row x 8-token pieces from all the partials at once (distributed
// shared memory, in split order: the same sums as the ticket path) and stores
// them; no global round trip.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"
#include "epi.cuh"
#include "sched.cuh"

namespace dsb {
namespace {

constexpr int kBK = 64;        // K elements per stage (one 128-byte swizzle row)
constexpr int kTileM = 128;    // weight rows per tile (MMA M)
constexpr int kThreads = 192;

struct GemmParams {
  int T, M, K, G;
  int64_t x_group_col;
  const int32_t* tok_offsets;  // [G+1] or null
  void* y;
  int64_t ldy, y_group_col;
  int y_f32;
  int epi;
  const float* row_scale;
  int max_splits;     // parts of each unit of the partial last round (sched.cuh)
  int m_tiles;
  float* ws;          // split partials: [tail unit][split][NT][128]
  int* counters;      // per-tail-unit tickets (zeroed; reset by the last split)
  int vec_out;        // y meets the alignment of the vectorised output (epi.cuh)
  int offsets_ready;  // grouped: the token offsets were complete before the previous kernel began
  int csplit;         // > 1: the splits of a unit are one cluster of csplit CTAs (one unit each)
};

template <int NT>
struct GemmShape {
  static constexpr int A_BYTES = kTileM * kBK * 2;  // 16 KB
  static constexpr int B_BYTES = NT * kBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STG = 4 * 32 * 32 * 4;       // output staging: 32 x 32 fp32 per epilogue warp
  static constexpr int NS = (212 * 1024 - STG) / STAGE;  // ring depth
  static constexpr int OFF_STG = NS * STAGE;
  static constexpr int OFF_SCHED = OFF_STG + STG;
  static constexpr int OFF_BAR = OFF_SCHED + ((int)sizeof(SchedTable) + 15) / 16 * 16;
  static constexpr int OFF_MISC = OFF_BAR + (2 * NS + 8) * 8;
  static constexpr int SMEM = OFF_MISC + 32 + 1024;
  static constexpr int PART_LD = NT + 4;              // cluster split-K partial [128][NT + 4] fp32 in the ring
  static_assert(kTileM * PART_LD * 4 <= NS * STAGE, "partial fits the ring");
  static constexpr uint32_t TC = NT < 32 ? 32 : NT;  // TMEM columns per accumulator
  static constexpr uint32_t TCOLS = 2 * TC;          // double-buffered
  static_assert(STAGE % 1024 == 0, "stage alignment");
  static_assert(SMEM <= 232448, "shared memory");
};

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                     GemmParams p, int* status) {
  using S = GemmShape<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* empty = full + S::NS;
  uint64_t* acc_full = empty + S::NS;   // [2] accumulator slot written by the MMAs
  uint64_t* acc_empty = acc_full + 2;   // [2] accumulator slot read by the epilogue
  uint64_t* drain = acc_full + 4;
  uint64_t* epi_bar = drain + 1;        // rendezvous of the 128 epilogue threads (split-K ticket)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);
  volatile int* no_abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 8);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 12);

  const int KB = (p.K + kBK - 1) / kBK;
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_init(epi_bar, 4);
    *abort = 0;
    *no_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, S::TCOLS);
    tmem_relinquish();
  }
  if (warp == 1 && lane == 0) {
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
  }
  SchedTable* sched = reinterpret_cast<SchedTable*>(smem + S::OFF_SCHED);
  const bool dense = p.tok_offsets == nullptr;
  // the unit table before the wait when nothing the previous kernel writes
  // goes into it (dense, or offsets written earlier in the stream)
  const bool early = dense || p.offsets_ready;
  if (early && warp == 2) sched_build(sched, p.tok_offsets, p.G, p.T, NT, p.m_tiles, p.max_splits, lane);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // everything above (barriers, TMEM, descriptor prefetch) overlaps the previous
  // kernel; its outputs (x, token offsets, y for ADD) are read only from here.
  // A dense GEMM's work items are known without them, so its producer also
  // starts the weight half of the first ring stages before the wait.
  int npre = 0;
  if (warp == 0 && lane == 0 && early) {
    const uint64_t pol_w = l2_policy_evict_first();
    SchedIter it{sched, p.m_tiles, NT, KB};
    while (npre < S::NS && it.next()) {
      for (int kb = it.kb0; kb < it.kb1 && npre < S::NS; ++kb, ++npre) {
        mbar_arrive_expect_tx(&full[npre], S::STAGE);
        tma_load_2d(smem + npre * S::STAGE, &map_w, &full[npre], kb * kBK, it.g * p.M + it.mt * kTileM, pol_w);
      }
    }
  }
  pdl_wait();
  if (!early) {  // the unit table of a grouped GEMM needs the token offsets
    if (warp == 2) sched_build(sched, p.tok_offsets, p.G, p.T, NT, p.m_tiles, p.max_splits, lane);
    __syncthreads();
  }
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights stream once; activations stay in L2
      SchedIter it{sched, p.m_tiles, NT, KB};
      int q = 0;  // global stage counter
      bool ok = true;
      while (ok && it.next()) {
        for (int kb = it.kb0; kb < it.kb1; ++kb, ++q) {
          const int s = q % S::NS;
          if (q >= S::NS && !mbar_wait(&empty[s], ((q / S::NS) - 1) & 1, abort)) {
            raise_abort(abort, status, kStatusTimeout);
            ok = false;
            break;
          }
          uint8_t* st = smem + s * S::STAGE;
          if (q >= npre) {  // (stages below npre got their weights before pdl_wait)
            mbar_arrive_expect_tx(&full[s], S::STAGE);
            tma_load_2d(st, &map_w, &full[s], kb * kBK, it.g * p.M + it.mt * kTileM, pol_w);
          }
          tma_load_2d(st + S::A_BYTES, &map_x, &full[s], (int)(it.g * p.x_group_col + kb * kBK), it.tok0 + it.nt * NT);
        }
      }
      pdl_launch_dependents();  // every load of this CTA is issued: the next kernel may be scheduled
      if (*abort) {
        const int first = q > S::NS ? q - S::NS : 0;
        for (int i = first; i < q; ++i) mbar_wait(&full[i % S::NS], (i / S::NS) & 1, no_abort);
      }
    }
    if (p.csplit > 1) {  // the epilogue's two cluster barriers (every thread of the cluster passes both)
      __syncwarp();
      cluster_sync();
      cluster_sync();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(kTileM, NT < 16 ? 16 : NT, 0, 0);
      SchedIter it{sched, p.m_tiles, NT, KB};
      int q = 0, u = 0;
      bool ok = true;
      while (ok && it.next()) {
        const int slot = u & 1;
        if (u >= 2 && !mbar_wait(&acc_empty[slot], ((u >> 1) - 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + slot * S::TC;
        const int kb0 = it.kb0, kb1 = it.kb1;
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int s = q % S::NS;
          if (!mbar_wait(&full[s], (q / S::NS) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = sbase + s * S::STAGE, b = a + S::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks) {
            mma_bf16_ss(d, smem_desc(a + ks * 32, 16, 1024, kSwizzle128B),
                        smem_desc(b + ks * 32, 16, 1024, kSwizzle128B), IDESC, (kb > kb0 || ks > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[slot]);
        ++u;
      }
      if (!ok) raise_abort(abort, status, kStatusTimeout);
      tc_commit(drain);
      mbar_wait(drain, 0, no_abort);
    }
    if (p.csplit > 1) {
      __syncwarp();
      cluster_sync();
      cluster_sync();
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const uint32_t qtr = warp & 3;  // TMEM lane quarter of this warp
    const int r = (int)(qtr * 32 + lane);  // weight row within the tile
    const int et = threadIdx.x - 64;  // 0..127
    const bool silu = p.epi == DSB_EPI_SILU_GATE;
    float* stg = reinterpret_cast<float*>(smem + S::OFF_STG) + (warp - 2) * 32 * 32;  // this warp's staging block
    SchedIter it{sched, p.m_tiles, NT, KB};
    int u = 0, epi_phase = 0, csyncs = 0;
    while (it.next()) {
      const int slot = u & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[slot], (u >> 1) & 1, abort))) {
        raise_abort(abort, status, kStatusTimeout);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + ((qtr * 32) << 16) + slot * S::TC;
      const int tbase = it.tok0 + it.nt * NT;
      const int tcount = min(NT, it.tok1 - tbase);
      constexpr int NCH = NT < 32 ? 1 : NT / 32;
      // output of one 32-token chunk of this thread's weight row (called by
      // all lanes of the warp)
      auto apply = [&](int c, float (&v)[32]) {
        if (silu) {
          // rows 2j / 2j+1 of the tile are gate / up of output feature 64*mt + j
          float hv[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float up = __shfl_xor_sync(0xffffffffu, v[i], 1);
            hv[i] = v[i] / (1.0f + __expf(-v[i])) * up;
          }
          if (p.vec_out) {
            warp_store_block<32, true, 0>(stg, hv, lane, tcount - c * 32, 16, p.y, p.ldy,
                                       (int64_t)it.g * p.y_group_col + it.mt * 64 + qtr * 16, tbase + c * 32,
                                       p.y_f32, false);
            return;
          }
          const int64_t col = (int64_t)it.g * p.y_group_col + it.mt * 64 + (r >> 1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = c * 32 + i;
            if ((r & 1) == 0 && t < tcount) {
              const int64_t o = (int64_t)(tbase + t) * p.ldy + col;
              if (p.y_f32) static_cast<float*>(p.y)[o] = hv[i];
              else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(hv[i]);
            }
          }
          return;
        }
        // The token weights (ROWSCALE) are all loaded before the first store
        // (a load cannot be moved above a store that may alias it, so
        // interleaving them serialises 32 memory round trips); the residual
        // add is a reduction into y, which needs no load: each element of y
        // receives exactly one add, so the result is y + x rounded once.
        if (p.epi == DSB_EPI_ROWSCALE) {
          float pre[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = c * 32 + i;
            pre[i] = t < tcount ? __ldg(p.row_scale + tbase + t) : 0.0f;
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= pre[i];
        }
        if (p.vec_out) {
          const int ncols = max(0, min(32, p.M - it.mt * kTileM - (int)qtr * 32));
          warp_store_block<32, false, 0>(stg, v, lane, tcount - c * 32, ncols, p.y, p.ldy,
                                      (int64_t)it.g * p.y_group_col + it.mt * kTileM + qtr * 32, tbase + c * 32,
                                      p.y_f32, p.epi == DSB_EPI_ADD);
          return;
        }
        if (it.mt * kTileM + r < p.M) {
          const int64_t col = (int64_t)it.g * p.y_group_col + it.mt * kTileM + r;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = c * 32 + i;
            if (t < tcount) {
              const int64_t o = (int64_t)(tbase + t) * p.ldy + col;
              if (p.epi == DSB_EPI_ADD) {
                atomicAdd(static_cast<float*>(p.y) + o, v[i]);
              } else if (p.y_f32) {
                static_cast<float*>(p.y)[o] = v[i];
              } else {
                static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v[i]);
              }
            }
          }
        }
      };
      const int nsplit = it.nsplit, tail_j = it.tail_j;
      constexpr int CW = NT < 32 ? NT : 32;  // valid columns per chunk
      if (p.csplit > 1) {
        // cluster split-K: this CTA's only unit.  Its partial goes to its own
        // shared memory (the ring, idle now: the unit's MMAs have completed),
        // row r at part_s + r * PART_LD; after the cluster barrier, warp w of
        // cluster CTA q sums the pieces (8 tokens, the 32 rows of warp w)
        // numbered pc with pc % csplit == q over the CTAs in split order.
        float* part_s = reinterpret_cast<float*>(smem) + r * S::PART_LD;
        for (int c = 0; c < NCH; ++c) {
          uint32_t raw[32];
          tmem_ld32(taddr + c * 32, raw);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < CW; i += 4)
            *reinterpret_cast<float4*>(part_s + c * 32 + i) =
                make_float4(__uint_as_float(raw[i]), __uint_as_float(raw[i + 1]), __uint_as_float(raw[i + 2]),
                            __uint_as_float(raw[i + 3]));
        }
        tc_fence_before();
        warp_arrive(&acc_empty[slot]);
        ++u;
        cluster_sync();
        ++csyncs;
        if (!__any_sync(0xffffffffu, *abort != 0)) {
          // pieces of 8 tokens x this warp's 32 rows; piece pc goes to cluster CTA pc % csplit
          const uint32_t my = cluster_ctarank();
          constexpr int HW = 8, NH = CW / HW;
          const int ncols = max(0, min(32, p.M - it.mt * kTileM - (int)qtr * 32));
          const int64_t col0 = (int64_t)it.g * p.y_group_col + it.mt * kTileM + qtr * 32;
          for (int c = 0; c < NCH; ++c) {
            for (int h = 0; h < NH; ++h) {
              if (((c * NH + h) * 4 + (int)qtr) % p.csplit != (int)my) continue;  // warp-uniform
              float4 w[8][HW / 4];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (j < p.csplit) {
                  const float4* src =
                      reinterpret_cast<const float4*>(map_cluster_ptr(part_s + c * 32 + h * HW, (uint32_t)j));
#pragma unroll
                  for (int i = 0; i < HW / 4; ++i) w[j][i] = src[i];
                }
              }
              float v[HW];
#pragma unroll
              for (int i = 0; i < HW; ++i) v[i] = 0.0f;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (j < p.csplit) {
#pragma unroll
                  for (int i = 0; i < HW / 4; ++i) {
                    v[4 * i] += w[j][i].x;
                    v[4 * i + 1] += w[j][i].y;
                    v[4 * i + 2] += w[j][i].z;
                    v[4 * i + 3] += w[j][i].w;
                  }
                }
              }
              warp_store_block<HW, false, 0>(stg, v, lane, tcount - c * 32 - h * HW, ncols, p.y, p.ldy, col0,
                                             tbase + c * 32 + h * HW, p.y_f32, p.epi == DSB_EPI_ADD);
            }
          }
        }
        cluster_sync();  // no CTA leaves while a peer may still read its partial
        ++csyncs;
        continue;
      }
      float* part = nsplit > 1 ? p.ws + ((int64_t)tail_j * nsplit + it.split) * (int64_t)NT * kTileM : nullptr;
      for (int c = 0; c < NCH; ++c) {
        uint32_t raw[32];
        tmem_ld32(taddr + c * 32, raw);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
        if (part != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i < NT) part[(c * 32 + i) * kTileM + r] = v[i];
        } else {
          apply(c, v);
        }
      }
      // the accumulator slot is free once every chunk has been read
      tc_fence_before();
      warp_arrive(&acc_empty[slot]);
      ++u;
      if (part != nullptr) {
        // the last split to finish sums the partials in split order
        __threadfence();
        if (!__all_sync(0xffffffffu, mbar_rendezvous(epi_bar, epi_phase, abort))) {
          raise_abort(abort, status, kStatusTimeout);
          break;
        }
        if (et == 0) {
          const int prev = atomicAdd(&p.counters[tail_j], 1);
          *last_flag = (prev == nsplit - 1) ? 1 : 0;
        }
        if (!__all_sync(0xffffffffu, mbar_rendezvous(epi_bar, epi_phase, abort))) {
          raise_abort(abort, status, kStatusTimeout);
          break;
        }
        if (*last_flag != 0) {
          __threadfence();
          const float* pbase = p.ws + (int64_t)tail_j * nsplit * (int64_t)NT * kTileM + r;
          for (int c = 0; c < NCH; ++c) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.0f;
            // four splits' loads in flight at a time, summed in split order
            for (int s2 = 0; s2 < nsplit; s2 += 4) {
              float w4[4][CW];
#pragma unroll
              for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < CW; ++i)
                  w4[j][i] = s2 + j < nsplit ? __ldcg(pbase + (int64_t)(s2 + j) * NT * kTileM + (c * 32 + i) * kTileM)
                                               : 0.0f;
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (s2 + j < nsplit) {
#pragma unroll
                  for (int i = 0; i < CW; ++i) v[i] += w4[j][i];
                }
            }
            apply(c, v);
          }
          if (et == 0) p.counters[tail_j] = 0;  // ready for the next call
        }
      }
    }
    // an early exit (timed-out wait) still passes the cluster barriers
    if (p.csplit > 1)
      for (; csyncs < 2; ++csyncs) cluster_sync();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TCOLS);
  }
}

template <int NT>
int launch_gemm(dsb_ctx* ctx, const dsb_linear_args* a, int max_splits, int m_tiles, bool offsets_ready) {
  using S = GemmShape<NT>;
  CUtensorMap map_w, map_x;
  const uint64_t w_rows = (uint64_t)a->G * a->M;
  int rc = make_tmap_2d(ctx, &map_w, a->w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->K, w_rows, a->ldw * 2, kBK, kTileM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != DSB_OK) return rc;
  rc = make_tmap_2d(ctx, &map_x, a->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)a->ldx, (uint64_t)a->T,
                    a->ldx * 2, kBK, NT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != DSB_OK) return rc;
  GemmParams p;
  p.T = a->T;
  p.M = a->M;
  p.K = a->K;
  p.G = a->G;
  p.x_group_col = a->x_group_col;
  p.tok_offsets = a->tok_offsets;
  p.y = a->y;
  p.ldy = a->ldy;
  p.y_group_col = a->y_group_col;
  p.y_f32 = a->y_f32;
  p.epi = a->epilogue;
  p.row_scale = a->row_scale;
  p.max_splits = max_splits;
  p.m_tiles = m_tiles;
  p.ws = nullptr;
  p.counters = nullptr;
  p.vec_out = vec_out_ok(a->y, a->y_f32, a->ldy, a->y_group_col,
                         a->epilogue == DSB_EPI_SILU_GATE ? a->M / 2 : a->M) ? 1 : 0;
  p.offsets_ready = (offsets_ready && a->tok_offsets != nullptr) ? 1 : 0;
  p.csplit = 0;
  auto kern = gemm_bf16_kernel<NT>;
  static std::atomic<bool> attr_set[kMaxDevices];
  if (int rc2 = smem_attr_once(ctx, kern, S::SMEM, attr_set); rc2 != DSB_OK) return rc2;
  // A grouped launch's units are known only on the device (sched.cuh), so it
  // takes every SM; a dense one launches no more CTAs than it has work items.
  int grid = ctx->sm_count;
  if (a->tok_offsets == nullptr) {
    const int units = a->G * m_tiles * ((a->T + NT - 1) / NT);
    const SchedShape sh = sched_shape(units, grid, max_splits);
    grid = std::min(grid, sh.items);
    if (sh.full == 0 && sh.splits > 1 && p.vec_out &&
        (a->epilogue == DSB_EPI_STORE || a->epilogue == DSB_EPI_ADD)) {
      // one round of split units: the splits of a unit as one cluster, as
      // many splits as lets every cluster be resident at once
      static std::atomic<int> fit[kMaxDevices][9];
      int cs = std::min(sh.splits, 8);
      for (; cs > 1; --cs) {
        std::atomic<int>& f = fit[ctx->device % kMaxDevices][cs];
        int n = f.load();
        if (n == 0) {
          cudaLaunchConfig_t qc{};
          qc.gridDim = dim3((unsigned)(units * cs));
          qc.blockDim = dim3(kThreads);
          qc.dynamicSmemBytes = S::SMEM;
          cudaLaunchAttribute qa[1];
          qa[0].id = cudaLaunchAttributeClusterDimension;
          qa[0].val.clusterDim.x = (unsigned)cs;
          qa[0].val.clusterDim.y = 1;
          qa[0].val.clusterDim.z = 1;
          qc.attrs = qa;
          qc.numAttrs = 1;
          if (cudaOccupancyMaxActiveClusters(&n, kern, &qc) != cudaSuccess) {
            (void)cudaGetLastError();
            n = -1;  // not available: the ticket reduction
          }
          f.store(n == 0 ? -1 : n);
        }
        if (n >= units) break;
      }
      if (cs > 1) {
        p.csplit = cs;
        max_splits = cs;
        grid = units * cs;
      }
    }
  }
  grid = std::max(grid, 1);
  if (max_splits > 1 && p.csplit == 0) {
    // split partials and tickets: at most one per CTA of the last round
    rc = ensure_workspace(ctx, (size_t)grid * NT * kTileM * sizeof(float));
    if (rc != DSB_OK) return rc;
    rc = ensure_counters(ctx, grid);
    if (rc != DSB_OK) return rc;
    p.ws = static_cast<float*>(ctx->ws);
    p.counters = ctx->counters;
  }
  p.max_splits = max_splits;
  if (p.csplit > 1) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = S::SMEM;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.csplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    DSB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, map_w, map_x, p, ctx->d_status));
  } else {
    DSB_CUDA_TRY(ctx, launch_pdl(kern, grid, kThreads, S::SMEM, ctx->stream, map_w, map_x, p, ctx->d_status));
  }
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches++;
  ctx->stats.gemm_calls++;
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

extern "C" int dsb_linear(dsb_ctx* ctx, const dsb_linear_args* a) { return dsb::linear_ex(ctx, a, false); }

int dsb::linear_ex(dsb_ctx* ctx, const dsb_linear_args* a, bool offsets_ready) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (a == nullptr || a->w == nullptr || a->x == nullptr || a->y == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_linear: null argument");
  if (a->T <= 0 || a->M <= 0 || a->K <= 0 || a->G <= 0 || a->G > kSchedMaxGroups || a->ldw < a->K || a->ldx <= 0)
    return fail(ctx, DSB_EINVAL, "dsb_linear: bad sizes T=%d M=%d K=%d G=%d (G <= %d)", a->T, a->M, a->K, a->G,
                kSchedMaxGroups);
  if ((a->K % 64) || (a->ldw % 8) || (a->ldx % 8) || (a->x_group_col % 8))
    return fail(ctx, DSB_EINVAL, "dsb_linear: K must be a multiple of 64, row pitches and group column offsets multiples of 8");
  if (a->epilogue < DSB_EPI_STORE || a->epilogue > DSB_EPI_ROWSCALE)
    return fail(ctx, DSB_EINVAL, "dsb_linear: unknown epilogue %d", a->epilogue);
  if (a->epilogue == DSB_EPI_SILU_GATE && (a->M % kTileM) != 0)
    return fail(ctx, DSB_EINVAL, "dsb_linear: SiLU-gate needs M (gate+up rows) to be a multiple of 128");
  if (a->epilogue == DSB_EPI_ADD && !a->y_f32)
    return fail(ctx, DSB_EINVAL, "dsb_linear: the residual-add epilogue needs an fp32 output");
  if (a->epilogue == DSB_EPI_ROWSCALE && a->row_scale == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_linear: row-scale epilogue needs row_scale");
  const int bound = a->max_tokens_per_group > 0 ? a->max_tokens_per_group : a->T;
  const int m_tiles = (a->M + kTileM - 1) / kTileM;
  const int KB = (a->K + kBK - 1) / kBK;
  int NT = 16;
  while (NT < bound && NT < 256) NT *= 2;
  // K splits of the units of the partial last round (sched.cuh): a small
  // dense GEMM (fewer units than SMs) takes the cost model's choice, so the
  // SMs share its weight stream; otherwise parts of at least 8 K blocks
  int max_splits = std::max(1, std::min(8, KB / 8));
  if (a->tok_offsets == nullptr) {
    const int units = a->G * m_tiles * ((a->T + NT - 1) / NT);
    if (units < ctx->sm_count) max_splits = pick_splits(units, KB, ctx->sm_count, 4, 128.0 * a->K * 2, NT);
  }
  switch (NT) {
    case 16: return launch_gemm<16>(ctx, a, max_splits, m_tiles, offsets_ready);
    case 32: return launch_gemm<32>(ctx, a, max_splits, m_tiles, offsets_ready);
    case 64: return launch_gemm<64>(ctx, a, max_splits, m_tiles, offsets_ready);
    case 128: return launch_gemm<128>(ctx, a, max_splits, m_tiles, offsets_ready);
    default: return launch_gemm<256>(ctx, a, max_splits, m_tiles, offsets_ready);
  }
}
