// Grouped bf16 linear layer on tcgen05, weights as the 128-row A operand
// ("swap AB"): for group g, token rows t and output features n
//     y[t, g*y_group_col + n] = sum_k x[t, g*x_group_col + k] * W[g*M + n, k]
// One CTA owns a 128-feature tile of one group (and a K split), streams its
// weight tile once through a TMA ring, and multiplies it against all of the
// group's tokens held as the N side of the MMA (16..256 columns).  Decode
// GEMMs have few tokens per weight row, so the weight stream is the roofline
// and the token count only sets the TMEM width.
//
// Replaces cublasSgemv / cublasGemmEx in gemv_row_major_mixed
// (src/models/deepseek/cuda_backend.cpp:459-498), the GEMV chains of
// dense_mlp_to_slot / moe_to_slot (cuda_backend.cpp:820-883) and the
// ds_silu_mul_kernel / ds_scale_add_kernel elementwise passes
// (src/ops/cuda/elementwise_kernels.cu:35-45), which become epilogues.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2-5
// epilogue (warp w reads TMEM lanes 32*(w%4)..+31 = feature rows).
// Split-K (dense groups with <= 256 tokens only): every split writes an fp32
// partial, the last split to finish (atomic ticket) sums the partials in split
// order - deterministic - and runs the epilogue.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

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
  int splits;
  int m_tiles;
  float* ws;          // split partials
  int* counters;      // per-tile tickets (zeroed; reset by the last split)
};

template <int NT>
struct GemmShape {
  static constexpr int A_BYTES = kTileM * kBK * 2;  // 16 KB
  static constexpr int B_BYTES = NT * kBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NS = NT <= 32 ? 6 : (NT <= 64 ? 5 : (NT <= 128 ? 4 : 3));
  static constexpr int XCH_BYTES = 64 * 32 * 4;  // SiLU exchange chunk
  static constexpr int OFF_XCH = NS * STAGE;
  static constexpr int OFF_BAR = OFF_XCH + XCH_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + (2 * NS + 4) * 8;
  static constexpr int SMEM = OFF_MISC + 32 + 1024;
  static constexpr uint32_t TCOLS = NT < 32 ? 32 : NT;
  static_assert(STAGE % 1024 == 0, "stage alignment");
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int NT>
__global__ void __launch_bounds__(kThreads)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                     GemmParams p, int* status) {
  using S = GemmShape<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* empty = full + S::NS;
  uint64_t* d_full = empty + S::NS;
  uint64_t* d_empty = d_full + 1;
  uint64_t* drain = d_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);
  volatile int* no_abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 8);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 12);
  float* xch = reinterpret_cast<float*>(smem + S::OFF_XCH);

  const int mt = blockIdx.x, g = blockIdx.y, split = blockIdx.z;
  int tok0 = 0, tok1 = p.T;
  if (p.tok_offsets != nullptr) {
    tok0 = p.tok_offsets[g];
    tok1 = p.tok_offsets[g + 1];
  }
  const int ntok = tok1 - tok0;
  if (ntok <= 0) return;  // uniform across the CTA: nothing allocated yet
  const int n_ttiles = (ntok + NT - 1) / NT;
  const int KB = (p.K + kBK - 1) / kBK;
  const int kb0 = (int)((int64_t)split * KB / p.splits), kb1 = (int)((int64_t)(split + 1) * KB / p.splits);
  const int nkb = kb1 - kb0;
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, 128);
    mbar_init(drain, 1);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);
  const int total = n_ttiles * nkb;  // (token tile, k block) steps in order

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights stream once; activations stay in L2
      int issued = 0;
      for (int i = 0; i < total; ++i) {
        const int s = i % S::NS;
        if (i >= S::NS && !mbar_wait(&empty[s], ((i / S::NS) - 1) & 1, abort)) {
          raise_abort(abort, status, kStatusTimeout);
          break;
        }
        const int nt = i / nkb, kb = kb0 + i % nkb;
        uint8_t* st = smem + s * S::STAGE;
        mbar_arrive_expect_tx(&full[s], S::STAGE);
        tma_load_2d(st, &map_w, &full[s], kb * kBK, g * p.M + mt * kTileM, pol_w);
        tma_load_2d(st + S::A_BYTES, &map_x, &full[s], (int)(g * p.x_group_col + kb * kBK), tok0 + nt * NT);
        ++issued;
      }
      if (*abort) {
        const int first = issued > S::NS ? issued - S::NS : 0;
        for (int i = first; i < issued; ++i) mbar_wait(&full[i % S::NS], (i / S::NS) & 1, no_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(kTileM, NT < 16 ? 16 : NT, 0, 0);
      bool ok = true;
      for (int i = 0; ok && i < total; ++i) {
        const int s = i % S::NS;
        const int nt = i / nkb, kk = i % nkb;
        if (kk == 0 && nt > 0 && !mbar_wait(d_empty, (nt - 1) & 1, abort)) { ok = false; break; }
        if (!mbar_wait(&full[s], (i / S::NS) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a = sbase + s * S::STAGE, b = a + S::A_BYTES;
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          mma_bf16_ss(tmem, smem_desc(a + ks * 32, 16, 1024, kSwizzle128B), smem_desc(b + ks * 32, 16, 1024, kSwizzle128B),
                      IDESC, (kk > 0 || ks > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
        if (kk == nkb - 1) tc_commit(d_full);
      }
      if (!ok) raise_abort(abort, status, kStatusTimeout);
      tc_commit(drain);
      mbar_wait(drain, 0, no_abort);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const uint32_t q = warp & 3;  // TMEM lane quarter of this warp
    const int r = (int)(q * 32 + lane);  // weight row within the tile
    const uint32_t taddr = tmem + ((q * 32) << 16);
    const int et = threadIdx.x - 64;  // 0..127
    for (int nt = 0; nt < n_ttiles; ++nt) {
      if (!__all_sync(0xffffffffu, mbar_wait(d_full, nt & 1, abort))) {
        raise_abort(abort, status, kStatusTimeout);
        break;
      }
      tc_fence_after();
      const int tbase = tok0 + nt * NT;
      const int tcount = min(NT, tok1 - tbase);
      const int tile_id = g * p.m_tiles + mt;
      bool do_epi = true;
      if (p.splits > 1) {
        // write this split's partial, then the last split reduces
        float* part = p.ws + ((int64_t)tile_id * p.splits + split) * (int64_t)NT * kTileM;
        for (int c = 0; c < (NT < 32 ? 1 : NT / 32); ++c) {
          uint32_t v[32];
          tmem_ld32(taddr + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i < NT) part[(c * 32 + i) * kTileM + r] = __uint_as_float(v[i]);
        }
        __threadfence();
        epi_bar();
        if (et == 0) {
          const int prev = atomicAdd(&p.counters[tile_id], 1);
          *last_flag = (prev == p.splits - 1) ? 1 : 0;
        }
        epi_bar();
        do_epi = *last_flag != 0;
        if (do_epi) __threadfence();
      }
      if (do_epi) {
        // columns of this thread's output feature
        const bool silu = p.epi == DSB_EPI_SILU_GATE;
        const int feat = silu ? mt * 64 + (r & 63) : mt * kTileM + r;
        const bool row_ok = silu ? true : (mt * kTileM + r < p.M);
        const int64_t col = (int64_t)g * p.y_group_col + feat;
        for (int c = 0; c < (NT < 32 ? 1 : NT / 32); ++c) {
          float acc[32];
          if (p.splits > 1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
            for (int s2 = 0; s2 < p.splits; ++s2) {
              const float* part = p.ws + ((int64_t)tile_id * p.splits + s2) * (int64_t)NT * kTileM;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (c * 32 + i < NT) acc[i] += __ldcg(part + (c * 32 + i) * kTileM + r);
            }
          } else {
            uint32_t v[32];
            tmem_ld32(taddr + c * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(v[i]);
          }
          if (silu) {
            // rows 64..127 of the tile are the up projections of rows 0..63
            if (r >= 64) {
#pragma unroll
              for (int i = 0; i < 32; ++i) xch[(r - 64) * 32 + ((i + r) & 31)] = acc[i];
            }
            epi_bar();
            if (r < 64) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int t = c * 32 + i;
                if (t < tcount) {
                  const float gt = acc[i], up = xch[r * 32 + ((i + r + 64) & 31)];
                  const float hval = gt / (1.0f + __expf(-gt)) * up;
                  const int64_t o = (int64_t)(tbase + t) * p.ldy + col;
                  if (p.y_f32) static_cast<float*>(p.y)[o] = hval;
                  else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(hval);
                }
              }
            }
            epi_bar();
          } else if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int t = c * 32 + i;
              if (t < tcount) {
                const int64_t o = (int64_t)(tbase + t) * p.ldy + col;
                float v = acc[i];
                if (p.epi == DSB_EPI_ROWSCALE) v *= p.row_scale[tbase + t];
                if (p.epi == DSB_EPI_ADD) {
                  static_cast<float*>(p.y)[o] += v;
                } else if (p.y_f32) {
                  static_cast<float*>(p.y)[o] = v;
                } else {
                  static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v);
                }
              }
            }
          }
        }
        if (p.splits > 1 && et == 0) p.counters[tile_id] = 0;  // ready for the next call
      }
      tc_fence_before();
      mbar_arrive(d_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TCOLS);
  }
}

template <int NT>
int launch_gemm(dsb_ctx* ctx, const dsb_linear_args* a, int splits, int m_tiles) {
  using S = GemmShape<NT>;
  CUtensorMap map_w, map_x;
  const uint64_t w_rows = (uint64_t)a->G * a->M;
  int rc = make_tmap_2d(ctx, &map_w, a->w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->K, w_rows, a->ldw * 2, kBK, kTileM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != DSB_OK) return rc;
  const uint64_t x_cols = (uint64_t)a->ldx;
  rc = make_tmap_2d(ctx, &map_x, a->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x_cols, (uint64_t)a->T, a->ldx * 2, kBK,
                    NT, CU_TENSOR_MAP_SWIZZLE_128B);
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
  p.splits = splits;
  p.m_tiles = m_tiles;
  p.ws = nullptr;
  p.counters = nullptr;
  if (splits > 1) {
    const size_t tiles = (size_t)m_tiles * a->G;
    const size_t part_bytes = tiles * splits * NT * kTileM * sizeof(float);
    const size_t ctr_off = (part_bytes + 255) & ~size_t(255);
    rc = ensure_workspace(ctx, ctr_off + tiles * sizeof(int));
    if (rc != DSB_OK) return rc;
    rc = ensure_counters(ctx, tiles);
    if (rc != DSB_OK) return rc;
    p.ws = static_cast<float*>(ctx->ws);
    p.counters = ctx->counters;
  }
  auto kern = gemm_bf16_kernel<NT>;
  static bool attr_set = false;
  if (!attr_set) {
    DSB_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM));
    attr_set = true;
  }
  dim3 grid((unsigned)m_tiles, (unsigned)a->G, (unsigned)splits);
  kern<<<grid, kThreads, S::SMEM, ctx->stream>>>(map_w, map_x, p, ctx->d_status);
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches++;
  ctx->stats.gemm_calls++;
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

extern "C" int dsb_linear(dsb_ctx* ctx, const dsb_linear_args* a) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (a == nullptr || a->w == nullptr || a->x == nullptr || a->y == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_linear: null argument");
  if (a->T <= 0 || a->M <= 0 || a->K <= 0 || a->G <= 0 || a->ldw < a->K || a->ldx <= 0)
    return fail(ctx, DSB_EINVAL, "dsb_linear: bad sizes T=%d M=%d K=%d G=%d", a->T, a->M, a->K, a->G);
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
  int splits = 1;
  if (a->tok_offsets == nullptr && a->T <= 256) {
    const int tiles = m_tiles * a->G;
    const int want = (2 * ctx->sm_count) / std::max(1, tiles);
    splits = std::max(1, std::min({want, KB / 4, 16}));
  }
  int NT = 16;
  while (NT < bound && NT < 256) NT *= 2;
  switch (NT) {
    case 16: return launch_gemm<16>(ctx, a, splits, m_tiles);
    case 32: return launch_gemm<32>(ctx, a, splits, m_tiles);
    case 64: return launch_gemm<64>(ctx, a, splits, m_tiles);
    case 128: return launch_gemm<128>(ctx, a, splits, m_tiles);
    default: return launch_gemm<256>(ctx, a, splits, m_tiles);
  }
}
