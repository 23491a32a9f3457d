// Grouped FP8 (e4m3) linear layer with DeepSeek-V3 block scaling, on tcgen05:
//     y[t, g*y_group_col + n] = sum_kb  sw(g, n, kb) * sx[t, kb]
//                               * sum_{k in block kb} xq[t, g*x_group_col + k] * wq[g*M + n, k]
// wq e4m3 with one fp32 scale per 128x128 block, xq e4m3 with one fp32 scale
// per token and 128 columns (dsb_quant_act_1x128).
//
// The scales change every 128 columns of K, so the tensor cores cannot carry
// one accumulator across K: each 128-deep K block is its own 4-instruction
// kind::f8f6f4 MMA chain into one of the TMEM partial buffers (a ring that
// fills all 512 columns), and the epilogue warps promote it - acc += partial *
// sw * sx[t] in fp32 registers - while the MMAs of later blocks fill the
// other buffers.
//
// Same tiling as the bf16 kernel: weights are the 128-row A operand ("swap
// AB"), tokens the N side (16..128 columns), one persistent CTA per SM walks
// the work units of a schedule built on the device (sched.cuh), the TMA ring
// streams across unit boundaries, and split units write fp32 partials
// reduced in split order by the last split.  One stage (128 weight rows x 128
// bytes) is exactly one scale block and one 128-byte swizzle row.
//
// The reference has no FP8 path (its safetensors dtype parser stops at
// F32/F16/BF16, src/hf/safetensors.cpp:12-20); this replaces the expert and
// linear GEMVs of moe_to_slot / linear_to_slot (src/models/deepseek/
// cuda_backend.cpp:782-883) for block-scaled FP8 checkpoints.
//
// Roles: warp 0 TMA producer, warp 1 MMA issuer, the other warps promotion +
// epilogue (warp w owns TMEM lanes 32*(w%4)..+31 and all, or from 64 tokens up
// half, of the token columns); up to 32 tokens two such groups take
// alternate K blocks; 320 threads in every case.

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

constexpr int kBK = 128;      // K bytes (e4m3 elements) per stage = one scale block
constexpr int kTileM = 128;   // weight rows per tile (MMA M)

struct Fp8Params {
  int T, M, K, G;
  int64_t x_group_col;         // elements (= bytes)
  const int32_t* tok_offsets;  // [G+1] or null
  const float* w_scale;        // [(G*m_tiles)*scale_rows, K/128]
  int scale_rows;              // 1, or 2 for row-interleaved gate|up
  const float* x_scale;        // [T, ld_xs]
  int64_t ld_xs;
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
};

template <int NT>
struct Fp8Shape {
  static constexpr int A_BYTES = kTileM * kBK;  // 16 KB
  static constexpr int B_BYTES = NT * kBK;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  // TMEM partial buffers filling all 512 columns: the MMAs run up to NBUF-1
  // K blocks ahead of the promotion (and through the epilogue of a unit)
  static constexpr int NBUF = 512 / (NT < 32 ? 32 : NT);
  static constexpr int CG = NT < 64 ? 1 : 2;        // token-column groups of the epilogue
  static constexpr int KG = NT < 64 ? 2 : 1;        // epilogue groups taking alternate K blocks
  static_assert(CG == 1 || KG == 1, "column groups or K groups, not both");
  static constexpr int GT = 128 * CG;               // threads of one K group: 4 lane quarters x CG
  static constexpr int EPI = GT * KG;
  static constexpr int THREADS = 64 + EPI;
  static constexpr int HC = NT / CG;                // token columns per epilogue thread
  static constexpr int XCH = KG > 1 ? kTileM * NT * 4 : 0;    // odd group's sums for the even group
  static constexpr int SX = (EPI / 32) * 4 * HC * 4;          // [warps][2 buffers][2 row parities][HC]
  static constexpr int RS = (EPI / 32) * NT * 4;              // [warps][NT] token weights (ROWSCALE)
  static constexpr int STG = (GT / 32) * 32 * 32 * 4;         // output staging of the writing warps
  static constexpr int SCH = ((int)sizeof(SchedTable) + 15) / 16 * 16;  // work schedule table
  static constexpr int NS = (212 * 1024 - XCH - SX - RS - STG - SCH) / STAGE;  // ring depth
  static constexpr int OFF_BAR = NS * STAGE;
  static constexpr int OFF_MISC = OFF_BAR + (2 * NS + 2 * NBUF + 4) * 8;
  static constexpr int OFF_XCH = OFF_MISC + 64;
  static constexpr int OFF_SX = OFF_XCH + XCH;
  static constexpr int OFF_RS = OFF_SX + SX;
  static constexpr int OFF_STG = OFF_RS + RS;
  static constexpr int OFF_SCHED = OFF_STG + STG;
  static constexpr int SMEM = OFF_SCHED + SCH + 1024;
  static constexpr uint32_t TC = NT < 32 ? 32 : NT;  // TMEM columns per partial buffer
  static constexpr uint32_t TCOLS = NBUF * TC;       // <= 512
  static_assert(STAGE % 1024 == 0, "stage alignment");
  static_assert(SMEM <= 232448, "shared memory");
};

template <int NT>
__global__ void __launch_bounds__(Fp8Shape<NT>::THREADS, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                    Fp8Params p, int* status) {
  using S = Fp8Shape<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* empty = full + S::NS;
  uint64_t* part_full = empty + S::NS;        // [NBUF] partial buffer written by one K block's MMAs
  uint64_t* part_empty = part_full + S::NBUF; // [NBUF] partial buffer promoted by the epilogue
  uint64_t* drain = part_empty + S::NBUF;
  uint64_t* xch_full = drain + 1;   // the odd K group's sums are in xch
  uint64_t* xch_empty = drain + 2;  // the even K group has read them
  uint64_t* epi_bar = drain + 3;    // rendezvous of the even K group (split-K ticket)
  float* xch = reinterpret_cast<float*>(smem + S::OFF_XCH);  // [NT][128]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);
  volatile int* no_abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 8);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 12);
  float* sx_smem = reinterpret_cast<float*>(smem + S::OFF_SX);

  const int KB = p.K / kBK;
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < S::NBUF; ++b) {
      mbar_init(&part_full[b], 1);
      mbar_init(&part_empty[b], S::GT / 32);  // one arrival per warp of the K group reading the buffer
    }
    mbar_init(drain, 1);
    mbar_init(xch_full, S::GT / 32);  // (warp counts)
    mbar_init(xch_empty, S::GT / 32);
    mbar_init(epi_bar, S::GT / 32);
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
      const uint64_t pol_w = l2_policy_evict_first();
      SchedIter it{sched, p.m_tiles, NT, KB};
      int q = 0;
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
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_e4m3_f32(kTileM, NT < 16 ? 16 : NT);
      SchedIter it{sched, p.m_tiles, NT, KB};
      int q = 0, pk = 0;
      bool ok = true;
      while (ok && it.next()) {
        const int kb0 = it.kb0, kb1 = it.kb1;
        for (int kb = kb0; kb < kb1; ++kb, ++q, ++pk) {
          const int s = q % S::NS, b = pk % S::NBUF;
          if (pk >= S::NBUF && !mbar_wait(&part_empty[b], ((pk / S::NBUF) - 1) & 1, abort)) { ok = false; break; }
          if (!mbar_wait(&full[s], (q / S::NS) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem + b * S::TC;
          const uint32_t a = sbase + s * S::STAGE, bb = a + S::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < kBK / 32; ++ks) {
            mma_f8_ss(d, smem_desc(a + ks * 32, 16, 1024, kSwizzle128B), smem_desc(bb + ks * 32, 16, 1024, kSwizzle128B),
                      IDESC, ks > 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&part_full[b]);
        }
      }
      if (!ok) raise_abort(abort, status, kStatusTimeout);
      tc_commit(drain);
      mbar_wait(drain, 0, no_abort);
    }
  } else {
    // ------------------------------------------------- promotion + epilogue
    // Warp w reads TMEM lanes 32*(w%4)..+31 (weight rows of the tile) and
    // token columns [cg*HC, (cg+1)*HC); with KG = 2 two groups of such warps
    // take alternate K blocks (by the parity of the running partial index),
    // each summing its own blocks, and the even group adds the odd group's
    // sums (handed over in shared memory) before the epilogue.
    constexpr int HC = S::HC;              // token columns per thread (16, 32 or 64)
    constexpr int LW = HC < 32 ? HC : 32;  // columns per tcgen05.ld
    constexpr int NL = HC / LW;            // loads per K block
    constexpr int PER = (HC + 31) / 32;    // token scales loaded per lane
    const uint32_t qtr = warp & 3;
    // with KG = 2, CG = 1: warps 2-5 are K group 0, warps 6-9 K group 1
    const int kg = S::KG == 1 ? 0 : (int)((warp - 2) >> 2);
    const int c0 = S::KG == 1 ? (int)((warp - 2) >> 2) * HC : 0;  // this thread's first token column
    const int r = (int)(qtr * 32 + lane);         // weight row within the tile (parity = lane parity)
    const int et = (int)threadIdx.x - 64 - kg * S::GT;  // index within the K group
    const bool silu = p.epi == DSB_EPI_SILU_GATE;
    // this warp's scale vectors: [2 buffers][row parity][HC], sw(row) * sx[t] of one K block
    float* sxw = sx_smem + (warp - 2) * 4 * HC;
    // this warp's copy of the unit's token weights (ROWSCALE), read by the epilogue
    float* rsw = reinterpret_cast<float*>(smem + S::OFF_RS) + (warp - 2) * NT;
    // output staging block of the warps that write (the even K group's, or all)
    float* stg = reinterpret_cast<float*>(smem + S::OFF_STG) + ((warp - 2) % (S::GT / 32)) * 32 * 32;
    int epi_phase = 0;
    SchedIter it{sched, p.m_tiles, NT, KB};
    int pk = 0, own = 0, u = 0;  // running partial index, K blocks this group promoted (KG > 1), units
    bool ok = true;
    while (ok && it.next()) {
      const int tbase = it.tok0 + it.nt * NT;
      const int tcount = min(NT, it.tok1 - tbase);
      const int wtile = it.g * p.m_tiles + it.mt;  // weight tile (its scale rows)
      const int kb0 = it.kb0, kb1 = it.kb1;
      const float* ws_even = p.w_scale + (int64_t)wtile * p.scale_rows * KB;
      const float* ws_odd = ws_even + (int64_t)(p.scale_rows - 1) * KB;
      const float* sxrow = p.x_scale + it.g * (p.x_group_col / kBK);
      if (p.epi == DSB_EPI_ROWSCALE && kg == 0) {
        // fetched now, used after the K loop (no load waits in the epilogue)
        __syncwarp();
        for (int j = (int)lane; j < NT; j += 32) rsw[j] = j < tcount ? __ldg(p.row_scale + tbase + j) : 0.0f;
        __syncwarp();
      }
      float acc[HC];
#pragma unroll
      for (int i = 0; i < HC; ++i) acc[i] = 0.0f;
      // The scales of the next K block are fetched (one value per lane) while
      // the current one is promoted, then stored premultiplied by the weight
      // scale of each row parity, so the promotion is one FMA per element.
      // The loads run two of this group's K blocks ahead (registers nx/nwe/nwo
      // hold the next block's scales, qx/qwe/qwo the one after), so an L2
      // round trip has two promotion periods to land.
      float nx[PER], nwe = 0.0f, nwo = 0.0f;
      float qx[PER], qwe = 0.0f, qwo = 0.0f;
      auto fetch = [&](int kb, float (&x)[PER], float& we, float& wo) {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          const int i = (int)lane + 32 * j, t = c0 + i;
          x[j] = (i < HC && t < tcount) ? __ldg(sxrow + (int64_t)(tbase + t) * p.ld_xs + kb) : 0.0f;
        }
        we = __ldg(ws_even + kb);
        wo = __ldg(ws_odd + kb);
      };
      auto load_sx = [&](int kb) { fetch(kb, nx, nwe, nwo); };
      auto store_sx = [&](int buf) {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          const int i = (int)lane + 32 * j;
          if (i < HC) {
            sxw[(buf * 2 + 0) * HC + i] = nwe * nx[j];
            sxw[(buf * 2 + 1) * HC + i] = nwo * nx[j];
          }
        }
      };
      // this group's first K block of the unit
      const int kbf = S::KG == 1 ? kb0 : kb0 + (int)((kg - pk % S::KG + S::KG) % S::KG);
      if (S::KG == 1 || kbf < kb1) {
        __syncwarp();
        load_sx(kbf);
        store_sx((S::KG == 1 ? pk : own) & 1);
        __syncwarp();
        if (kbf + S::KG < kb1) load_sx(kbf + S::KG);
      }
      for (int kb = kb0; kb < kb1; ++kb, ++pk) {
        if (S::KG > 1 && pk % S::KG != kg) continue;
        const int b = pk % S::NBUF, sb = (S::KG == 1 ? pk : own) & 1;  // TMEM partial buffer, scale buffer
        if constexpr (S::KG > 1) ++own;
        if (kb + 2 * S::KG < kb1) fetch(kb + 2 * S::KG, qx, qwe, qwo);
        if (!__all_sync(0xffffffffu, mbar_wait(&part_full[b], (pk / S::NBUF) & 1, abort))) {
          raise_abort(abort, status, kStatusTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + ((qtr * 32) << 16) + b * S::TC + c0;
        const float4* s4 = reinterpret_cast<const float4*>(sxw + (sb * 2 + (int)(lane & 1)) * HC);
#pragma unroll
        for (int l = 0; l < NL; ++l) {
          uint32_t raw[LW];
          if constexpr (LW == 32) tmem_ld32(taddr + l * LW, raw);
          else if constexpr (LW == 16) tmem_ld16(taddr + l * LW, raw);
          else tmem_ld8(taddr + l * LW, raw);
          tmem_ld_wait();
          if (l == NL - 1) {
            // the partial buffer is free once it has been read into registers
            tc_fence_before();
            warp_arrive(&part_empty[b]);
          }
#pragma unroll
          for (int i = 0; i < LW; i += 4) {
            const int ci = l * LW + i;
            const float4 sv = s4[ci >> 2];
            acc[ci] = fmaf(__uint_as_float(raw[i]), sv.x, acc[ci]);
            acc[ci + 1] = fmaf(__uint_as_float(raw[i + 1]), sv.y, acc[ci + 1]);
            acc[ci + 2] = fmaf(__uint_as_float(raw[i + 2]), sv.z, acc[ci + 2]);
            acc[ci + 3] = fmaf(__uint_as_float(raw[i + 3]), sv.w, acc[ci + 3]);
          }
        }
        if (kb + S::KG < kb1) {
          __syncwarp();  // every lane is done with the buffer written next
          store_sx(sb ^ 1);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < PER; ++j) nx[j] = qx[j];
          nwe = qwe;
          nwo = qwo;
        }
      }
      if (!ok) break;
      if constexpr (S::KG > 1) {
        // hand the odd group's sums to the even group (bounded waits)
        if (kg == 1) {
          if (u > 0 && !__all_sync(0xffffffffu, mbar_wait(xch_empty, (u - 1) & 1, abort))) {
            raise_abort(abort, status, kStatusTimeout);
            break;
          }
#pragma unroll
          for (int i = 0; i < HC; ++i) xch[(c0 + i) * kTileM + r] = acc[i];
          warp_arrive(xch_full);
          ++u;
          continue;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(xch_full, u & 1, abort))) {
          raise_abort(abort, status, kStatusTimeout);
          break;
        }
#pragma unroll
        for (int i = 0; i < HC; ++i) acc[i] = __fadd_rn(acc[i], xch[(c0 + i) * kTileM + r]);
        warp_arrive(xch_empty);
        ++u;
      }

      auto apply = [&](float (&v)[HC]) {  // called by all lanes of the warp
        constexpr int BT = HC < 32 ? HC : 32;  // token rows per staged block
        if (silu) {
          // rows 2j / 2j+1 of the tile are gate / up of output feature 64*mt + j
          // in place: the partner lane's v[i] is read before either lane rewrites it
#pragma unroll
          for (int i = 0; i < HC; ++i) {
            const float up = __shfl_xor_sync(0xffffffffu, v[i], 1);
            v[i] = v[i] / (1.0f + __expf(-v[i])) * up;
          }
          if (p.vec_out) {
            const int64_t col0 = (int64_t)it.g * p.y_group_col + it.mt * 64 + qtr * 16;
            warp_store_block<BT, true, 0>(stg, v, lane, tcount - c0, 16, p.y, p.ldy, col0, tbase + c0, p.y_f32, false);
            if constexpr (HC > BT)
              warp_store_block<BT, true, BT>(stg, v, lane, tcount - c0 - BT, 16, p.y, p.ldy, col0, tbase + c0 + BT,
                                             p.y_f32, false);
            return;
          }
          const int64_t col = (int64_t)it.g * p.y_group_col + it.mt * 64 + (r >> 1);
#pragma unroll
          for (int i = 0; i < HC; ++i) {
            const int t = c0 + i;
            if ((r & 1) == 0 && t < tcount) {
              const int64_t o = (int64_t)(tbase + t) * p.ldy + col;
              if (p.y_f32) static_cast<float*>(p.y)[o] = v[i];
              else static_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v[i]);
            }
          }
          return;
        }
        // The token weights (ROWSCALE) come from shared memory, staged at the
        // start of the unit (a global load here could not be moved above the
        // previous column's store, which may alias it: one memory round trip
        // per column); the residual add is a reduction into y, which needs no
        // load: each element of y receives exactly one add, so the result is
        // y + x rounded once.
        if (p.epi == DSB_EPI_ROWSCALE) {
#pragma unroll
          for (int i = 0; i < HC; ++i) v[i] *= rsw[c0 + i];
        }
        if (p.vec_out) {
          const int ncols = max(0, min(32, p.M - it.mt * kTileM - (int)qtr * 32));
          const int64_t col0 = (int64_t)it.g * p.y_group_col + it.mt * kTileM + qtr * 32;
          const bool add = p.epi == DSB_EPI_ADD;
          warp_store_block<BT, false, 0>(stg, v, lane, tcount - c0, ncols, p.y, p.ldy, col0, tbase + c0, p.y_f32, add);
          if constexpr (HC > BT)
            warp_store_block<BT, false, BT>(stg, v, lane, tcount - c0 - BT, ncols, p.y, p.ldy, col0, tbase + c0 + BT,
                                            p.y_f32, add);
          return;
        }
        if (it.mt * kTileM + r < p.M) {
          const int64_t col = (int64_t)it.g * p.y_group_col + it.mt * kTileM + r;
#pragma unroll
          for (int i = 0; i < HC; ++i) {
            const int t = c0 + i;
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
      if (nsplit > 1) {
        // split-K: publish this split's promoted sum; the last split reduces
        // (into acc, in split order) and runs the epilogue
        float* part = p.ws + ((int64_t)tail_j * nsplit + it.split) * (int64_t)NT * kTileM;
#pragma unroll
        for (int i = 0; i < HC; ++i) part[(c0 + i) * kTileM + r] = acc[i];
        __threadfence();
        if (!__all_sync(0xffffffffu, mbar_rendezvous(epi_bar, epi_phase, abort))) {  // the even K group only
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
        if (*last_flag == 0) continue;
        __threadfence();
        const float* pbase = p.ws + (int64_t)tail_j * nsplit * (int64_t)NT * kTileM + r;
#pragma unroll
        for (int i = 0; i < HC; ++i) acc[i] = 0.0f;
        for (int s2 = 0; s2 < nsplit; ++s2) {
#pragma unroll
          for (int i = 0; i < HC; ++i) acc[i] += __ldcg(pbase + (int64_t)s2 * NT * kTileM + (c0 + i) * kTileM);
        }
        if (et == 0) p.counters[tail_j] = 0;
      }
      apply(acc);
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
int launch_fp8(dsb_ctx* ctx, const dsb_linear_fp8_args* a, int max_splits, int m_tiles, bool offsets_ready) {
  using S = Fp8Shape<NT>;
  CUtensorMap map_w, map_x;
  const uint64_t w_rows = (uint64_t)a->G * a->M;
  int rc = make_tmap_2d(ctx, &map_w, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, a->K, w_rows, a->ldw, kBK, kTileM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != DSB_OK) return rc;
  rc = make_tmap_2d(ctx, &map_x, a->x, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)a->ldx, (uint64_t)a->T, a->ldx, kBK,
                    NT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != DSB_OK) return rc;
  Fp8Params p;
  p.T = a->T;
  p.M = a->M;
  p.K = a->K;
  p.G = a->G;
  p.x_group_col = a->x_group_col;
  p.tok_offsets = a->tok_offsets;
  p.w_scale = a->w_scale;
  p.scale_rows = a->scale_rows;
  p.x_scale = a->x_scale;
  p.ld_xs = a->ld_xs;
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
  // A grouped launch's units are known only on the device (sched.cuh), so it
  // takes every SM; a dense one launches no more CTAs than it has work items.
  int grid = ctx->sm_count;
  if (a->tok_offsets == nullptr)
    grid = std::min(grid, sched_shape(a->G * m_tiles * ((a->T + NT - 1) / NT), grid, max_splits).items);
  grid = std::max(grid, 1);
  if (max_splits > 1) {
    // split partials and tickets: at most one per CTA of the last round
    rc = ensure_workspace(ctx, (size_t)grid * NT * kTileM * sizeof(float));
    if (rc != DSB_OK) return rc;
    rc = ensure_counters(ctx, grid);
    if (rc != DSB_OK) return rc;
    p.ws = static_cast<float*>(ctx->ws);
    p.counters = ctx->counters;
  }
  auto kern = gemm_fp8_kernel<NT>;
  static std::atomic<bool> attr_set[kMaxDevices];
  if (int rc = smem_attr_once(ctx, kern, S::SMEM, attr_set); rc != DSB_OK) return rc;
  DSB_CUDA_TRY(ctx, launch_pdl(kern, grid, S::THREADS, S::SMEM, ctx->stream, map_w, map_x, p, ctx->d_status));
  DSB_CUDA_TRY(ctx, cudaGetLastError());
  ctx->stats.kernel_launches++;
  ctx->stats.gemm_calls++;
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

extern "C" int dsb_linear_fp8(dsb_ctx* ctx, const dsb_linear_fp8_args* a) { return dsb::linear_fp8_ex(ctx, a, false); }

int dsb::linear_fp8_ex(dsb_ctx* ctx, const dsb_linear_fp8_args* a, bool offsets_ready) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (a == nullptr || a->w == nullptr || a->w_scale == nullptr || a->x == nullptr || a->x_scale == nullptr ||
      a->y == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: null argument");
  if (a->T <= 0 || a->M <= 0 || a->K <= 0 || a->G <= 0 || a->G > kSchedMaxGroups || a->ldw < a->K || a->ldx <= 0 ||
      a->ld_xs <= 0)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: bad sizes T=%d M=%d K=%d G=%d (G <= %d)", a->T, a->M, a->K, a->G,
                kSchedMaxGroups);
  if ((a->K % kBK) || (a->ldw % 16) || (a->ldx % 16) || (a->x_group_col % kBK))
    return fail(ctx, DSB_EINVAL,
                "dsb_linear_fp8: K and group column offsets must be multiples of 128, row pitches multiples of 16");
  if (a->scale_rows != 1 && a->scale_rows != 2)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: scale_rows must be 1 or 2");
  if (a->epilogue < DSB_EPI_STORE || a->epilogue > DSB_EPI_ROWSCALE)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: unknown epilogue %d", a->epilogue);
  if (a->epilogue == DSB_EPI_SILU_GATE && (a->M % kTileM) != 0)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: SiLU-gate needs M (gate+up rows) to be a multiple of 128");
  if (a->epilogue == DSB_EPI_ADD && !a->y_f32)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: the residual-add epilogue needs an fp32 output");
  if (a->epilogue == DSB_EPI_ROWSCALE && a->row_scale == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_linear_fp8: row-scale epilogue needs row_scale");
  const int bound = a->max_tokens_per_group > 0 ? a->max_tokens_per_group : a->T;
  const int m_tiles = (a->M + kTileM - 1) / kTileM;
  const int KB = a->K / kBK;
  int NT = 16;
  while (NT < bound && NT < 128) NT *= 2;
  // K splits of the units of the partial last round (sched.cuh): a small
  // dense GEMM (fewer units than SMs) splits K so the SMs share its weight
  // stream, in one wave of work items (the per-K-block promotion keeps this
  // kernel's per-SM stream rate below the bf16 kernel's, so extra waves cost
  // more than the idle SMs of a partial wave); otherwise parts of at least
  // 8 K blocks
  int max_splits = std::max(1, std::min(8, KB / 8));
  if (a->tok_offsets == nullptr) {
    const int units = a->G * m_tiles * ((a->T + NT - 1) / NT);
    if (units < ctx->sm_count) max_splits = std::max(1, std::min({ctx->sm_count / units, KB / 2, 8}));
  }
  switch (NT) {
    case 16: return launch_fp8<16>(ctx, a, max_splits, m_tiles, offsets_ready);
    case 32: return launch_fp8<32>(ctx, a, max_splits, m_tiles, offsets_ready);
    case 64: return launch_fp8<64>(ctx, a, max_splits, m_tiles, offsets_ready);
    default: return launch_fp8<128>(ctx, a, max_splits, m_tiles, offsets_ready);
  }
}
