// Absorbed MLA decode attention over a paged latent cache, sm_100a.
//
// Math (one query token per sequence, per head h):
//   s_t = ([q_lat_h | q_rope_h] . [c_t | kr_t]) * scale,  p = softmax(s),
//   out_h = sum_t p_t c_t
// which is the reference's per-head attention (src/models/deepseek/mla.cpp:86-116)
// with W_UK folded into the query and W_UV applied after the sum.
//
// Work decomposition.  A work item is a run of whole 64-token pages of one
// sequence.  Each item is processed by a cluster of NCTA CTAs; CTA r owns the
// latent columns [r*VD, (r+1)*VD) (VD = R / NCTA) and rope columns
// [R + r*PD, R + (r+1)*PD) (PD = P / NCTA) of every cache row, so every cache
// byte is read from HBM once.  Per 64-token page:
//   TMA warp   : loads the CTA's column slice of the page (SW128 / SW64 tiles)
//   MMA warp   : S = Q_r K_r^T (tcgen05, A = Q from TMEM, B = page from smem)
//                then O_r += P V_r (A = P from TMEM, B = the same page, MN-major)
//   4 softmax warps (thread i <-> head i <-> TMEM lane i):
//                read S_r, exchange it with the peer CTA (each CTA writes
//                its fp16 partial to a local send buffer, one thread ships
//                the 16 KB tile with a single shared-to-shared bulk copy),
//                S = S_0 + S_1 (bitwise equal in both CTAs),
//                online softmax in the exp2 domain with a lazy running max,
//                write P (bf16) to TMEM.
// TMEM (512 columns): O [VD] | S [64] | P [32] | Q [(VD+PD)/2].
// Items that cover a whole sequence write bf16 output; split sequences write
// fp32 partials (O, running max, sum) merged by mla_combine_kernel.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <queue>
#include <vector>

#include "dsb_internal.h"
#include "dsb_ptx.cuh"

namespace dsb {
namespace {

constexpr int kTok = 64;            // tokens per tile == page size
constexpr int kMaxItemPages = 256;  // pages per work item (16384 tokens)
constexpr int kHeadsPad = 128;      // MMA M (heads padded to 128)
constexpr float kLazyRescale = 8.0f;  // log2 headroom before O is rescaled

struct MlaItem {
  int32_t b;        // sequence
  int32_t page0;    // first page index within the sequence
  int32_t npages;   // pages in this item
  int32_t tok_end;  // absolute end token (exclusive) of this item
  int32_t partial;  // -1: whole sequence, write out; else partial slot
};

struct MlaCombine {
  int32_t b;
  int32_t first;  // first partial slot
  int32_t n;      // number of partial slots
};

template <int R, int P, int NCTA>
struct MlaShape {
  static constexpr int VD = R / NCTA;             // latent columns per CTA
  static constexpr int PD = P / NCTA;             // rope columns per CTA
  static constexpr int QD = VD + PD;              // QK contraction per CTA
  static constexpr int NCH = VD / 64;             // SW128 chunks per page slice
  static constexpr int CH_BYTES = kTok * 128;     // 64 rows x 128 B
  static constexpr int ROPE_BYTES = kTok * PD * 2;
  static constexpr int STAGE_BYTES = NCH * CH_BYTES + ROPE_BYTES;
  static constexpr int NSTAGE = (NCTA == 2) ? 4 : 8;
  static constexpr int XCH_BUF = kHeadsPad * kTok * 2;             // one tile of fp16 partial scores
  // send [2] then receive [2] buffers (double-buffered by page parity)
  static constexpr int XCH_BYTES = (NCTA == 2) ? 4 * XCH_BUF : 0;
  static constexpr int OFF_RECV_REL = 2 * XCH_BUF;
  // TMEM column map
  static constexpr uint32_t T_O = 0;
  static constexpr uint32_t T_S = VD;
  static constexpr uint32_t T_P = VD + 64;
  static constexpr uint32_t T_Q = VD + 96;
  static constexpr uint32_t T_COLS = 512;
  static_assert(T_Q + QD / 2 <= T_COLS, "TMEM overflow");
  static_assert(PD == 32, "rope slice must be 32 columns (SW64 tile)");
  static_assert(VD % 64 == 0, "latent slice must be whole 64-column chunks");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  // shared memory map (offsets from a 1024-aligned base)
  static constexpr int OFF_STAGE = 0;
  static constexpr int OFF_XCH = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_RED = OFF_XCH + XCH_BYTES;  // [3 slots][2 half][128]: row maxima (2 parities), final sums
  static constexpr int OFF_BAR = OFF_RED + 3 * 2 * kHeadsPad * 4;
  static constexpr int NBAR = 2 * NSTAGE + 15;
  static constexpr int OFF_PAGES = OFF_BAR + NBAR * 8;
  static constexpr int OFF_MISC = OFF_PAGES + kMaxItemPages * 4;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static_assert(OFF_XCH % 128 == 0 && XCH_BUF % 16 == 0, "bulk copy alignment");
};

constexpr int kSoftmaxWarps = 8;    // two warps per TMEM lane quarter (column halves)
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kMlaThreads = kSoftmaxThreads + 64;  // + TMA warp + MMA warp

template <int R, int P, int NCTA>
__global__ void __launch_bounds__(kMlaThreads, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_r,
                      const __nv_bfloat16* __restrict__ q_lat, const __nv_bfloat16* __restrict__ q_rope,
                      const int32_t* __restrict__ block_table, int max_blocks, const MlaItem* __restrict__ items,
                      int H, float scale_log2, __nv_bfloat16* __restrict__ out, float* __restrict__ ws_o,
                      float2* __restrict__ ws_ml, int* __restrict__ status) {
  using S = MlaShape<R, P, NCTA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  uint64_t* full = bars;                  // [NSTAGE] page slice landed
  uint64_t* empty = bars + S::NSTAGE;     // [NSTAGE] page slice consumed by PV
  uint64_t* s_full = bars + 2 * S::NSTAGE + 0;
  uint64_t* s_free = bars + 2 * S::NSTAGE + 1;
  uint64_t* p_full = bars + 2 * S::NSTAGE + 2;
  uint64_t* pv_done = bars + 2 * S::NSTAGE + 3;
  uint64_t* q_ready = bars + 2 * S::NSTAGE + 4;
  uint64_t* drain = bars + 2 * S::NSTAGE + 5;
  uint64_t* xch_full = bars + 2 * S::NSTAGE + 6;   // [2] peer's partial S landed in my XCH buffer
  uint64_t* peer_free = bars + 2 * S::NSTAGE + 8;  // [2] peer finished reading its XCH buffer
  uint64_t* red_bar = bars + 2 * S::NSTAGE + 10;   // [2] both column halves posted their row maxima
  uint64_t* fin_bar = bars + 2 * S::NSTAGE + 12;   // both halves posted their softmax sums
  uint64_t* send_ready = bars + 2 * S::NSTAGE + 13;  // [2] every softmax thread wrote its send row
  int32_t* pages = reinterpret_cast<int32_t*>(smem + S::OFF_PAGES);
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);
  // never raised: drain waits keep their time limit but ignore the abort flag
  volatile int* no_abort = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 8);
  float* red = reinterpret_cast<float*>(smem + S::OFF_RED);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = (NCTA == 2) ? cluster_ctarank() : 0u;
  const MlaItem item = items[blockIdx.x / NCTA];
  const int n_tiles = item.npages;
  constexpr uint32_t kTmaWarp = kSoftmaxWarps, kMmaWarp = kSoftmaxWarps + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, kSoftmaxWarps);
    mbar_init(p_full, kSoftmaxWarps);
    mbar_init(pv_done, 1);
    mbar_init(q_ready, kSoftmaxWarps);
    mbar_init(drain, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&xch_full[b], 1);            // the local expect_tx arrival + the peer's 16 KB bulk copy
      mbar_init(&peer_free[b], kSoftmaxWarps);  // one remote arrival per peer softmax warp
      mbar_init(&red_bar[b], kSoftmaxWarps);
    }
    mbar_init(fin_bar, kSoftmaxWarps);
    for (int b = 0; b < 2; ++b) mbar_init(&send_ready[b], kSoftmaxWarps);
    *abort = 0;
    *no_abort = 0;
    // the softmax warps' barriers count warps: each warp arrives once, from
    // lane 0 after a __syncwarp that orders the other lanes' writes (shared
    // memory, and TMEM with their tcgen05 fences) before the arrival
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_base_smem, S::T_COLS);
    tmem_relinquish();
  }
  if (warp == kTmaWarp) {
    for (int i = lane; i < n_tiles; i += 32)
      pages[i] = block_table[(int64_t)item.b * max_blocks + item.page0 + i];
    if (lane == 0) {
      tma_prefetch_desc(&map_v);
      tma_prefetch_desc(&map_r);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (NCTA == 2) cluster_sync();  // peer barriers initialised before any remote access
  pdl_wait();                     // the previous kernel's q / cache writes are visible from here
  pdl_launch_dependents();        // the next kernel may begin its prologue; it still waits for this one
  const uint32_t tmem = *tmem_base_smem;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % S::NSTAGE;
        if (j >= S::NSTAGE && !mbar_wait(&empty[s], ((j / S::NSTAGE) - 1) & 1, abort)) {
          raise_abort(abort, status, kStatusTimeout);
          break;
        }
        mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
        uint8_t* st = smem + S::OFF_STAGE + s * S::STAGE_BYTES;
        const int y = pages[j] * kTok;
#pragma unroll
        for (int c = 0; c < S::NCH; ++c)
          tma_load_2d(st + c * S::CH_BYTES, &map_v, &full[s], (int)(rank * S::VD + 64 * c), y, policy);
        tma_load_2d(st + S::NCH * S::CH_BYTES, &map_r, &full[s], (int)(R + rank * S::PD), y, policy);
        ++issued;
      }
      if (*abort) {
        // drain loads still in flight before shared memory is released
        const int first = issued > S::NSTAGE ? issued - S::NSTAGE : 0;
        for (int j = first; j < issued; ++j) mbar_wait(&full[j % S::NSTAGE], (j / S::NSTAGE) & 1, no_abort);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 64, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, S::VD, 0, 1);
      const uint32_t tS = tmem + S::T_S, tO = tmem + S::T_O, tP = tmem + S::T_P, tQ = tmem + S::T_Q;
      bool ok = mbar_wait(q_ready, 0, abort);
      auto issue_pv = [&](int jj) {
        const uint32_t base = smem_base + S::OFF_STAGE + (jj % S::NSTAGE) * S::STAGE_BYTES;
#pragma unroll
        for (int ks = 0; ks < kTok / 16; ++ks) {
          const uint64_t bdesc = smem_desc(base + ks * 16 * 128, S::CH_BYTES, 1024, kSwizzle128B);
          mma_bf16_ts(tO, tP + ks * 8, bdesc, IDESC_PV, (jj > 0 || ks > 0) ? 1u : 0u);
        }
        tc_commit(pv_done);
        tc_commit(&empty[jj % S::NSTAGE]);
      };
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int s = j % S::NSTAGE;
        if (!mbar_wait(&full[s], (j / S::NSTAGE) & 1, abort)) { ok = false; break; }
        if (j > 0 && !mbar_wait(s_free, (j - 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t base = smem_base + S::OFF_STAGE + s * S::STAGE_BYTES;
#pragma unroll
        for (int ks = 0; ks < S::QD / 16; ++ks) {
          uint64_t bdesc;
          if (ks < S::VD / 16) {
            bdesc = smem_desc(base + (ks >> 2) * S::CH_BYTES + (ks & 3) * 32, 16, 1024, kSwizzle128B);
          } else {
            const int rk = ks - S::VD / 16;
            bdesc = smem_desc(base + S::NCH * S::CH_BYTES + rk * 32, 16, 512, kSwizzle64B);
          }
          mma_bf16_ts(tS, tQ + ks * 8, bdesc, IDESC_QK, ks > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        if (j > 0) {
          if (!mbar_wait(p_full, (j - 1) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          issue_pv(j - 1);
        }
      }
      if (ok && n_tiles > 0) {
        if (mbar_wait(p_full, (n_tiles - 1) & 1, abort)) {
          tc_fence_after();
          issue_pv(n_tiles - 1);
        } else {
          ok = false;
        }
      }
      if (!ok) raise_abort(abort, status, kStatusTimeout);
      // all issued tensor-core work must finish before TMEM is released
      tc_commit(drain);
      mbar_wait(drain, 0, no_abort);
    }
  } else {
    // ---------------------------------------------------- softmax warps 0-7
    // Warp w reads TMEM lane quarter q = w % 4 (rows = heads 32q..32q+31) and
    // owns score columns [32h, 32h + 32) of each tile, h = w / 4.
    const uint32_t q = warp & 3, hf = warp >> 2;
    const int t = (int)(q * 32 + lane);  // head index == TMEM lane
    const uint32_t lane_off = (q * 32) << 16;
    const bool live = t < H;
    // Q slice -> TMEM (K order: latent columns of this CTA, then its rope
    // columns): this thread's 16-column chunks c = hf, hf + 2, ..., every load
    // issued before the first store
    {
      constexpr int NQC = S::QD / 32;        // 16-column chunks (32 bf16)
      constexpr int NMY = (NQC + 1) / 2;     // chunks per thread (at most)
      const uint4* ql = reinterpret_cast<const uint4*>(q_lat + ((int64_t)item.b * H + (live ? t : 0)) * R +
                                                       rank * S::VD);
      const uint4* qr = reinterpret_cast<const uint4*>(q_rope + ((int64_t)item.b * H + (live ? t : 0)) * P +
                                                       rank * S::PD);
      uint4 v[NMY][4];
#pragma unroll
      for (int k = 0; k < NMY; ++k) {
        const int c = 2 * k + (int)hf;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 x = make_uint4(0, 0, 0, 0);
          if (live && c < NQC) x = (c < S::VD / 32) ? ql[c * 4 + i] : qr[(c - S::VD / 32) * 4 + i];
          v[k][i] = x;
        }
      }
#pragma unroll
      for (int k = 0; k < NMY; ++k) {
        const int c = 2 * k + (int)hf;
        if (c < NQC) {
          const uint32_t w[16] = {v[k][0].x, v[k][0].y, v[k][0].z, v[k][0].w, v[k][1].x, v[k][1].y,
                                  v[k][1].z, v[k][1].w, v[k][2].x, v[k][2].y, v[k][2].z, v[k][2].w,
                                  v[k][3].x, v[k][3].y, v[k][3].z, v[k][3].w};
          tmem_st16(tmem + lane_off + S::T_Q + c * 16, w);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(q_ready);
    }

    uint32_t peer_recv = 0, peer_xch_full = 0, peer_peer_free = 0;
    if (NCTA == 2) {
      const uint32_t peer = rank ^ 1u;
      peer_recv = mapa_shared(smem_base + S::OFF_XCH + S::OFF_RECV_REL, peer);
      peer_xch_full = mapa_shared(smem_u32(xch_full), peer);
      peer_peer_free = mapa_shared(smem_u32(peer_free), peer);
    }

    float m_run = -INFINITY, l_half = 0.0f;  // l_half: this thread's 32 columns
    bool ok = true;
    const int tok0 = item.page0 * kTok;
    for (int j = 0; j < n_tiles; ++j) {
      const int buf = j & 1;
      if (NCTA == 2 && threadIdx.x == 0) mbar_arrive_expect_tx(&xch_full[buf], S::XCH_BUF);
      if (!__all_sync(0xffffffffu, mbar_wait(s_full, j & 1, abort))) { ok = false; break; }
      tc_fence_after();
      float s[32];
      {
        uint32_t r0[32];
        tmem_ld32(tmem + lane_off + S::T_S + hf * 32, r0);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = __uint_as_float(r0[i]);
      }
      tc_fence_before();
      warp_arrive(s_free);

      if (NCTA == 2) {
        // Scores are summed over the two CTAs' column slices.  Each partial is
        // scaled into the log2 domain and rounded to fp16 in both CTAs, so the
        // pair computes bit-identical sums.  My partial goes to my send
        // buffer (row t = 128 bytes, 16-byte chunk c at c ^ (t & 7)); once all
        // rows are written, thread 0 copies the tile to the peer's receive
        // buffer in one bulk copy that completes on the peer's xch_full[buf].
        // peer_free[buf] (the peer consumed page j-2) frees both my send
        // buffer (that copy has landed) and the peer's receive buffer.
        uint32_t hv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hv[i] = pack_half2(s[2 * i] * scale_log2, s[2 * i + 1] * scale_log2);
          const float2 f = unpack_half2(hv[i]);
          s[2 * i] = f.x;
          s[2 * i + 1] = f.y;
        }
        if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait<true>(&peer_free[buf], ((j >> 1) - 1) & 1, abort))) {
          ok = false;
          break;
        }
        uint4* srow = reinterpret_cast<uint4*>(smem + S::OFF_XCH + buf * S::XCH_BUF + t * 128);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          srow[((int)hf * 4 + c) ^ (t & 7)] = make_uint4(hv[4 * c], hv[4 * c + 1], hv[4 * c + 2], hv[4 * c + 3]);
        fence_proxy_async_shared();  // read by the bulk copy
        warp_arrive(&send_ready[buf]);
        if (threadIdx.x == 0) {
          if (mbar_wait(&send_ready[buf], (j >> 1) & 1, abort)) {
            bulk_copy_to_peer(peer_recv + buf * S::XCH_BUF, smem_base + S::OFF_XCH + buf * S::XCH_BUF, S::XCH_BUF,
                              peer_xch_full + buf * 8);
          }
        }
        if (!__all_sync(0xffffffffu, mbar_wait<true>(&xch_full[buf], (j >> 1) & 1, abort))) { ok = false; break; }
        const uint4* row =
            reinterpret_cast<const uint4*>(smem + S::OFF_XCH + S::OFF_RECV_REL + buf * S::XCH_BUF + t * 128);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 v = row[((int)hf * 4 + c) ^ (t & 7)];
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_half2(w[k]);
            s[8 * c + 2 * k] += f.x;
            s[8 * c + 2 * k + 1] += f.y;
          }
        }
        __syncwarp();
        if (lane == 0 && j + 2 < n_tiles) mbar_arrive_cluster_relaxed(peer_peer_free + buf * 8);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] *= scale_log2;
      }

      // mask tokens past the item, row max (tree)
      const int tbase = tok0 + j * kTok + (int)hf * 32;
      float mx[16];
#pragma unroll
      for (int i = 0; i < 32; ++i) s[i] = (tbase + i < item.tok_end) ? s[i] : -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i) mx[i] = fmaxf(s[2 * i], s[2 * i + 1]);
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
      float* red_j = red + (j & 1) * 2 * kHeadsPad;
      red_j[hf * kHeadsPad + t] = mx[0];
      warp_arrive(&red_bar[j & 1]);
      if (!__all_sync(0xffffffffu, mbar_wait(&red_bar[j & 1], (j >> 1) & 1, abort))) { ok = false; break; }
      const float mt = fmaxf(mx[0], red_j[(hf ^ 1) * kHeadsPad + t]);
      // lazy rescale: keep the running max until a tile exceeds it by 2^8
      float factor = 1.0f;
      bool rescale = false;
      if (mt > m_run + kLazyRescale) {
        factor = fast_exp2(m_run - mt);
        m_run = mt;
        rescale = (j > 0);
      }
      uint32_t pk[16];
      float ps[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t w = pack_bf16x2(fast_exp2(s[2 * i] - m_run), fast_exp2(s[2 * i + 1] - m_run));
        pk[i] = w;
        ps[i] = bf16lo_to_f32(w) + bf16hi_to_f32(w);
      }
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) ps[i] += ps[i + w];
      l_half = l_half * factor + ps[0];
      if (j > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, abort))) { ok = false; break; }
        tc_fence_after();
      }
      // tcgen05.ld/st are warp-collective: rescale the warp's rows (its half of
      // the O columns) when any head of the warp needs it (factor 1 otherwise)
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = (int)hf * (S::VD / 64); c < ((int)hf + 1) * (S::VD / 64); ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + S::T_O + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(tmem + lane_off + S::T_O + c * 32, o);
        }
      }
      tmem_st16(tmem + lane_off + S::T_P + hf * 16, pk);
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(p_full);
    }
    if (ok && n_tiles > 0 && !__all_sync(0xffffffffu, mbar_wait(pv_done, (n_tiles - 1) & 1, abort))) ok = false;
    if (!ok) {
      raise_abort(abort, status, kStatusTimeout);
    } else {
      // combine the two column halves of the softmax denominator
      float* red_l = red + 2 * 2 * kHeadsPad;  // slot 2
      red_l[hf * kHeadsPad + t] = l_half;
      warp_arrive(fin_bar);
      ok = __all_sync(0xffffffffu, mbar_wait(fin_bar, 0, abort));
    }
    if (!ok) {
      raise_abort(abort, status, kStatusTimeout);
    } else {
      const float l_run = l_half + red[2 * 2 * kHeadsPad + (hf ^ 1) * kHeadsPad + t];
      tc_fence_after();
      const int c0 = (int)hf * (S::VD / 64), c1 = c0 + S::VD / 64;  // this warp's 32-column O chunks
      if (item.partial < 0) {
        const float inv = 1.0f / l_run;
        __nv_bfloat16* dst = out + ((int64_t)item.b * H + (live ? t : 0)) * R + rank * S::VD;
#pragma unroll 1
        for (int c = c0; c < c1; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + S::T_O + c * 32, o);
          tmem_ld_wait();
          uint32_t pkd[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pkd[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
          if (live) {
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pkd[4 * i], pkd[4 * i + 1], pkd[4 * i + 2], pkd[4 * i + 3]);
          }
        }
      } else {
        float* dst = ws_o + ((int64_t)item.partial * kHeadsPad + t) * R + rank * S::VD;
#pragma unroll 1
        for (int c = c0; c < c1; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + S::T_O + c * 32, o);
          tmem_ld_wait();
          float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
          if (live) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              d4[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                  __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
          }
        }
        if (rank == 0 && hf == 0 && live) ws_ml[(int64_t)item.partial * kHeadsPad + t] = make_float2(m_run, l_run);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (NCTA == 2) cluster_sync();  // no CTA leaves while its peer may still address its smem
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::T_COLS);
  }
}

// Merge split-KV partials: out = sum_i 2^(m_i - M) O_i / sum_i 2^(m_i - M) l_i.
template <int R>
__global__ void __launch_bounds__(128) mla_combine_kernel(const MlaCombine* __restrict__ list, int H,
                                                          const float* __restrict__ ws_o,
                                                          const float2* __restrict__ ws_ml,
                                                          __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();  // the next kernel may begin its prologue; it still waits for this one
  const MlaCombine cmb = list[blockIdx.x];
  const int h = blockIdx.y;
  float M = -INFINITY;
  for (int i = 0; i < cmb.n; ++i) M = fmaxf(M, ws_ml[(int64_t)(cmb.first + i) * kHeadsPad + h].x);
  float den = 0.0f;
  constexpr int PER = R / 128;
  float acc[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) acc[k] = 0.0f;
  for (int i = 0; i < cmb.n; ++i) {
    const float2 ml = ws_ml[(int64_t)(cmb.first + i) * kHeadsPad + h];
    const float w = exp2f(ml.x - M);
    den += w * ml.y;
    const float* o = ws_o + ((int64_t)(cmb.first + i) * kHeadsPad + h) * R;
#pragma unroll
    for (int k = 0; k < PER; ++k) acc[k] += w * o[threadIdx.x + 128 * k];
  }
  const float inv = 1.0f / den;
  __nv_bfloat16* dst = out + ((int64_t)cmb.b * H + h) * R;
#pragma unroll
  for (int k = 0; k < PER; ++k) dst[threadIdx.x + 128 * k] = __float2bfloat16_rn(acc[k] * inv);
}

// Split each sequence into page runs so that the clusters of one wave finish
// together.  A handful of candidate run lengths (caps: the longest sequence
// in 1..16 equal runs, and the even spread of all pages over 1..8 waves) are
// scored by a longest-first list schedule over the available cluster slots
// with cost = pages + a fixed per-item overhead (prologue, pipeline fill,
// epilogue: 2 pages) + for an item of a split sequence the merge: its fp32
// partial [H, R] written and read back, in pages of the same bytes, plus one
// page for the merge launch; the cheapest cap wins.
void plan_items(const int32_t* seq_lens, int B, int slots, int H, int R, int P, std::vector<MlaItem>* items,
                std::vector<MlaCombine>* combines, int* n_partial) {
  std::vector<int> pages(B);
  int64_t total = 0;
  int maxp = 1;
  for (int b = 0; b < B; ++b) {
    pages[b] = (seq_lens[b] + kTok - 1) / kTok;
    total += pages[b];
    maxp = std::max(maxp, pages[b]);
  }
  const double overhead = 2.0;  // pages-equivalent cost of an item's setup
  const double split_cost = 1.0 + (double)H * R * 4 * 2 / ((double)kTok * (R + P) * 2);
  std::vector<int> caps;
  caps.push_back(std::min(maxp, kMaxItemPages));
  for (int n = 2; n <= 16; ++n) caps.push_back(std::max(2, std::min((maxp + n - 1) / n, kMaxItemPages)));
  for (int k = 1; k <= 8; ++k) {
    const int64_t c = (total + (int64_t)k * slots - 1) / ((int64_t)k * slots);
    caps.push_back((int)std::max<int64_t>(2, std::min<int64_t>(c, kMaxItemPages)));
  }
  std::sort(caps.begin(), caps.end());
  caps.erase(std::unique(caps.begin(), caps.end()), caps.end());
  int best_cap = caps.back();
  double best_cost = 1e300;
  std::vector<double> costs;
  for (int cap : caps) {
    costs.clear();
    for (int b = 0; b < B; ++b) {
      const int n = (pages[b] + cap - 1) / cap;
      for (int i = 0; i < n; ++i) {
        const int np = (int)((int64_t)(i + 1) * pages[b] / n - (int64_t)i * pages[b] / n);
        costs.push_back(np + overhead + (n > 1 ? split_cost : 0.0));
      }
    }
    std::sort(costs.begin(), costs.end(), std::greater<double>());
    std::priority_queue<double, std::vector<double>, std::greater<double>> q;
    for (int i = 0; i < slots; ++i) q.push(0.0);
    double makespan = 0.0;
    for (double c : costs) {
      const double t0 = q.top();
      q.pop();
      q.push(t0 + c);
      makespan = std::max(makespan, t0 + c);
    }
    if (makespan < best_cost - 1e-9) {
      best_cost = makespan;
      best_cap = cap;
    }
  }
  items->clear();
  combines->clear();
  int slot = 0;
  for (int b = 0; b < B; ++b) {
    const int n = (pages[b] + best_cap - 1) / best_cap;
    if (n > 1) combines->push_back(MlaCombine{b, slot, n});
    for (int i = 0; i < n; ++i) {
      const int p0 = (int)((int64_t)i * pages[b] / n), p1 = (int)((int64_t)(i + 1) * pages[b] / n);
      const int end = std::min(seq_lens[b], p1 * kTok);
      items->push_back(MlaItem{b, p0, p1 - p0, end, n > 1 ? slot++ : -1});
    }
  }
  // longest items first so the block scheduler back-fills with short ones
  std::stable_sort(items->begin(), items->end(),
                   [](const MlaItem& a, const MlaItem& b) { return a.npages > b.npages; });
  *n_partial = slot;
}

template <int R, int P, int NCTA>
int launch_mla(dsb_ctx* ctx, const dsb_mla_plan* plan, const void* q_lat, const void* q_rope, const void* kv_cache,
               int64_t n_blocks, const int32_t* block_table, int max_blocks, float scale, void* out) {
  using S = MlaShape<R, P, NCTA>;
  auto align = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t off_ml = align((size_t)plan->n_partial * kHeadsPad * R * sizeof(float));
  const size_t need = align(off_ml + (size_t)plan->n_partial * kHeadsPad * sizeof(float2));
  int rc = ensure_workspace(ctx, need);
  if (rc != DSB_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(ctx->ws);

  CUtensorMap map_v, map_r;
  const uint64_t rows = (uint64_t)n_blocks * kTok;
  rc = make_tmap_2d(ctx, &map_v, kv_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, R + P, rows, (R + P) * 2, 64, kTok,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != DSB_OK) return rc;
  rc = make_tmap_2d(ctx, &map_r, kv_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, R + P, rows, (R + P) * 2, S::PD, kTok,
                    CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc != DSB_OK) return rc;

  auto kern = mla_decode_kernel<R, P, NCTA>;
  static std::atomic<bool> attr_set[kMaxDevices];  // per template instance
  if (int rc = smem_attr_once(ctx, kern, S::SMEM_BYTES, attr_set); rc != DSB_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(plan->n_items * NCTA));
  cfg.blockDim = dim3(kMlaThreads);
  cfg.dynamicSmemBytes = S::SMEM_BYTES;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = NCTA;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // prologue overlaps the previous kernel
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const float scale_log2 = scale * 1.4426950408889634f;
  DSB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, map_v, map_r, static_cast<const __nv_bfloat16*>(q_lat),
                                       static_cast<const __nv_bfloat16*>(q_rope), block_table, max_blocks,
                                       static_cast<const MlaItem*>(plan->d_items), plan->H, scale_log2,
                                       static_cast<__nv_bfloat16*>(out), reinterpret_cast<float*>(ws),
                                       reinterpret_cast<float2*>(ws + off_ml), ctx->d_status));
  ctx->stats.kernel_launches++;
  if (plan->n_combines > 0) {
    launch_pdl(mla_combine_kernel<R>, dim3((unsigned)plan->n_combines, (unsigned)plan->H), 128, 0, ctx->stream, 
        static_cast<const MlaCombine*>(plan->d_combines), plan->H, reinterpret_cast<const float*>(ws),
        reinterpret_cast<const float2*>(ws + off_ml), static_cast<__nv_bfloat16*>(out));
    DSB_CUDA_TRY(ctx, cudaGetLastError());
    ctx->stats.kernel_launches++;
  }
  ctx->stats.mla_calls++;
  ctx->stats.mla_work_items += (uint64_t)plan->n_items;
  ctx->stats.mla_partials += (uint64_t)plan->n_partial;
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

static int mla_plan_create_impl(dsb_ctx* ctx, const int32_t* seq_lens, int B, int H, int R, int P,
                                   int block_size, dsb_mla_plan** out) {
  using namespace dsb;
  if (ctx == nullptr || out == nullptr) return DSB_EINVAL;
  *out = nullptr;
  if (seq_lens == nullptr || B <= 0 || H <= 0 || H > kHeadsPad)
    return fail(ctx, DSB_EINVAL, "dsb_mla_plan_create: bad sizes B=%d H=%d", B, H);
  if (block_size != kTok) return fail(ctx, DSB_EUNSUPPORTED, "dsb_mla_plan_create: block_size must be 64");
  if (!((R == 512 && P == 64) || (R == 128 && P == 32)))
    return fail(ctx, DSB_EUNSUPPORTED, "dsb_mla_plan_create: (R, P) = (%d, %d) not supported", R, P);
  int max_len = 0;
  for (int b = 0; b < B; ++b) {
    if (seq_lens[b] < 1) return fail(ctx, DSB_EINVAL, "dsb_mla_plan_create: seq_lens[%d]=%d < 1", b, seq_lens[b]);
    max_len = std::max(max_len, seq_lens[b]);
  }
  const int nct = (R == 512) ? 2 : 1;
  std::vector<MlaItem> items;
  std::vector<MlaCombine> combines;
  int n_partial = 0;
  plan_items(seq_lens, B, std::max(1, ctx->sm_count / nct), H, R, P, &items, &combines, &n_partial);
  auto* plan = new dsb_mla_plan();
  plan->B = B;
  plan->H = H;
  plan->R = R;
  plan->P = P;
  plan->n_items = (int)items.size();
  plan->n_combines = (int)combines.size();
  plan->n_partial = n_partial;
  plan->max_len = max_len;
  plan->device = ctx->device;
  cudaError_t e = cudaMalloc(&plan->d_items, items.size() * sizeof(MlaItem) + 256 +
                                                 std::max<size_t>(1, combines.size()) * sizeof(MlaCombine));
  if (e != cudaSuccess) {
    delete plan;
    return fail(ctx, DSB_ENOMEM, "dsb_mla_plan_create: %s", cudaGetErrorString(e));
  }
  plan->d_combines = static_cast<uint8_t*>(plan->d_items) + ((items.size() * sizeof(MlaItem) + 255) & ~size_t(255));
  e = cudaMemcpyAsync(plan->d_items, items.data(), items.size() * sizeof(MlaItem), cudaMemcpyHostToDevice,
                      ctx->stream);
  if (e == cudaSuccess && !combines.empty())
    e = cudaMemcpyAsync(plan->d_combines, combines.data(), combines.size() * sizeof(MlaCombine),
                        cudaMemcpyHostToDevice, ctx->stream);
  // pageable-source async copies are staged before they return, so the host
  // vectors may die here; the stream orders the copies before any kernel
  if (e != cudaSuccess) {
    cudaFree(plan->d_items);
    delete plan;
    return fail(ctx, DSB_ECUDA, "dsb_mla_plan_create: %s", cudaGetErrorString(e));
  }
  *out = plan;
  return DSB_OK;
}

extern "C" int dsb_mla_plan_destroy(dsb_mla_plan* plan) {
  if (plan == nullptr) return DSB_OK;
  cudaSetDevice(plan->device);
  cudaFree(plan->d_items);
  delete plan;
  return DSB_OK;
}

extern "C" int dsb_mla_plan_info(const dsb_mla_plan* plan, int* n_items, int* n_partial) {
  if (plan == nullptr) return DSB_EINVAL;
  if (n_items) *n_items = plan->n_items;
  if (n_partial) *n_partial = plan->n_partial;
  return DSB_OK;
}

extern "C" int dsb_mla_decode_planned(dsb_ctx* ctx, const dsb_mla_plan* plan, const void* q_lat, const void* q_rope,
                                      const void* kv_cache, int64_t n_blocks, const int32_t* block_table,
                                      int max_blocks, float softmax_scale, void* out_lat) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (plan == nullptr || q_lat == nullptr || q_rope == nullptr || kv_cache == nullptr || block_table == nullptr ||
      out_lat == nullptr)
    return fail(ctx, DSB_EINVAL, "dsb_mla_decode: null pointer argument");
  if (n_blocks <= 0 || max_blocks <= 0 || (int64_t)max_blocks * kTok < plan->max_len)
    return fail(ctx, DSB_EINVAL, "dsb_mla_decode: n_blocks=%lld, max_blocks=%d cannot hold length %d",
                (long long)n_blocks, max_blocks, plan->max_len);
  if ((reinterpret_cast<uintptr_t>(q_lat) | reinterpret_cast<uintptr_t>(q_rope) |
       reinterpret_cast<uintptr_t>(out_lat) | reinterpret_cast<uintptr_t>(kv_cache)) & 15u)
    return fail(ctx, DSB_EINVAL, "dsb_mla_decode: pointers must be 16-byte aligned");
  if (plan->device != ctx->device)
    return fail(ctx, DSB_EINVAL, "dsb_mla_decode: plan made on device %d, context on device %d", plan->device,
                ctx->device);
  if (plan->R == 512)
    return launch_mla<512, 64, 2>(ctx, plan, q_lat, q_rope, kv_cache, n_blocks, block_table, max_blocks,
                                  softmax_scale, out_lat);
  return launch_mla<128, 32, 1>(ctx, plan, q_lat, q_rope, kv_cache, n_blocks, block_table, max_blocks, softmax_scale,
                                out_lat);
}

namespace dsb {

// Plan the split-KV work for these lengths into the context's reusable plan
// buffer (stream order protects its reuse); `plan` then refers to it.
int mla_plan_into_aux(dsb_ctx* ctx, const int32_t* seq_lens, int B, int H, int R, int P, dsb_mla_plan* plan) {
  int max_len = 0;
  for (int b = 0; b < B; ++b) max_len = std::max(max_len, seq_lens[b]);
  std::vector<MlaItem> items;
  std::vector<MlaCombine> combines;
  int n_partial = 0;
  plan_items(seq_lens, B, std::max(1, ctx->sm_count / (R == 512 ? 2 : 1)), H, R, P, &items, &combines, &n_partial);
  const size_t off_comb = (items.size() * sizeof(MlaItem) + 255) & ~size_t(255);
  int rc = ensure_aux(ctx, off_comb + std::max<size_t>(1, combines.size()) * sizeof(MlaCombine));
  if (rc != DSB_OK) return rc;
  DSB_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->aux, items.data(), items.size() * sizeof(MlaItem), cudaMemcpyHostToDevice,
                                    ctx->stream));
  if (!combines.empty())
    DSB_CUDA_TRY(ctx, cudaMemcpyAsync(static_cast<uint8_t*>(ctx->aux) + off_comb, combines.data(),
                                      combines.size() * sizeof(MlaCombine), cudaMemcpyHostToDevice, ctx->stream));
  plan->B = B;
  plan->H = H;
  plan->R = R;
  plan->P = P;
  plan->n_items = (int)items.size();
  plan->n_combines = (int)combines.size();
  plan->n_partial = n_partial;
  plan->max_len = max_len;
  plan->d_items = ctx->aux;
  plan->d_combines = static_cast<uint8_t*>(ctx->aux) + off_comb;
  plan->device = ctx->device;
  return DSB_OK;
}

}  // namespace dsb

static int mla_decode_impl(dsb_ctx* ctx, const void* q_lat, const void* q_rope, const void* kv_cache,
                              int64_t n_blocks, int block_size, const int32_t* block_table, int max_blocks,
                              const int32_t* seq_lens, int B, int H, int R, int P, float softmax_scale,
                              void* out_lat) {
  using namespace dsb;
  if (ctx == nullptr) return DSB_EINVAL;
  if (seq_lens == nullptr || B <= 0 || H <= 0 || H > kHeadsPad)
    return fail(ctx, DSB_EINVAL, "dsb_mla_decode: bad sizes B=%d H=%d", B, H);
  if (block_size != kTok) return fail(ctx, DSB_EUNSUPPORTED, "dsb_mla_decode: block_size must be 64");
  if (!((R == 512 && P == 64) || (R == 128 && P == 32)))
    return fail(ctx, DSB_EUNSUPPORTED, "dsb_mla_decode: (R, P) = (%d, %d) not supported", R, P);
  for (int b = 0; b < B; ++b) {
    if (seq_lens[b] < 1 || seq_lens[b] > (int64_t)max_blocks * kTok)
      return fail(ctx, DSB_EINVAL, "dsb_mla_decode: seq_lens[%d]=%d outside [1, max_blocks*64]", b, seq_lens[b]);
  }
  dsb_mla_plan plan;
  int rc = mla_plan_into_aux(ctx, seq_lens, B, H, R, P, &plan);
  if (rc != DSB_OK) return rc;
  return dsb_mla_decode_planned(ctx, &plan, q_lat, q_rope, kv_cache, n_blocks, block_table, max_blocks, softmax_scale,
                                out_lat);
}

// ===================================================== allocation-free variant
//
// dsb_mla_decode_noalloc serves callers that cannot allocate device memory on
// the call path: allocators and runtimes that own every byte of device memory
// themselves and forbid stray cudaMalloc/cudaFree (a cudaFree also
// synchronises the whole device), and plug-in hosts that hand this library
// only a stream and their own buffers.  Its scratch - the work list, the
// split-KV partials and the bounded-wait status word - lives in the fixed
// array below, which every GPU that loads the library holds until the process
// exits.  dsb_mla_noalloc_status reads the status word back.

namespace dsb {
namespace {

constexpr int kNoAllocMaxItems = 4096;     // work items per call
constexpr int kNoAllocMaxPartials = 24;    // split-KV partials per call
constexpr size_t kNoAllocOffItems = 256;   // [0, 256): status word
constexpr size_t kNoAllocOffComb = kNoAllocOffItems + kNoAllocMaxItems * sizeof(MlaItem);
constexpr size_t kNoAllocOffO = (kNoAllocOffComb + kNoAllocMaxItems * sizeof(MlaCombine) + 255) & ~size_t(255);
constexpr size_t kNoAllocPartialO = (size_t)kHeadsPad * 512 * sizeof(float);  // one partial at R = 512
constexpr size_t kNoAllocOffML = kNoAllocOffO + kNoAllocMaxPartials * kNoAllocPartialO;
constexpr size_t kNoAllocScratchBytes =
    (kNoAllocOffML + kNoAllocMaxPartials * kHeadsPad * sizeof(float2) + 255) & ~size_t(255);  // ~6.4 MB

static __device__ __align__(256) uint8_t g_mla_noalloc_scratch[kNoAllocScratchBytes];

// Per-device set-up, done by the first call on each device (which should come
// before any stream capture on that device): the device address of the
// scratch array (its name in host code is only a host-side stand-in), the SM
// count for planning, and the kernels' shared-memory opt-in.
struct NoAllocDevice {
  bool ready = false;
  uint8_t* scratch = nullptr;
  int sm_count = 0;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

int noalloc_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_mla_noalloc_scratch) != cudaSuccess || p == nullptr) return DSB_ECUDA;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return DSB_ECUDA;
    if (cudaFuncSetAttribute(mla_decode_kernel<512, 64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             MlaShape<512, 64, 2>::SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(mla_decode_kernel<128, 32, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             MlaShape<128, 32, 1>::SMEM_BYTES) != cudaSuccess)
      return DSB_ECUDA;
    d.scratch = static_cast<uint8_t*>(p);
    d.ready = true;
  }
  *out = &d;
  return DSB_OK;
}

template <int R, int P, int NCTA>
int noalloc_launch(cudaStream_t stream, uint8_t* scratch, const std::vector<MlaItem>& items,
                   const std::vector<MlaCombine>& combines, const void* q_lat, const void* q_rope,
                   const void* kv_cache, int64_t n_blocks, const int32_t* block_table, int max_blocks, int H,
                   float scale, void* out) {
  using S = MlaShape<R, P, NCTA>;
  // the status word must start at zero; the work list overwrites the last call's
  if (cudaMemsetAsync(scratch, 0, sizeof(int), stream) != cudaSuccess) return DSB_ECUDA;
  if (cudaMemcpyAsync(scratch + kNoAllocOffItems, items.data(), items.size() * sizeof(MlaItem),
                      cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return DSB_ECUDA;
  if (!combines.empty() && cudaMemcpyAsync(scratch + kNoAllocOffComb, combines.data(),
                                           combines.size() * sizeof(MlaCombine), cudaMemcpyHostToDevice,
                                           stream) != cudaSuccess)
    return DSB_ECUDA;
  CUtensorMap map_v, map_r;
  const uint64_t rows = (uint64_t)n_blocks * kTok;
  if (make_tmap_2d(nullptr, &map_v, kv_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, R + P, rows, (R + P) * 2, 64, kTok,
                   CU_TENSOR_MAP_SWIZZLE_128B) != DSB_OK ||
      make_tmap_2d(nullptr, &map_r, kv_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, R + P, rows, (R + P) * 2, S::PD,
                   kTok, CU_TENSOR_MAP_SWIZZLE_64B) != DSB_OK)
    return DSB_EINVAL;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items.size() * NCTA));
  cfg.blockDim = dim3(kMlaThreads);
  cfg.dynamicSmemBytes = S::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = NCTA;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  float* ws_o = reinterpret_cast<float*>(scratch + kNoAllocOffO);
  float2* ws_ml = reinterpret_cast<float2*>(scratch + kNoAllocOffML);
  if (cudaLaunchKernelEx(&cfg, mla_decode_kernel<R, P, NCTA>, map_v, map_r,
                         static_cast<const __nv_bfloat16*>(q_lat), static_cast<const __nv_bfloat16*>(q_rope),
                         block_table, max_blocks, reinterpret_cast<const MlaItem*>(scratch + kNoAllocOffItems), H,
                         scale * 1.4426950408889634f, static_cast<__nv_bfloat16*>(out), ws_o, ws_ml,
                         reinterpret_cast<int*>(scratch)) != cudaSuccess)
    return DSB_ECUDA;
  if (!combines.empty()) {
    launch_pdl(mla_combine_kernel<R>, dim3((unsigned)combines.size(), (unsigned)H), 128, 0, stream, 
        reinterpret_cast<const MlaCombine*>(scratch + kNoAllocOffComb), H, ws_o, ws_ml,
        static_cast<__nv_bfloat16*>(out));
    if (cudaGetLastError() != cudaSuccess) return DSB_ECUDA;
  }
  return DSB_OK;
}

}  // namespace
}  // namespace dsb

static int mla_decode_noalloc_impl(void* stream, const void* q_lat, const void* q_rope, const void* kv_cache,
                                      int64_t n_blocks, int block_size, const int32_t* block_table, int max_blocks,
                                      const int32_t* seq_lens, int B, int H, int R, int P, float softmax_scale,
                                      void* out_lat) {
  using namespace dsb;
  if (q_lat == nullptr || q_rope == nullptr || kv_cache == nullptr || block_table == nullptr || seq_lens == nullptr ||
      out_lat == nullptr || B <= 0 || H <= 0 || H > kHeadsPad || n_blocks <= 0 || max_blocks <= 0)
    return DSB_EINVAL;
  if (block_size != kTok || !((R == 512 && P == 64) || (R == 128 && P == 32))) return DSB_EUNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(q_lat) | reinterpret_cast<uintptr_t>(q_rope) |
       reinterpret_cast<uintptr_t>(out_lat) | reinterpret_cast<uintptr_t>(kv_cache)) & 15u)
    return DSB_EINVAL;
  for (int b = 0; b < B; ++b)
    if (seq_lens[b] < 1 || seq_lens[b] > (int64_t)max_blocks * kTok) return DSB_EINVAL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return DSB_ECUDA;
  NoAllocDevice* d = nullptr;
  int rc = noalloc_setup(dev, &d);
  if (rc != DSB_OK) return rc;
  const int slots = std::max(1, d->sm_count / (R == 512 ? 2 : 1));
  std::vector<MlaItem> items;
  std::vector<MlaCombine> combines;
  int n_partial = 0;
  plan_items(seq_lens, B, slots, H, R, P, &items, &combines, &n_partial);
  if (n_partial > kNoAllocMaxPartials) {
    // too many splits for the fixed scratch: one item per sequence where the
    // 16384-token item limit allows
    std::vector<int32_t> one(1);
    items.clear();
    combines.clear();
    n_partial = 0;
    for (int b = 0; b < B; ++b) {
      std::vector<MlaItem> it;
      std::vector<MlaCombine> cb;
      int np = 0;
      one[0] = seq_lens[b];
      plan_items(one.data(), 1, 1, H, R, P, &it, &cb, &np);  // a single slot never splits below the item limit
      for (auto& x : it) {
        x.b = b;
        if (x.partial >= 0) x.partial += n_partial;
        items.push_back(x);
      }
      for (auto& c : cb) combines.push_back(MlaCombine{b, c.first + n_partial, c.n});
      n_partial += np;
    }
  }
  if ((int)items.size() > kNoAllocMaxItems || n_partial > kNoAllocMaxPartials) return DSB_ELIMIT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (R == 512)
    return noalloc_launch<512, 64, 2>(s, d->scratch, items, combines, q_lat, q_rope, kv_cache, n_blocks, block_table,
                                      max_blocks, H, softmax_scale, out_lat);
  return noalloc_launch<128, 32, 1>(s, d->scratch, items, combines, q_lat, q_rope, kv_cache, n_blocks, block_table,
                                    max_blocks, H, softmax_scale, out_lat);
}

// The C entry points: no C++ exception (a host allocation of the work list)
// crosses the ABI.
extern "C" int dsb_mla_plan_create(dsb_ctx* ctx, const int32_t* seq_lens, int B, int H, int R, int P,
                                   int block_size, dsb_mla_plan** out) {
  return dsb::guarded(ctx, "dsb_mla_plan_create",
                      [&] { return mla_plan_create_impl(ctx, seq_lens, B, H, R, P, block_size, out); });
}

extern "C" int dsb_mla_decode(dsb_ctx* ctx, const void* q_lat, const void* q_rope, const void* kv_cache,
                              int64_t n_blocks, int block_size, const int32_t* block_table, int max_blocks,
                              const int32_t* seq_lens, int B, int H, int R, int P, float softmax_scale,
                              void* out_lat) {
  return dsb::guarded(ctx, "dsb_mla_decode", [&] {
    return mla_decode_impl(ctx, q_lat, q_rope, kv_cache, n_blocks, block_size, block_table, max_blocks, seq_lens, B,
                           H, R, P, softmax_scale, out_lat);
  });
}

// Status of the last dsb_mla_decode_noalloc call enqueued on this device:
// waits for `stream`, then reads the status word of the fixed scratch (a
// device-to-host copy of one int into the caller's stack, no allocation).
static int mla_noalloc_status_impl(void* stream) {
  using namespace dsb;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return DSB_ECUDA;
  NoAllocDevice* d = nullptr;
  int rc = noalloc_setup(dev, &d);
  if (rc != DSB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = 0;
  if (cudaMemcpyAsync(&st, d->scratch, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return DSB_ECUDA;
  if (st == kStatusOk) return DSB_OK;
  return st == kStatusBadInput ? DSB_EINVAL : DSB_ETIMEOUT;
}

extern "C" int dsb_mla_noalloc_status(void* stream) {
  return dsb::guarded(nullptr, "dsb_mla_noalloc_status", [&] { return mla_noalloc_status_impl(stream); });
}

extern "C" int dsb_mla_decode_noalloc(void* stream, const void* q_lat, const void* q_rope, const void* kv_cache,
                                      int64_t n_blocks, int block_size, const int32_t* block_table, int max_blocks,
                                      const int32_t* seq_lens, int B, int H, int R, int P, float softmax_scale,
                                      void* out_lat) {
  return dsb::guarded(nullptr, "dsb_mla_decode_noalloc", [&] {
    return mla_decode_noalloc_impl(stream, q_lat, q_rope, kv_cache, n_blocks, block_size, block_table, max_blocks,
                                   seq_lens, B, H, R, P, softmax_scale, out_lat);
  });
}
