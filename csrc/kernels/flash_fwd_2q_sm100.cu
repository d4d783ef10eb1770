// flash_fwd_2q_sm100.cu - bf16 flash-attention forward with two query tiles
// per CTA (256 query rows), for B200 (sm_100a).  Like the one-tile kernel it
// stands in for the reference's row-per-CTA partial attention kernel
// (src/attention/ring_attention_nccl_gpu_bench.cu:46-111) and its merge (:113-134).
//
// With one query tile the chain S_j -> softmax_j -> PV_j is serial: the exp
// work of a 128x128 tile (MUFU-bound, about as long as its two GEMMs) can hide
// behind little tensor work, and the tensor pipe idles half the time.  Here
// the tensor core alternates between two independent tiles A and B,
//     QK_A(j), PV_B(j-1), QK_B(j), PV_A(j), QK_A(j+1), ...
// so each tile's softmax runs while the other tile's GEMMs execute.  Causal
// launches hand P over in two 64-key halves, so PV starts half a softmax
// earlier.
//
// CTA = 12 warps, persistent over work items (head, 256-row query unit, KV chunk):
//   warp 0      TMA producer: Q_A / Q_B once per item, K / V tiles per step
//   warp 1      MMA issuer (one thread) and TMEM owner
//   warps 2-3   ring copy warps (fused mode), shared with the one-tile kernel
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B: one thread per
//               query row, the full 128-column S row in registers (one pass)
// Registers: warpgroup 0 (warps 0-3) gives up registers after start-up
// (setmaxnreg.dec to kRegsLow) and the two softmax warpgroups take them
// (setmaxnreg.inc to kRegsHigh); 128 * kRegsLow + 256 * kRegsHigh stays within
// the 168 * 384 registers the block is launched with.
// TMEM: S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [384,384+D); P is
// written back over S as packed bf16 (A operand of the PV MMA).
// Every wait is bounded; no TMA load uses cluster broadcast.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "flash.h"
#include "flash_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace rab {

using namespace sm100;
using namespace flash_detail;

namespace {

constexpr int kThreads2 = 384;
constexpr int kWTma = 0;
constexpr int kWMma = 1;
constexpr int kWComm = 2;
constexpr int kWSoft = 4;  // warps 4..7 tile A, 8..11 tile B
constexpr uint32_t kCols = 512;
constexpr uint32_t kRegsLaunch = 168;  // 65536 / 384, rounded down to a multiple of 8
constexpr uint32_t kRegsLow = 72;      // warpgroup 0: TMA, MMA, ring copy
constexpr uint32_t kRegsHigh = 216;    // softmax warpgroups
static_assert(128 * kRegsLow + 256 * kRegsHigh <= kRegsLaunch * 384,
              "register split exceeds the launch allocation");

// Causal launches: the MMA thread, which walks the visible KV tiles, hands the
// softmax warps each tile's first global key position through a ring of
// kKloSlots shared words (one mbarrier each; kKloEnd closes a work item), so
// the softmax, at its register cap, carries no walk state of its own.  The
// MMA thread is at most three entries ahead of either softmax warpgroup (it
// waits for their P of the previous tiles), so the ring never laps a reader.
constexpr int kKloSlots = 8;
constexpr int kKloEnd = -2147483647 - 1;

template <int D>
struct Cfg2 {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static constexpr int kN = 128;
  static constexpr int kQTile = kM * D * 2;
  static constexpr int kKTile = kN * D * 2;
  static constexpr int kVTile = kKTile;
  static constexpr int kStages = D == 64 ? 4 : 2;
  static constexpr int kSmemTiles = 2 * kQTile + kStages * (kKTile + kVTile);
  static constexpr int kNumBars = 4 * kStages + 10 + 2 * kItemSlots + kKloSlots + 2;
  static constexpr int kSmemBytes = kSmemTiles + 1024 + kNumBars * 8 + 64;
  static constexpr int kKSteps = D / 16;   // QK: K = head dim, 16 bf16 per MMA
  static constexpr int kPSteps = kN / 16;  // PV: K = keys
  static constexpr uint32_t kIdescQK = make_idesc(kFmtBF16, kFmtBF16, kM, kN, kMajorK, kMajorK);
  static constexpr uint32_t kIdescPV = make_idesc(kFmtBF16, kFmtBF16, kM, D, kMajorK, kMajorMN);
};

__device__ __forceinline__ uint32_t col_s(int x) { return x ? 128u : 0u; }
__device__ __forceinline__ uint32_t col_o(int x) { return x ? 384u : 256u; }

// Last global query position of the 256-row unit at local row q0: a KV tile is
// processed when either query tile sees it, i.e. when the later tile's last
// row does (positions grow along each chunk of the rank's rows, and the second
// zigzag chunk lies after the first).
__device__ __forceinline__ int unit_q_hi(const FlashParams& p, int q0) {
  return global_pos(q0 + kM, p.rank, p.Sq, p.world, p.zigzag) + kM - 1;
}

// kCausal: tiles are classified against the causal mask; a non-causal
// instantiation treats every tile as full.  kPParts = 2: the softmax hands P
// over in two halves of 64 keys (p_full, then p_hi), so the PV MMAs of the
// first half start while the second half's exponentials are computed.
template <int D, bool kCausal, int kPParts>
__global__ void __launch_bounds__(kThreads2, 1)
    flash_fwd_2q_kernel(const __grid_constant__ FlashParams p,
                        const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV) {
  using C = Cfg2<D>;
  constexpr int NS = C::kStages;
  constexpr int kN = C::kN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // [2][kQTile]
  uint8_t* sK = smem + 2 * C::kQTile;        // [NS][kKTile]
  uint8_t* sV = sK + NS * C::kKTile;         // [NS][kVTile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kSmemTiles);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + NS;
  uint64_t* v_full = bars + 2 * NS;
  uint64_t* v_empty = bars + 3 * NS;
  uint64_t* q_full = bars + 4 * NS;
  uint64_t* q_empty = bars + 4 * NS + 1;
  uint64_t* s_full = bars + 4 * NS + 2;   // [2]
  uint64_t* p_full = bars + 4 * NS + 4;   // [2]
  uint64_t* pv_done = bars + 4 * NS + 6;  // [2]
  uint64_t* o_final = bars + 4 * NS + 8;
  uint64_t* drain = bars + 4 * NS + 9;
  uint64_t* item_full = bars + 4 * NS + 10;                 // [kItemSlots] work-item queue
  uint64_t* item_empty = bars + 4 * NS + 10 + kItemSlots;  // [kItemSlots]
  uint64_t* klo_full = bars + 4 * NS + 10 + 2 * kItemSlots;  // [kKloSlots] (causal)
  uint64_t* p_hi = klo_full + kKloSlots;                      // [2] (kPParts == 2)
  __shared__ uint32_t tmem_slot;
  __shared__ int s_copy_ok;
  __shared__ Item s_items[kItemSlots];  // causal: TMA thread -> MMA and softmax roles
  __shared__ int s_klo[kKloSlots];      // causal: MMA thread -> softmax, per visible tile

  const uint32_t warp = warp_id();
  DeviceStatus* st = p.status;
  const uint64_t tmo = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);  // one arrival per softmax warp
      mbar_init(&p_hi[x], 4);
      mbar_init(&pv_done[x], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 1 + 8);  // the MMA thread + one lane per softmax warp
    }
    for (int i = 0; i < kKloSlots; ++i) {
      mbar_init(&klo_full[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == kWMma) {
    tmem_alloc(&tmem_slot, kCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int tpb = p.Skv / kN;
  const int tiles_total = p.nblk * tpb;
  if (warp < 4) {
  // warpgroup 0 gives up registers first thing, unconditionally: the softmax
  // warpgroups' increase below is served by this decrease
  warpgroup_reg_dec<kRegsLow>();
  if (warp == kWTma) {
    // ------------------------------------------------------------------ TMA
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      trace_stamp(p, 0, 0, globaltimer_ns());
      int g = 0, item_count = 0, ready_blocks = 1;
      bool ok = true;
      for (int w = 0; ok; ++w, ++item_count) {
        Item it;
        if constexpr (kCausal) {
          // take item w (claimed when p.dynamic) and publish it, or the end
          // marker, to the MMA and softmax roles
          const int slot = w % kItemSlots;
          if (w >= kItemSlots) {
            ok = mbar_wait(&item_empty[slot], ((w / kItemSlots) - 1) & 1, st, kSiteItemQueue, tmo);
            if (!ok) break;
          }
          bool have;
          if (p.dynamic) {
            have = claim_item(p, tiles_total, &it);
          } else {
            const int item = blockIdx.x + w * gridDim.x;
            have = item < p.n_items;
            if (have) it = make_item(p, item, tiles_total);
          }
          if (!have) it.unit = -1;
          s_items[slot] = it;
          mbar_arrive(&item_full[slot]);
          if (!have) break;
        } else {
          const int item = blockIdx.x + w * gridDim.x;
          if (item >= p.n_items) break;
          it = make_item(p, item, tiles_total);
        }
        ok = mbar_wait(q_empty, (item_count & 1) ^ 1, st, kSiteQFull, tmo);
        if (!ok) break;
        mbar_arrive_expect_tx(q_full, 2 * C::kQTile);
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int ds = 0; ds < D / 64; ++ds)
            tma_load_3d(sQ + x * C::kQTile + ds * (kM * 128), &tmQ, q_full, ds * 64, it.h,
                        it.q0 + x * kM);
        TileWalk<kN> wk;
        int v = it.v_begin;
        bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, unit_q_hi(p, it.q0))
                            : v < it.v_end;
        for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
          if constexpr (kCausal) v = wk.v;
          const int s = v / tpb, t = v - s * tpb;
          if (p.fused && s >= ready_blocks) {
            ok = wait_block(p, s);
            if (!ok) break;
            fence_proxy_async_global();
            ready_blocks = s + 1;
          }
          const int stage = g % NS;
          const uint32_t ph = (g / NS) & 1;
          ok = mbar_wait(&k_empty[stage], ph ^ 1, st, kSiteKEmpty, tmo);
          if (!ok) break;
          mbar_arrive_expect_tx(&k_full[stage], C::kKTile);
#pragma unroll
          for (int ds = 0; ds < D / 64; ++ds)
            tma_load_4d(sK + stage * C::kKTile + ds * (kN * 128), &tmK, &k_full[stage], ds * 64,
                        it.hk, t * kN, s);
          ok = mbar_wait(&v_empty[stage], ph ^ 1, st, kSiteVEmpty, tmo);
          if (!ok) break;
          mbar_arrive_expect_tx(&v_full[stage], C::kVTile);
#pragma unroll
          for (int ds = 0; ds < D / 64; ++ds)
            tma_load_4d(sV + stage * C::kVTile + ds * (kN * 128), &tmV, &v_full[stage], ds * 64,
                        it.hk, t * kN, s);
          ++g;
        }
      }
      trace_stamp(p, 0, 1, globaltimer_ns());
      if (!ok) {
        for (int i = 0; i < NS && i < g; ++i) {
          const int gg = g - 1 - i;
          mbar_wait(&k_full[gg % NS], (gg / NS) & 1, nullptr, kSiteKFull, 100000000ull);
          mbar_wait(&v_full[gg % NS], (gg / NS) & 1, nullptr, kSiteVFull, 100000000ull);
        }
        mbar_wait(q_full, (item_count & 1), nullptr, kSiteQFull, 100000000ull);
      }
    }
  } else if (warp == kWMma) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      int g = 0, item_count = 0;
      int e = 0;  // causal: entries written to the key-position ring
      bool ok = true;
      const uint32_t qbase = smem_u32(sQ);
      auto issue_qk = [&](int x, int stage) {
        const uint32_t kb = smem_u32(sK + stage * C::kKTile);
        const uint32_t qb = qbase + x * C::kQTile;
#pragma unroll
        for (int ks = 0; ks < C::kKSteps; ++ks) {
          const uint32_t sub = ks >> 2, inner = (ks & 3) * 32;
          const uint64_t adesc = make_sdesc(qb + sub * (kM * 128) + inner, 16, 1024);
          const uint64_t bdesc = make_sdesc(kb + sub * (kN * 128) + inner, 16, 1024);
          mma_ss<false>(tmem + col_s(x), adesc, bdesc, C::kIdescQK, ks ? 1u : 0u);
        }
        mma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int gp, bool first) -> bool {
        const int stage = gp % NS;
        if (!mbar_wait(&p_full[x], gp & 1, st, kSitePFull, tmo)) return false;
        if (x == 0 && !mbar_wait(&v_full[stage], (gp / NS) & 1, st, kSiteVFull, tmo)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(sV + stage * C::kVTile);
#pragma unroll
        for (int ks = 0; ks < C::kPSteps; ++ks) {
          if (kPParts == 2 && ks == C::kPSteps / 2) {  // keys 64..127 of P
            if (!mbar_wait(&p_hi[x], gp & 1, st, kSitePFull, tmo)) return false;
            tc_fence_after();
          }
          const uint64_t bdesc = make_sdesc(vb + ks * 2048, kN * 128, 1024);
          mma_ts<false>(tmem + col_o(x), tmem + col_s(x) + ks * 8, bdesc, C::kIdescPV,
                        (first && ks == 0) ? 0u : 1u);
        }
        if (x == 1) mma_commit(&v_empty[stage]);  // tile B is the last reader of V
        mma_commit(&pv_done[x]);
        return true;
      };
      for (int w = 0; ok; ++w, ++item_count) {
        Item it;
        if constexpr (kCausal) {
          const int slot = w % kItemSlots;
          ok = mbar_wait(&item_full[slot], (w / kItemSlots) & 1, st, kSiteItemQueue, tmo);
          if (!ok) break;
          it = s_items[slot];
          mbar_arrive(&item_empty[slot]);  // the item now lives in registers
          if (it.unit < 0) break;
        } else {
          const int item = blockIdx.x + w * gridDim.x;
          if (item >= p.n_items) break;
          it = make_item(p, item, tiles_total);
        }
        ok = mbar_wait(q_full, item_count & 1, st, kSiteQFull, tmo);
        if (!ok) break;
        tc_fence_after();
        int j = 0;
        TileWalk<kN> wk;
        int v = it.v_begin;
        bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, unit_q_hi(p, it.q0))
                            : v < it.v_end;
        for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
          if constexpr (kCausal) {
            s_klo[e % kKloSlots] = wk.k_lo;
            mbar_arrive(&klo_full[e % kKloSlots]);
            ++e;
          }
          const int stage = g % NS;
          ok = mbar_wait(&k_full[stage], (g / NS) & 1, st, kSiteKFull, tmo);
          if (!ok) break;
          tc_fence_after();
          issue_qk(0, stage);
          if (j > 0) {
            ok = issue_pv(1, g - 1, j == 1);
            if (!ok) break;
          }
          issue_qk(1, stage);
          mma_commit(&k_empty[stage]);
          ok = issue_pv(0, g, j == 0);
          if (!ok) break;
          ++j;
          ++g;
        }
        if (kCausal && ok) {  // the softmax's end of this item
          s_klo[e % kKloSlots] = kKloEnd;
          mbar_arrive(&klo_full[e % kKloSlots]);
          ++e;
        }
        if (ok && j > 0) {
          ok = issue_pv(1, g - 1, j == 1);
          if (ok) mma_commit(o_final);
        }
        mma_commit(q_empty);  // Q smem may be reloaded once these MMAs are done
      }
      mma_commit(drain);
      mbar_wait(drain, 0, nullptr, kSiteOReady, 1000000000ull);
    }
  } else {
    if (p.fused && p.world > 1) ring_copy_role(p, threadIdx.x - kWComm * 32, &s_copy_ok);
  }
  } else {
    warpgroup_reg_inc<kRegsHigh>();
    // -------------------------------------------------------------- softmax
    const int x = (warp - kWSoft) >> 2;             // query tile of this warpgroup
    const int row = (threadIdx.x - kWSoft * 32) & 127;
    const uint32_t lane_base = ((warp & 3) * 32) << 16;
    const float sl2 = p.scale_log2;
    const uint32_t s_col = tmem + lane_base + col_s(x);
    const uint32_t o_col = tmem + lane_base + col_o(x);
    int g = 0, final_count = 0;
    int e = 0;  // causal: entries read from the key-position ring
    bool ok = true;
    for (int w = 0; ok; ++w) {
      const int slot = w % kItemSlots;
      Item it;
      if constexpr (kCausal) {
        ok = __all_sync(0xffffffffu, mbar_wait(&item_full[slot], (w / kItemSlots) & 1, st,
                                               kSiteItemQueue, tmo));
        if (!ok) break;
        it = s_items[slot];
        if (it.unit < 0) break;
      } else {
        const int item = blockIdx.x + w * gridDim.x;
        if (item >= p.n_items) break;
        it = make_item(p, item, tiles_total);
      }
      const int q0 = it.q0 + x * kM;
      float m_run = -INFINITY, l_run = 0.f;
      int j = 0;
      // global positions of this warpgroup's query tile (causal classification)
      const int q_lo_own = kCausal ? global_pos(q0, p.rank, p.Sq, p.world, p.zigzag) : 0;
      int v = it.v_begin;  // non-causal: the tile
      int k_lo = 0;        // causal: the tile's first global key position (MMA thread)
      // causal: the next visible tile of this item from the ring; false at its end
      auto next_klo = [&]() -> bool {
        const int ks = e % kKloSlots;
        ok = __all_sync(0xffffffffu, mbar_wait(&klo_full[ks], (e / kKloSlots) & 1, st,
                                               kSiteSFull, tmo));
        if (!ok) return false;
        k_lo = s_klo[ks];
        ++e;
        return k_lo != kKloEnd;
      };
      bool more = kCausal ? next_klo() : v < it.v_end;
      for (; more && ok; more = kCausal ? next_klo() : ++v < it.v_end) {
        int lim = kN;   // visible columns: c <= lim
        int cls = 1;    // this query tile's class of the tile: 0 masked, 1 full, 2 diagonal
        if constexpr (kCausal) {
          // the tile is visible to the unit; classify it for this query tile
          cls = k_lo > q_lo_own + kM - 1 ? 0 : (k_lo + kN - 1 <= q_lo_own ? 1 : 2);
          lim = cls == 0 ? -1 : (cls == 2 ? q_lo_own + row - k_lo : kN);
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[x], g & 1, st, kSiteSFull, tmo));
        if (!ok) break;
        tc_fence_after();
        // the whole S row of this thread in registers
        uint32_t sr[kN];
#pragma unroll
        for (int c = 0; c < kN; c += 32) tmem_ld32(s_col + c, sr + c);
        tmem_ld_wait();
        if (kCausal && cls != 1) {
          // only tiles the mask cuts (the same class for every row of the query
          // tile, so the branch is uniform); full tiles skip the 128 selects
#pragma unroll
          for (int c = 0; c < kN; ++c)
            if (c > lim) sr[c] = 0xff800000u;  // -inf
        }
        // row max: 3-input max folds two new columns per instruction
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = __uint_as_float(sr[i]);
#pragma unroll
        for (int c = 8; c < kN; c += 2)
          pm[(c >> 1) & 7] =
              fmax3(pm[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        const float mx = fmaxf(fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]),
                                     pm[6]),
                               pm[7]) * sl2;
        const bool need = mx > m_run + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - mx);
          m_run = mx;
          l_run *= alpha;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // PV of this tile's previous step precedes this step's QK in the
          // MMA order, so it has completed; the wait is a safety net
          ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[x], (g - 1) & 1, st, kSitePvDone, tmo));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            uint32_t o[32];
            tmem_ld32(o_col + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_col + c, o);
          }
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        // exponentials, row sum, packed bf16 P over the first 64 S columns;
        // the scale-and-shift and the row sum run as packed fp32 pairs
        const float2 scale2 = make_float2(sl2, sl2);
        const float2 shift2 = make_float2(-m_use, -m_use);
        float2 ps2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        // two halves of 32 packed columns: each half's P goes to TMEM before the
        // next is formed (fewer live registers at the softmax's 216-register cap)
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
          uint32_t pk[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int i = hlf * 32 + j;
            const float2 x = ffma2(make_float2(__uint_as_float(sr[2 * i]),
                                               __uint_as_float(sr[2 * i + 1])),
                                   scale2, shift2);
            const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            ps2[j & 3] = fadd2(ps2[j & 3], e);
            pk[j] = pack_bf16x2(e.x, e.y);
          }
          tmem_st32(s_col + hlf * 32, pk);
          if (kPParts == 2 && hlf == 0) {  // keys 0..63 of P are ready for the MMA
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane_id() == 0) mbar_arrive(&p_full[x]);
          }
        }
        const float2 ps = fadd2(fadd2(ps2[0], ps2[1]), fadd2(ps2[2], ps2[3]));
        l_run += ps.x + ps.y;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();  // the warp's TMEM stores are complete and fenced
        if (lane_id() == 0) mbar_arrive(kPParts == 2 ? &p_hi[x] : &p_full[x]);
        ++j;
        ++g;
      }
      if (!ok) break;
      // ---- epilogue ----
      const bool have = j > 0;
      if (have) {
        ok = __all_sync(0xffffffffu, mbar_wait(o_final, final_count & 1, st, kSiteOReady, tmo));
        ++final_count;
        if (!ok) break;
        tc_fence_after();
      }
      const float m_nat = have ? m_run * kLn2 : -INFINITY;
      // the item again (queue slot or static list) rather than kept live across
      // the tile loop: the causal softmax runs at its register cap
      const Item ie = kCausal ? s_items[slot] : make_item(p, blockIdx.x + w * gridDim.x,
                                                         tiles_total);
      const int qrow = ie.q0 + x * kM + row;
      const size_t r = static_cast<size_t>(qrow) * p.Hq + ie.h;
      const bool split = ie.store >= 0;
      // (RAB_DEBUG_BOUNDS builds: an out-of-range row or record is reported, its stores skipped)
      const bool out_in =
          st_bounds(st, qrow < p.Sq && ie.h < p.Hq && (!split || ie.store < p.n_items),
                    split ? kBoundsRecord : kBoundsQRow, split ? ie.store : qrow);
      const float inv = (have && l_run > 0.f && !p.partial && !split) ? 1.f / l_run : 1.f;
      const size_t srow =
          static_cast<size_t>(split ? ie.store : 0) * p.rows_per_unit + x * kM + row;
      float* dst_f32 = nullptr;
      if (split)
        dst_f32 = p.split_acc + srow * D;
      else if (p.partial)
        dst_f32 = p.acc + r * D;
      else if (!p.out_bf16)
        dst_f32 = static_cast<float*>(p.out) + r * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        if (have) {
          tmem_ld32(o_col + c, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (!out_in) {
          // nothing stored (the TMEM load above is warp-collective and stays)
        } else if (dst_f32 != nullptr) {
          float4* d4 = reinterpret_cast<float4*>(dst_f32 + c);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                __uint_as_float(o[4 * i + 2]) * inv,
                                __uint_as_float(o[4 * i + 3]) * inv);
        } else {
          uint4* d4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + r * D + c);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv,
                                           __uint_as_float(o[8 * i + 1]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv,
                                           __uint_as_float(o[8 * i + 3]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv,
                                           __uint_as_float(o[8 * i + 5]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv,
                                           __uint_as_float(o[8 * i + 7]) * inv));
        }
      }
      if (!out_in) {
        // reported above
      } else if (split) {
        p.split_m[srow] = m_nat;
        p.split_l[srow] = l_run;
      } else if (p.partial) {
        if (p.m_out) p.m_out[r] = m_nat;
        if (p.l_out) p.l_out[r] = l_run;
      } else if (p.lse != nullptr) {
        p.lse[r] = (have && l_run > 0.f) ? m_nat + logf(l_run) : -INFINITY;
      }
      tc_fence_before();
      if constexpr (kCausal) {
        __syncwarp();
        if (lane_id() == 0) mbar_arrive(&item_empty[slot]);  // queue slot free again
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (kCausal && p.dynamic && threadIdx.x == 0) {
    // every CTA has stopped claiming; the last one resets the claim counter
    // for the next launch that uses this status block
    __threadfence();
    if (atomicAdd(&st->pad[1], 1u) == gridDim.x - 1) {
      atomicExch(&st->pad[0], 0u);
      atomicExch(&st->pad[1], 0u);
    }
  }
  if (threadIdx.x == 0) finish_launch(p);  // device-side epochs: bump the call counter
  if (warp == kWMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

template <int D, bool kCausal, int kPParts>
int launch2(const FlashParams& p, const CUtensorMap& tq, const FlashMaps& maps, int grid,
            bool cooperative, cudaStream_t stream) {
  using C = Cfg2<D>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaFuncSetAttribute(flash_fwd_2q_kernel<D, kCausal, kPParts>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  if (cooperative) {
    void* args[] = {const_cast<FlashParams*>(&p), const_cast<CUtensorMap*>(&tq),
                    const_cast<CUtensorMap*>(&maps.k), const_cast<CUtensorMap*>(&maps.v)};
    return static_cast<int>(cudaLaunchCooperativeKernel(
        reinterpret_cast<void*>(flash_fwd_2q_kernel<D, kCausal, kPParts>), dim3(grid), dim3(kThreads2), args,
        C::kSmemBytes, stream));
  }
  flash_fwd_2q_kernel<D, kCausal, kPParts><<<grid, kThreads2, C::kSmemBytes, stream>>>(p, tq, maps.k, maps.v);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

CUtensorMap flash_make_q_map(const void* q, int Sq, int Hq, int D) {
  uint64_t dims[3] = {(uint64_t)D, (uint64_t)Hq, (uint64_t)Sq};
  uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)Hq * D * 2};
  uint32_t box[3] = {64, 1, 128};
  return make_tmap(q, TmapDtype::kBF16, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int flash_forward_2q_launch(const FlashParams& p, const CUtensorMap& tq, const FlashMaps& maps,
                            int grid, bool cooperative, cudaStream_t stream) {
  if (p.rows_per_unit != 256 || p.Sq % 256 != 0)
    throw std::runtime_error("flash 2q: needs 256-row units");
  if (p.Skv % 128 != 0) throw std::runtime_error("flash 2q: keys per block must be a multiple of 128");
  if (p.D == 64)
    return p.causal ? launch2<64, true, 1>(p, tq, maps, grid, cooperative, stream)
                    : launch2<64, false, 1>(p, tq, maps, grid, cooperative, stream);
  if (p.D == 128) {
    // P in two halves for causal launches (measured on B200, 16k x 32 heads:
    // 1160 vs 1029 TFLOP/s; 64k GQA: 1164 vs 1075), whole for non-causal ones
    // (1139 vs 1247); RAB_FLASH_PSPLIT=1|2 overrides for comparison
    const char* e = std::getenv("RAB_FLASH_PSPLIT");
    const bool two = e != nullptr && (std::strcmp(e, "1") == 0 || std::strcmp(e, "2") == 0)
                         ? std::strcmp(e, "2") == 0
                         : p.causal != 0;
    if (two)
      return p.causal ? launch2<128, true, 2>(p, tq, maps, grid, cooperative, stream)
                      : launch2<128, false, 2>(p, tq, maps, grid, cooperative, stream);
    return p.causal ? launch2<128, true, 1>(p, tq, maps, grid, cooperative, stream)
                    : launch2<128, false, 1>(p, tq, maps, grid, cooperative, stream);
  }
  throw std::runtime_error("flash 2q: head_dim must be 64 or 128");
}

}  // namespace rab
