// flash_fwd_2sm_sm100.cu - bf16 flash-attention forward on CTA PAIRS (thread-
// block clusters of two, tcgen05 cta_group::2) for B200 (sm_100a).  Like the
// other flash kernels it stands in for the reference's row-per-CTA partial
// attention kernel (src/attention/ring_attention_nccl_gpu_bench.cu:46-111) and
// its merge (:113-134); the reference re-reads every K/V row from global
// memory once per query row, this kernel shares each K/V tile between the
// four 128-row query tiles a CTA pair holds.
//
// Work unit: 512 query rows of one head, two pair tiles of 256 rows, A = rows
// [0, 256) and B = rows [256, 512).  CTA r of the pair (r = 0 is the leader)
// holds rows [128r, 128r + 128) of A and of B: its own Q in shared memory, its
// own S and O accumulators in TMEM, its own softmax.  Each K/V tile of 128 keys
// is loaded HALF by each CTA into its own shared memory, with plain TMA loads
// (no cluster broadcast): K rows [64r, 64r + 64) and V columns [64r, 64r + 64).
// One thread of the leader issues every MMA of the pair as an M = 256
// cta_group::2 MMA, which reads the A rows and the B half of each CTA:
//     S_x = Q_x K^T   (A = Q from shared memory, B = the two K halves)
//     O_x += P_x V    (A = P from TMEM,          B = the two V halves)
// in the two-tile ping-pong order QK_A, PV_B, QK_B, PV_A, so each tile's
// softmax runs while the other tile's MMAs execute.  Per CTA this halves the
// K/V shared-memory footprint and load traffic of the two-tile kernel (four
// stages fit instead of two) and the B-operand reads of every MMA.
//
// Synchronisation inside the pair:
//  * each CTA's TMA loads complete on its own mbarriers; warp 1 of the
//    non-leader CTA relays each completed stage (Q, K half, V half) to the
//    leader's barrier of that stage (count 2: the leader's own arrive with its
//    bytes, plus the relay), so the leader's MMA waits for both halves and each
//    CTA drains its own loads on an error;
//  * the MMA's completions (S ready, stage free, PV done, O final, Q free)
//    are committed to the same barrier in both CTAs (multicast commit);
//  * both CTAs' softmax warps arrive on the leader's P-ready barriers;
//  * causal launches claim work items dynamically in the leader's TMA thread,
//    which writes each item into both CTAs' shared-memory queues.
// Every wait is bounded; the pair unwinds together and meets at a cluster
// barrier before the TMEM is released.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>
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

constexpr int kThreadsP = 384;
constexpr int kPWTma = 0;
constexpr int kPWMma = 1;     // leader: MMA issuer; non-leader: relay of completed loads
constexpr int kPWComm = 2;    // warps 2-3: ring copy (fused mode)
constexpr int kPWSoft = 4;    // warps 4-7 tile A, 8-11 tile B
constexpr uint32_t kPCols = 512;
constexpr uint32_t kPRegsLaunch = 168;
constexpr uint32_t kPRegsLow = 72;
constexpr uint32_t kPRegsHigh = 216;
static_assert(128 * kPRegsLow + 256 * kPRegsHigh <= kPRegsLaunch * 384,
              "register split exceeds the launch allocation");

constexpr int kD = 128;                  // head dim (the pair kernel is d = 128 only)
constexpr int kN = 128;                  // keys per KV tile (both halves)
constexpr int kHalfN = 64;               // keys of K (and d columns of V) per CTA
constexpr int kQTile = 128 * kD * 2;     // 32 KiB: one CTA's 128 rows of a pair tile
constexpr int kKHalf = kHalfN * kD * 2;  // 16 KiB
constexpr int kVHalf = kN * kHalfN * 2;  // 16 KiB
constexpr int kStages = 4;
constexpr int kSmemTiles = 2 * kQTile + kStages * (kKHalf + kVHalf);
constexpr int kNumBars = 4 * kStages + 10 + 2 * kItemSlots;
constexpr int kSmemBytes = kSmemTiles + 1024 + kNumBars * 8 + 64;
constexpr int kUnitRows = 512;
constexpr int kItemWords = sizeof(Item) / 4;
static_assert(sizeof(Item) % 4 == 0, "Item is copied as 32-bit words");
// M = 256 pair MMAs: QK^T (N = 128 keys), PV (N = 128 head dims, V MN-major)
constexpr uint32_t kIdescQK = make_idesc(kFmtBF16, kFmtBF16, 256, kN, kMajorK, kMajorK);
constexpr uint32_t kIdescPV = make_idesc(kFmtBF16, kFmtBF16, 256, kD, kMajorK, kMajorMN);
constexpr uint16_t kPair = 0x3;  // multicast mask: both CTAs

__device__ __forceinline__ uint32_t pcol_s(int x) { return x ? 128u : 0u; }
__device__ __forceinline__ uint32_t pcol_o(int x) { return x ? 384u : 256u; }

// Last global query position of the 512-row unit at local row q0: a KV tile is
// processed when the unit's last 128 query rows see it (later rows see more
// keys, so a tile masked for them is masked for all four query tiles).
__device__ __forceinline__ int unit_q_hi(const FlashParams& p, int q0) {
  return global_pos(q0 + kUnitRows - kM, p.rank, p.Sq, p.world, p.zigzag) + kM - 1;
}

template <bool kCausal>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsP, 1)
    flash_fwd_2sm_kernel(const __grid_constant__ FlashParams p,
                         const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // [2][kQTile]
  uint8_t* sK = smem + 2 * kQTile;          // [kStages][kKHalf]
  uint8_t* sV = sK + kStages * kKHalf;      // [kStages][kVHalf]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemTiles);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + kStages;
  uint64_t* v_full = bars + 2 * kStages;
  uint64_t* v_empty = bars + 3 * kStages;
  uint64_t* q_full = bars + 4 * kStages;
  uint64_t* q_empty = bars + 4 * kStages + 1;
  uint64_t* s_full = bars + 4 * kStages + 2;   // [2]
  uint64_t* p_full = bars + 4 * kStages + 4;   // [2] (leader's are the ones used)
  uint64_t* pv_done = bars + 4 * kStages + 6;  // [2]
  uint64_t* o_final = bars + 4 * kStages + 8;
  uint64_t* drain = bars + 4 * kStages + 9;
  uint64_t* item_full = bars + 4 * kStages + 10;                 // [kItemSlots]
  uint64_t* item_empty = bars + 4 * kStages + 10 + kItemSlots;  // [kItemSlots] (leader's)
  __shared__ uint32_t tmem_slot;
  __shared__ int s_copy_ok;
  __shared__ Item s_items[kItemSlots];

  const uint32_t warp = warp_id();
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int n_pairs = static_cast<int>(gridDim.x >> 1);
  DeviceStatus* st = p.status;
  const uint64_t tmo = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], leader ? 2 : 1);  // leader: own loads + the peer's relay
      mbar_init(&v_full[i], leader ? 2 : 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(q_full, leader ? 2 : 1);
    mbar_init(q_empty, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 8);  // one arrival per softmax warp of each CTA
      mbar_init(&pv_done[x], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&item_full[i], 1);
      // leader: its MMA thread + 8 softmax warps, the peer's 8 softmax warps,
      // the peer's TMA thread and relay thread
      mbar_init(&item_empty[i], 1 + 8 + 8 + 1 + 1);
    }
    fence_barrier_init();
  }
  if (warp == kPWMma) {
    tmem_alloc2(&tmem_slot, kPCols);
    tmem_relinquish2();
  }
  __syncthreads();
  tc_fence_after();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
  const uint32_t tmem = tmem_slot;
  const int tpb = p.Skv / kN;
  const int tiles_total = p.nblk * tpb;
  // shared::cluster addresses of the leader's barriers / the peer's queue
  auto leader_bar = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 0); };

  // The k-th work item of this pair (static schedule) or of the queue.
  auto static_item = [&](int w, Item* it) -> bool {
    const int item = pair + w * n_pairs;
    if (item >= p.n_items) return false;
    *it = make_item(p, item, tiles_total);
    return true;
  };
  // consumers of the causal queue release a slot on the leader's barrier
  auto release_slot = [&](int slot) {
    if (leader)
      mbar_arrive(&item_empty[slot]);
    else
      mbar_arrive_cluster(leader_bar(&item_empty[slot]));
  };

  if (warp < 4) {
    warpgroup_reg_dec<kPRegsLow>();
    if (warp == kPWTma) {
      // -------------------------------------------------------------- TMA
      if (elect_one()) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        trace_stamp(p, 0, 0, globaltimer_ns());
        int g = 0, item_count = 0, ready_blocks = 1;
        bool ok = true;
        for (int w = 0; ok; ++w, ++item_count) {
          Item it;
          int slot = 0;
          if constexpr (kCausal) {
            slot = w % kItemSlots;
            if (leader) {
              if (w >= kItemSlots) {
                ok = mbar_wait_cl(&item_empty[slot], ((w / kItemSlots) - 1) & 1, st,
                                  kSiteItemQueue, tmo);
                if (!ok) break;
              }
              bool have;
              if (p.dynamic) {
                have = claim_item(p, tiles_total, &it);
              } else {
                have = static_item(w, &it);
              }
              if (!have) it.unit = -1;
              s_items[slot] = it;
              // the same item into the peer's queue, then release it to both CTAs
              const uint32_t* src = reinterpret_cast<const uint32_t*>(&it);
              const uint32_t dst = mapa_shared(smem_u32(&s_items[slot]), 1);
#pragma unroll
              for (int i = 0; i < kItemWords; ++i) st_cluster_u32(dst + 4 * i, src[i]);
              mbar_arrive(&item_full[slot]);
              mbar_arrive_cluster(mapa_shared(smem_u32(&item_full[slot]), 1));
              if (!have) break;
            } else {
              ok = mbar_wait_cl(&item_full[slot], (w / kItemSlots) & 1, st, kSiteItemQueue, tmo);
              if (!ok) break;
              it = s_items[slot];
              release_slot(slot);  // copied into registers
              if (it.unit < 0) break;
            }
          } else {
            if (!static_item(w, &it)) break;
          }
          // this CTA's 128 rows of pair tiles A and B
          ok = mbar_wait_cl(q_empty, (item_count & 1) ^ 1, st, kSiteQFull, tmo);
          if (!ok) break;
          mbar_arrive_expect_tx(q_full, 2 * kQTile);
#pragma unroll
          for (int x = 0; x < 2; ++x)
#pragma unroll
            for (int ds = 0; ds < kD / 64; ++ds)
              tma_load_3d(sQ + x * kQTile + ds * (kM * 128), &tmQ, q_full, ds * 64, it.h,
                          it.q0 + x * 256 + static_cast<int>(crank) * kM);
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
            const int stage = g % kStages;
            const uint32_t ph = (g / kStages) & 1;
            ok = mbar_wait_cl(&k_empty[stage], ph ^ 1, st, kSiteKEmpty, tmo);
            if (!ok) break;
            mbar_arrive_expect_tx(&k_full[stage], kKHalf);
            // K rows [64 crank, 64 crank + 64) of the tile, both 64-column blocks
#pragma unroll
            for (int ds = 0; ds < kD / 64; ++ds)
              tma_load_4d(sK + stage * kKHalf + ds * (kHalfN * 128), &tmK, &k_full[stage], ds * 64,
                          it.hk, t * kN + static_cast<int>(crank) * kHalfN, s);
            ok = mbar_wait_cl(&v_empty[stage], ph ^ 1, st, kSiteVEmpty, tmo);
            if (!ok) break;
            mbar_arrive_expect_tx(&v_full[stage], kVHalf);
            // V columns [64 crank, 64 crank + 64) of all 128 keys
            tma_load_4d(sV + stage * kVHalf, &tmV, &v_full[stage],
                        static_cast<int>(crank) * kHalfN, it.hk, t * kN, s);
            ++g;
          }
        }
        trace_stamp(p, 0, 1, globaltimer_ns());
        if (!ok) {
          // drain this CTA's own loads (their barriers are local)
          for (int i = 0; i < kStages && i < g; ++i) {
            const int gg = g - 1 - i;
            mbar_wait(&k_full[gg % kStages], (gg / kStages) & 1, nullptr, kSiteKFull, 100000000ull);
            mbar_wait(&v_full[gg % kStages], (gg / kStages) & 1, nullptr, kSiteVFull, 100000000ull);
          }
          mbar_wait(q_full, item_count & 1, nullptr, kSiteQFull, 100000000ull);
        }
      }
    } else if (warp == kPWMma) {
      if (leader) {
        // ---------------------------------------------------- MMA (leader)
        if (elect_one()) {
          int g = 0, item_count = 0;
          bool ok = true;
          const uint32_t qbase = smem_u32(sQ);
          auto issue_qk = [&](int x, int stage) {
            const uint32_t kb = smem_u32(sK + stage * kKHalf);
            const uint32_t qb = qbase + x * kQTile;
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks) {
              const uint32_t sub = ks >> 2, inner = (ks & 3) * 32;
              const uint64_t adesc = make_sdesc(qb + sub * (kM * 128) + inner, 16, 1024);
              const uint64_t bdesc = make_sdesc(kb + sub * (kHalfN * 128) + inner, 16, 1024);
              mma2_ss(tmem + pcol_s(x), adesc, bdesc, kIdescQK, ks ? 1u : 0u);
            }
            mma_commit2_mc(&s_full[x], kPair);
          };
          auto issue_pv = [&](int x, int gp, bool first) -> bool {
            const int stage = gp % kStages;
            if (!mbar_wait_cl(&p_full[x], gp & 1, st, kSitePFull, tmo)) return false;
            if (x == 0 &&
                !mbar_wait_cl(&v_full[stage], (gp / kStages) & 1, st, kSiteVFull, tmo))
              return false;
            tc_fence_after();
            const uint32_t vb = smem_u32(sV + stage * kVHalf);
#pragma unroll
            for (int ks = 0; ks < kN / 16; ++ks) {
              // MN-major V half: 64 head dims (one 128-byte block) x 16 keys per step
              const uint64_t bdesc = make_sdesc(vb + ks * 2048, kN * 128, 1024);
              mma2_ts(tmem + pcol_o(x), tmem + pcol_s(x) + ks * 8, bdesc, kIdescPV,
                      (first && ks == 0) ? 0u : 1u);
            }
            if (x == 1) mma_commit2_mc(&v_empty[stage], kPair);  // tile B reads V last
            mma_commit2_mc(&pv_done[x], kPair);
            return true;
          };
          for (int w = 0; ok; ++w, ++item_count) {
            Item it;
            if constexpr (kCausal) {
              const int slot = w % kItemSlots;
              ok = mbar_wait_cl(&item_full[slot], (w / kItemSlots) & 1, st, kSiteItemQueue, tmo);
              if (!ok) break;
              it = s_items[slot];
              mbar_arrive(&item_empty[slot]);
              if (it.unit < 0) break;
            } else {
              if (!static_item(w, &it)) break;
            }
            ok = mbar_wait_cl(q_full, item_count & 1, st, kSiteQFull, tmo);
            if (!ok) break;
            tc_fence_after();
            int j = 0;
            TileWalk<kN> wk;
            int v = it.v_begin;
            bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, unit_q_hi(p, it.q0))
                                : v < it.v_end;
            for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
              const int stage = g % kStages;
              ok = mbar_wait_cl(&k_full[stage], (g / kStages) & 1, st, kSiteKFull, tmo);
              if (!ok) break;
              tc_fence_after();
              issue_qk(0, stage);
              if (j > 0) {
                ok = issue_pv(1, g - 1, j == 1);
                if (!ok) break;
              }
              issue_qk(1, stage);
              mma_commit2_mc(&k_empty[stage], kPair);
              ok = issue_pv(0, g, j == 0);
              if (!ok) break;
              ++j;
              ++g;
            }
            if (ok && j > 0) {
              ok = issue_pv(1, g - 1, j == 1);
              if (ok) mma_commit2_mc(o_final, kPair);
            }
            mma_commit2_mc(q_empty, kPair);  // Q may be reloaded once these MMAs are done
          }
          mma_commit2_mc(drain, kPair);
          mbar_wait_cl(drain, 0, nullptr, kSiteOReady, 1000000000ull);
        }
      } else {
        // ------------------------------------- relay (non-leader CTA)
        // Follows the TMA thread's sequence; forwards each completed local
        // load to the leader's barrier of the same stage.
        if (elect_one()) {
          int g = 0, item_count = 0;
          bool ok = true;
          for (int w = 0; ok; ++w, ++item_count) {
            Item it;
            if constexpr (kCausal) {
              const int slot = w % kItemSlots;
              ok = mbar_wait_cl(&item_full[slot], (w / kItemSlots) & 1, st, kSiteItemQueue, tmo);
              if (!ok) break;
              it = s_items[slot];
              release_slot(slot);
              if (it.unit < 0) break;
            } else {
              if (!static_item(w, &it)) break;
            }
            ok = mbar_wait(q_full, item_count & 1, st, kSiteQFull, tmo);
            if (!ok) break;
            mbar_arrive_cluster(leader_bar(q_full));
            TileWalk<kN> wk;
            int v = it.v_begin;
            bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, unit_q_hi(p, it.q0))
                                : v < it.v_end;
            for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
              const int stage = g % kStages;
              const uint32_t ph = (g / kStages) & 1;
              ok = mbar_wait(&k_full[stage], ph, st, kSiteKFull, tmo);
              if (!ok) break;
              mbar_arrive_cluster(leader_bar(&k_full[stage]));
              ok = mbar_wait(&v_full[stage], ph, st, kSiteVFull, tmo);
              if (!ok) break;
              mbar_arrive_cluster(leader_bar(&v_full[stage]));
              ++g;
            }
          }
        }
      }
    } else {
      if (p.fused && p.world > 1) ring_copy_role(p, threadIdx.x - kPWComm * 32, &s_copy_ok);
    }
  } else {
    warpgroup_reg_inc<kPRegsHigh>();
    // ------------------------------------------------------------ softmax
    const int x = (warp - kPWSoft) >> 2;  // pair tile of this warpgroup
    const int row = (threadIdx.x - kPWSoft * 32) & 127;
    const uint32_t lane_base = ((warp & 3) * 32) << 16;
    const float sl2 = p.scale_log2;
    const uint32_t s_col = tmem + lane_base + pcol_s(x);
    const uint32_t o_col = tmem + lane_base + pcol_o(x);
    const uint32_t p_bar = leader ? 0u : leader_bar(&p_full[x]);
    const int my_off = x * 256 + static_cast<int>(crank) * kM;  // first unit row of this tile
    int g = 0, final_count = 0;
    bool ok = true;
    for (int w = 0; ok; ++w) {
      const int slot = w % kItemSlots;
      Item it;
      if constexpr (kCausal) {
        ok = __all_sync(0xffffffffu, mbar_wait_cl(&item_full[slot], (w / kItemSlots) & 1, st,
                                                  kSiteItemQueue, tmo));
        if (!ok) break;
        it = s_items[slot];
        if (it.unit < 0) break;
      } else {
        if (!static_item(w, &it)) break;
      }
      const int q0 = it.q0 + my_off;
      const int qrow = q0 + row;
      float m_run = -INFINITY, l_run = 0.f;
      int j = 0;
      const int q_lo_own = kCausal ? global_pos(q0, p.rank, p.Sq, p.world, p.zigzag) : 0;
      TileWalk<kN> wk;
      int v = it.v_begin;
      bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, unit_q_hi(p, it.q0))
                          : v < it.v_end;
      for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
        int lim = kN;
        int cls = 1;
        if constexpr (kCausal) {
          const int k_lo = wk.k_lo;  // visible to the unit; classify for this query tile
          cls = k_lo > q_lo_own + kM - 1 ? 0 : (k_lo + kN - 1 <= q_lo_own ? 1 : 2);
          lim = cls == 0 ? -1 : (cls == 2 ? q_lo_own + row - k_lo : kN);
        }
        ok = __all_sync(0xffffffffu, mbar_wait_cl(&s_full[x], g & 1, st, kSiteSFull, tmo));
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[kN];
#pragma unroll
        for (int c = 0; c < kN; c += 32) tmem_ld32(s_col + c, sr + c);
        tmem_ld_wait();
        if (kCausal && cls != 1) {
#pragma unroll
          for (int c = 0; c < kN; ++c)
            if (c > lim) sr[c] = 0xff800000u;  // -inf
        }
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
          ok = __all_sync(0xffffffffu,
                          mbar_wait_cl(&pv_done[x], (g - 1) & 1, st, kSitePvDone, tmo));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < kD; c += 32) {
            uint32_t o[32];
            tmem_ld32(o_col + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_col + c, o);
          }
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
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
            const float2 xx = ffma2(make_float2(__uint_as_float(sr[2 * i]),
                                               __uint_as_float(sr[2 * i + 1])),
                                   scale2, shift2);
            const float2 e = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
            ps2[j & 3] = fadd2(ps2[j & 3], e);
            pk[j] = pack_bf16x2(e.x, e.y);
          }
          tmem_st32(s_col + hlf * 32, pk);
        }
        const float2 ps = fadd2(fadd2(ps2[0], ps2[1]), fadd2(ps2[2], ps2[3]));
        l_run += ps.x + ps.y;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();  // the warp's TMEM stores are complete and fenced
        if (lane_id() == 0) {
          if (leader)
            mbar_arrive(&p_full[x]);
          else
            mbar_arrive_cluster(p_bar);
        }
        ++j;
        ++g;
      }
      if (!ok) break;
      // ---- epilogue: this CTA's rows of tile x ----
      const bool have = j > 0;
      if (have) {
        ok = __all_sync(0xffffffffu, mbar_wait_cl(o_final, final_count & 1, st, kSiteOReady, tmo));
        ++final_count;
        if (!ok) break;
        tc_fence_after();
      }
      const float m_nat = have ? m_run * kLn2 : -INFINITY;
      const size_t r = static_cast<size_t>(qrow) * p.Hq + it.h;
      const bool split = it.store >= 0;
      const bool out_in =
          st_bounds(st, qrow < p.Sq && it.h < p.Hq && (!split || it.store < p.n_items),
                    split ? kBoundsRecord : kBoundsQRow, split ? it.store : qrow);
      const float inv = (have && l_run > 0.f && !p.partial && !split) ? 1.f / l_run : 1.f;
      const size_t srow = static_cast<size_t>(split ? it.store : 0) * p.rows_per_unit + my_off + row;
      float* dst_f32 = nullptr;
      if (split)
        dst_f32 = p.split_acc + srow * kD;
      else if (p.partial)
        dst_f32 = p.acc + r * kD;
      else if (!p.out_bf16)
        dst_f32 = static_cast<float*>(p.out) + r * kD;
#pragma unroll
      for (int c = 0; c < kD; c += 32) {
        uint32_t o[32];
        if (have) {
          tmem_ld32(o_col + c, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (!out_in) {
        } else if (dst_f32 != nullptr) {
          float4* d4 = reinterpret_cast<float4*>(dst_f32 + c);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                __uint_as_float(o[4 * i + 2]) * inv,
                                __uint_as_float(o[4 * i + 3]) * inv);
        } else {
          uint4* d4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + r * kD + c);
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
        if (lane_id() == 0) release_slot(slot);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (kCausal && p.dynamic && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&st->pad[1], 1u) == gridDim.x - 1) {
      atomicExch(&st->pad[0], 0u);
      atomicExch(&st->pad[1], 0u);
    }
  }
  if (threadIdx.x == 0) finish_launch(p);  // device-side epochs: bump the call counter
  // neither CTA leaves (or frees TMEM) while the pair's MMAs or the peer's
  // remote arrivals can still touch it
  cluster_sync();
  if (warp == kPWMma) {
    tc_fence_after();
    tmem_dealloc2(tmem, kPCols);
  }
}

template <bool kCausal>
int launch_pair(const FlashParams& p, const CUtensorMap& tq, const CUtensorMap& tk,
                const CUtensorMap& tv, int grid, bool cooperative, cudaStream_t stream) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaFuncSetAttribute(flash_fwd_2sm_kernel<kCausal>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBytes);
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsP);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  // The fused mode needs every CTA resident at once (the copy slices of all
  // CTAs feed every CTA's loads): callers size `grid` with flash_pair_max_grid,
  // the number of pairs the GPU holds at once, instead of a cooperative launch.
  (void)cooperative;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, flash_fwd_2sm_kernel<kCausal>, p, tq, tk, tv));
}

}  // namespace

int flash_pair_max_grid() {
  // CTA pairs that can be resident at once (a pair needs two SMs of one GPC);
  // the fused mode needs every CTA resident
  static int cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  cudaFuncSetAttribute(flash_fwd_2sm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       kSmemBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * flash_sm_count());
  cfg.blockDim = dim3(kThreadsP);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.attrs = nullptr;  // the cluster shape is the kernel's compile-time (2, 1, 1)
  cfg.numAttrs = 0;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, flash_fwd_2sm_kernel<false>, &cfg) != cudaSuccess ||
      clusters <= 0) {
    cudaGetLastError();
    clusters = flash_sm_count() / 2;
  }
  const int g = 2 * std::min(clusters, flash_sm_count() / 2);
  if (dev >= 0 && dev < 64) cache[dev] = g;
  return g;
}

int flash_forward_2sm_launch(const FlashParams& p, const CUtensorMap& tq, const void* k_base,
                             const void* v_base, size_t slot_stride, int grid, bool cooperative,
                             cudaStream_t stream) {
  if (p.D != kD) throw std::runtime_error("flash pair kernel: head_dim must be 128");
  if (p.rows_per_unit != kUnitRows || p.Sq % kUnitRows != 0)
    throw std::runtime_error("flash pair kernel: needs 512-row units");
  if (p.Skv % kN != 0) throw std::runtime_error("flash pair kernel: keys per block % 128");
  if (p.causal && p.zigzag && (p.Sq / 2) % kUnitRows != 0)
    throw std::runtime_error("flash pair kernel: zigzag halves must be multiples of 512 rows");
  if (grid % 2 != 0 || grid <= 0) throw std::runtime_error("flash pair kernel: grid must be even");
  if (p.dynamic && !p.causal)
    throw std::runtime_error("flash pair kernel: dynamic claiming is for causal launches");
  if (slot_stride == 0) slot_stride = ring_block_bytes(Prec::kBF16, p.Skv, p.Hkv, kD);
  // K in halves of 64 keys; V and Q in 128-row boxes of 64 columns
  uint64_t dims[4] = {(uint64_t)kD, (uint64_t)p.Hkv, (uint64_t)p.Skv, (uint64_t)p.nblk};
  uint64_t strides[3] = {(uint64_t)kD * 2, (uint64_t)p.Hkv * kD * 2, slot_stride};
  uint32_t kbox[4] = {64, 1, (uint32_t)kHalfN, 1};
  uint32_t vbox[4] = {64, 1, (uint32_t)kN, 1};
  const CUtensorMap tk =
      make_tmap(k_base, TmapDtype::kBF16, 4, dims, strides, kbox, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tv =
      make_tmap(v_base, TmapDtype::kBF16, 4, dims, strides, vbox, CU_TENSOR_MAP_SWIZZLE_128B);
  return p.causal ? launch_pair<true>(p, tq, tk, tv, grid, cooperative, stream)
                  : launch_pair<false>(p, tq, tk, tv, grid, cooperative, stream);
}

}  // namespace rab
