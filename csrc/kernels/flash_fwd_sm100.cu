// flash_fwd_sm100.cu - tcgen05 flash-attention forward for B200 (sm_100a),
// optionally fused with the ring: while the tensor cores consume the K/V blocks
// already in local memory, two copy warps in every CTA pull the blocks of the
// other ranks over NVLink (peer-mapped loads, 16-byte vectors) into this rank's
// ring slots.  Online softmax state stays on chip across all ring steps, so the
// per-step merge of the reference (src/attention/ring_attention_nccl_gpu_bench.cu
// :341-348, kernels C16 + C17) disappears into the running rescale.
//
// CTA = 12 warps, one 128-row query tile of one head at a time (persistent
// over work items):
//   warp 0      TMA producer: K / V tiles of the ring slots -> shared memory
//   warp 1      MMA issuer (one thread): S = Q K^T and O += P V on tcgen05,
//               commits to mbarriers; also owns the TMEM allocation
//   warps 2-3   ring copy warps (fused mode): peer slot -> local slot
//   warps 4-11  softmax, two warpgroups: each thread owns one query row and
//               one half of the key columns; S and O live in TMEM, P is
//               written back over S (A operand of the PV MMA from TMEM)
//
// Precisions:
//   kBF16   bf16 Q/K/V, kind::f16, fp32 accumulation, bf16 P.
//   kF32x3  fp32 Q/K/V.  Every product is formed as three kind::tf32 MMAs on
//           tf32 big/small splits (a_b*b_b + a_b*b_s + a_s*b_b; Ootomo &
//           Yokota 2022), P included, which keeps fp32-level accuracy on the
//           tensor cores.  Q is split in the kernel; K and V^T arrive pre-split
//           in the ring slots.
//
// The softmax uses lazy rescaling: the running max only moves (and O is only
// rescaled in TMEM) when a row max grows by more than 2^8, which keeps the
// exponentials <= 256 and the result exact up to rounding.
//
// Every wait is bounded (globaltimer); a timeout records the wait site in the
// status word and the CTA unwinds (draining its own TMA loads and MMAs) instead
// of hanging.  No TMA load here uses cluster multicast.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cstdint>
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

constexpr int kThreads = 384;  // 12 warps
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpComm = 2;      // warps 2 and 3
constexpr int kWarpSoftmax = 4;   // warps 4..11 (two warpgroups)
constexpr uint32_t kTmemCols = 512;

template <Prec P, int D>
struct Cfg {
  static constexpr bool kTF32 = (P == Prec::kF32x3);
  static_assert(!kTF32 || D == 64, "3xTF32 path supports head_dim 64");
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static constexpr int kN = kTF32 ? 64 : 128;       // keys per tile
  static constexpr int kEsize = kTF32 ? 4 : 2;
  static constexpr int kElems128 = 128 / kEsize;    // elements in a 128-byte row
  static constexpr int kPlanes = kTF32 ? 2 : 1;
  static constexpr int kKTile = kN * D * kEsize * kPlanes;  // bytes
  static constexpr int kVTile = kKTile;
  static constexpr int kStages = (kKTile + kVTile) <= 32768 ? 4 : 3;
  static constexpr int kSmemTiles = kStages * (kKTile + kVTile);
  static constexpr int kNumBars = 4 * kStages + 12 + 2 * kItemSlots;
  static constexpr int kSmemBytes = kSmemTiles + 1024 + kNumBars * 8 + 64;
  // TMEM columns
  static constexpr uint32_t kColQ = 0;                       // Q (tf32: Qb at 0, Qs at D)
  static constexpr uint32_t kQCols = kTF32 ? D : D / 2;      // per plane (tf32 only uses it)
  static constexpr uint32_t kColS0 = 128;
  static constexpr uint32_t kColS1 = kColS0 + (kTF32 ? 64 : 128);
  static constexpr uint32_t kColPs0 = kTF32 ? 256 : 0;       // tf32 small P planes
  static constexpr uint32_t kColPs1 = kTF32 ? 320 : 0;
  static constexpr uint32_t kColO = 384;
  // K-steps (each tcgen05.mma consumes 32 bytes of K)
  static constexpr int kKStepsQK = D * kEsize / 32;
  static constexpr int kKStepsPV = kN * kEsize / 32;
  static constexpr uint32_t kIdescQK =
      make_idesc(kTF32 ? kFmtTF32 : kFmtBF16, kTF32 ? kFmtTF32 : kFmtBF16, kM, kN, kMajorK, kMajorK);
  static constexpr uint32_t kIdescPV = make_idesc(kTF32 ? kFmtTF32 : kFmtBF16,
                                                  kTF32 ? kFmtTF32 : kFmtBF16, kM, D, kMajorK,
                                                  kTF32 ? kMajorK : kMajorMN);
};

// Last global query position of the 128-row query tile at local row q0.
__device__ __forceinline__ int tile_q_hi(const FlashParams& p, int q0) {
  return global_pos(q0, p.rank, p.Sq, p.world, p.zigzag) + kM - 1;
}

// kCausal: causal launch.  Its work items reach the MMA and softmax roles
// through the in-CTA queue (claimed from the dynamic counter when p.dynamic,
// else from the static list), and tiles are classified against the mask.  A
// non-causal instantiation has no classification at all and every role walks
// the CTA's static (or balanced) list itself.
template <Prec P, int D, bool kCausal>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ FlashParams p, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV) {
  using C = Cfg<P, D>;
  constexpr int kN = C::kN;
  constexpr int NS = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + NS * C::kKTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kSmemTiles);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + NS;
  uint64_t* v_full = bars + 2 * NS;
  uint64_t* v_empty = bars + 3 * NS;
  uint64_t* s_full = bars + 4 * NS;       // [2]
  uint64_t* p_full = bars + 4 * NS + 2;   // [2]
  uint64_t* pv_done = bars + 4 * NS + 4;
  uint64_t* q_full = bars + 4 * NS + 5;
  uint64_t* o_final = bars + 4 * NS + 6;
  uint64_t* drain = bars + 4 * NS + 7;
  uint64_t* xbar = bars + 4 * NS + 8;   // [2] row-max exchange between the softmax halves
  uint64_t* lbar = bars + 4 * NS + 10;  // [2] row-sum exchange
  uint64_t* item_full = bars + 4 * NS + 12;                 // [kItemSlots] work-item queue
  uint64_t* item_empty = bars + 4 * NS + 12 + kItemSlots;  // [kItemSlots]
  __shared__ uint32_t tmem_slot;
  __shared__ int s_copy_ok;
  __shared__ float s_xmax[2][2][kM];  // [tile parity][half][row] partial row maxima
  __shared__ float s_xl[2][2][kM];    // [item parity][half][row] partial row sums
  __shared__ int s_work[kWorkWords];  // this CTA's work description (work_setup)
  __shared__ Item s_items[kItemSlots];  // work-item queue: TMA thread -> MMA and softmax roles

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  DeviceStatus* st = p.status;
  const uint64_t tmo = p.timeout_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 8);  // one arrival per softmax warp
    mbar_init(&p_full[1], 8);
    mbar_init(pv_done, 1);
    mbar_init(q_full, 8);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&xbar[i], 256);
      mbar_init(&lbar[i], 256);
    }
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 1 + 8);  // the MMA thread + one lane per softmax warp
    }
    fence_barrier_init();
  }
  const int tpb = p.Skv / kN;                 // tiles per block
  const int tiles_total = p.nblk * tpb;
  if (threadIdx.x == 32) work_setup(p, tiles_total, s_work);
  if (warp == kWarpMma) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == kWarpTma) {
    // ------------------------------------------------------------------ TMA
    if (elect_one()) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      trace_stamp(p, 0, 0, globaltimer_ns());
      int g = 0;
      int ready_blocks = 1;  // blocks [0, ready_blocks) known present locally
      bool ok = true;
      for (int w = 0; ok; ++w) {
        Item it;
        if constexpr (kCausal) {
          // take item w and publish it (or the end marker) to the MMA and softmax roles
          const int slot = w % kItemSlots;
          if (w >= kItemSlots) {
            ok = mbar_wait(&item_empty[slot], ((w / kItemSlots) - 1) & 1, st, kSiteItemQueue, tmo);
            if (!ok) break;
          }
          bool have;
          if (p.dynamic) {
            have = claim_item(p, tiles_total, &it);
          } else {
            have = w < s_work[0];
            if (have) it = work_item(p, w, tiles_total, s_work);
          }
          if (!have) it.unit = -1;
          s_items[slot] = it;
          mbar_arrive(&item_full[slot]);
          if (!have) break;
        } else {
          if (w >= s_work[0]) break;
          it = work_item(p, w, tiles_total, s_work);
        }
        TileWalk<kN> wk;
        int v = it.v_begin;
        bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, tile_q_hi(p, it.q0))
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
          uint8_t* kdst = sK + stage * C::kKTile;
          if constexpr (C::kTF32) {
#pragma unroll
            for (int ds = 0; ds < D / C::kElems128; ++ds)
              tma_load_5d(kdst + ds * (2 * kN * 128), &tmK, &k_full[stage], ds * C::kElems128,
                          it.hk, t * kN, 0, s);
          } else {
#pragma unroll
            for (int ds = 0; ds < D / C::kElems128; ++ds)
              tma_load_4d(kdst + ds * (kN * 128), &tmK, &k_full[stage], ds * C::kElems128, it.hk,
                          t * kN, s);
          }
          ok = mbar_wait(&v_empty[stage], ph ^ 1, st, kSiteVEmpty, tmo);
          if (!ok) break;
          mbar_arrive_expect_tx(&v_full[stage], C::kVTile);
          uint8_t* vdst = sV + stage * C::kVTile;
          if constexpr (C::kTF32) {
#pragma unroll
            for (int ks = 0; ks < kN / C::kElems128; ++ks)
              tma_load_5d(vdst + ks * (2 * D * 128), &tmV, &v_full[stage],
                          t * kN + ks * C::kElems128, 0, it.hk, 0, s);
          } else {
#pragma unroll
            for (int ds = 0; ds < D / C::kElems128; ++ds)
              tma_load_4d(vdst + ds * (kN * 128), &tmV, &v_full[stage], ds * C::kElems128, it.hk,
                          t * kN, s);
          }
          ++g;
        }
      }
      trace_stamp(p, 0, 1, globaltimer_ns());
      if (!ok) {
        // drain the loads this thread issued before giving up
        for (int i = 0; i < NS && i < g; ++i) {
          const int gg = g - 1 - i;
          const int stage = gg % NS;
          const uint32_t ph = (gg / NS) & 1;
          mbar_wait(&k_full[stage], ph, nullptr, kSiteKFull, 100000000ull);
          mbar_wait(&v_full[stage], ph, nullptr, kSiteVFull, 100000000ull);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------------ MMA
    if (elect_one()) {
      int g = 0;
      int item_count = 0;
      int final_count = 0;  // items that had at least one visible tile
      bool ok = true;
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
          if (w >= s_work[0]) break;
          it = work_item(p, w, tiles_total, s_work);
        }
        ok = mbar_wait(q_full, item_count & 1, st, kSiteQFull, tmo);
        if (!ok) break;
        tc_fence_after();
        int j = 0;
        auto issue_pv = [&](int gp, bool first) -> bool {
          const int b = gp & 1;
          const int stage = gp % NS;
          if (!mbar_wait(&p_full[b], (gp >> 1) & 1, st, kSitePFull, tmo)) return false;
          if (!mbar_wait(&v_full[stage], (gp / NS) & 1, st, kSiteVFull, tmo)) return false;
          tc_fence_after();
          const uint32_t vbase = smem_u32(sV + stage * C::kVTile);
          const uint32_t d_tm = tmem + C::kColO;
          if constexpr (C::kTF32) {
            const uint32_t pb = tmem + (b ? C::kColS1 : C::kColS0);
            const uint32_t ps = tmem + (b ? C::kColPs1 : C::kColPs0);
            // passes: (Ps, Vb), (Pb, Vs), (Pb, Vb); V^T planes: b at +0, s at +D*128
#pragma unroll
            for (int pass = 0; pass < 3; ++pass) {
              const uint32_t a_col = pass == 0 ? ps : pb;
              const uint32_t plane = pass == 1 ? D * 128 : 0;
#pragma unroll
              for (int ks = 0; ks < C::kKStepsPV; ++ks) {
                const uint32_t sub = ks >> 2, inner = (ks & 3) * 32;
                const uint64_t bdesc =
                    make_sdesc(vbase + sub * (2 * D * 128) + plane + inner, 16, 1024);
                const uint32_t acc = (first && pass == 0 && ks == 0) ? 0u : 1u;
                mma_ts<true>(d_tm, a_col + ks * 8, bdesc, C::kIdescPV, acc);
              }
            }
          } else {
            const uint32_t pa = tmem + (b ? C::kColS1 : C::kColS0);
#pragma unroll
            for (int ks = 0; ks < C::kKStepsPV; ++ks) {
              // MN-major V: 16 keys (2 x 8-row atoms) per step; 64-wide d blocks at LBO
              const uint64_t bdesc = make_sdesc(vbase + ks * 2048, kN * 128, 1024);
              const uint32_t acc = (first && ks == 0) ? 0u : 1u;
              mma_ts<false>(d_tm, pa + ks * 8, bdesc, C::kIdescPV, acc);
            }
          }
          mma_commit(&v_empty[stage]);
          mma_commit(pv_done);
          return true;
        };
        TileWalk<kN> wk;
        int v = it.v_begin;
        bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, tile_q_hi(p, it.q0))
                            : v < it.v_end;
        for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
          const int stage = g % NS;
          const int b = g & 1;
          ok = mbar_wait(&k_full[stage], (g / NS) & 1, st, kSiteKFull, tmo);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kbase = smem_u32(sK + stage * C::kKTile);
          const uint32_t s_tm = tmem + (b ? C::kColS1 : C::kColS0);
          if constexpr (C::kTF32) {
            // passes: (Qs, Kb), (Qb, Ks), (Qb, Kb); K planes: b at +0, s at +kN*128
#pragma unroll
            for (int pass = 0; pass < 3; ++pass) {
              const uint32_t a_col = tmem + C::kColQ + (pass == 0 ? C::kQCols : 0);
              const uint32_t plane = pass == 1 ? kN * 128 : 0;
#pragma unroll
              for (int ks = 0; ks < C::kKStepsQK; ++ks) {
                const uint32_t sub = ks >> 2, inner = (ks & 3) * 32;
                const uint64_t bdesc =
                    make_sdesc(kbase + sub * (2 * kN * 128) + plane + inner, 16, 1024);
                mma_ts<true>(s_tm, a_col + ks * 8, bdesc, C::kIdescQK,
                             (pass == 0 && ks == 0) ? 0u : 1u);
              }
            }
          } else {
#pragma unroll
            for (int ks = 0; ks < C::kKStepsQK; ++ks) {
              const uint32_t sub = ks >> 2, inner = (ks & 3) * 32;
              const uint64_t bdesc = make_sdesc(kbase + sub * (kN * 128) + inner, 16, 1024);
              mma_ts<false>(s_tm, tmem + C::kColQ + ks * 8, bdesc, C::kIdescQK, ks ? 1u : 0u);
            }
          }
          mma_commit(&s_full[b]);
          mma_commit(&k_empty[stage]);
          if (j > 0) ok = issue_pv(g - 1, j == 1);
          ++j;
          ++g;
        }
        if (ok && j > 0) {
          ok = issue_pv(g - 1, j == 1);
          if (ok) mma_commit(o_final);
          ++final_count;
        }
      }
      // make sure nothing of ours is still running before TMEM is released
      mma_commit(drain);
      mbar_wait(drain, 0, nullptr, kSiteOReady, 1000000000ull);
    }
  } else if (warp == kWarpComm || warp == kWarpComm + 1) {
    // ------------------------------------------------------------ ring copy
    if (p.fused && p.world > 1) ring_copy_role(p, threadIdx.x - kWarpComm * 32, &s_copy_ok);
  } else {
    // -------------------------------------------------------------- softmax
    // Two warpgroups per query tile: warpgroup `half` owns the S (and P)
    // columns [half*kN/2, (half+1)*kN/2) and the Q / O columns
    // [half*D/2, (half+1)*D/2) of all 128 rows.  The row max is exchanged
    // through shared memory each tile; the partial row sums are combined once
    // per work item.  Two softmax warps per SM sub-partition keep the exp /
    // conversion pipe and the tensor pipe busy at the same time.
    constexpr int kHalfN = kN / 2;
    constexpr int kHalfD = D / 2;
    const int sm_t = threadIdx.x - kWarpSoftmax * 32;  // 0..255
    const int half = sm_t >> 7;
    const int row = sm_t & 127;                          // TMEM lane
    const uint32_t lane_base = ((warp & 3) * 32) << 16;
    const float sl2 = p.scale_log2;
    int g = 0;
    int item_count = 0;
    int final_count = 0;
    bool ok = true;
    for (int w = 0; ok; ++w, ++item_count) {
      const int slot = w % kItemSlots;
      Item it;
      if constexpr (kCausal) {
        ok = __all_sync(0xffffffffu, mbar_wait(&item_full[slot], (w / kItemSlots) & 1, st,
                                               kSiteItemQueue, tmo));
        if (!ok) break;
        it = s_items[slot];
        if (it.unit < 0) break;
      } else {
        if (w >= s_work[0]) break;
        it = work_item(p, w, tiles_total, s_work);
      }
      const int qrow = it.q0 + row;
      // (RAB_DEBUG_BOUNDS builds: an out-of-range row is reported and row 0 read instead)
      const bool q_in = st_bounds(st, qrow < p.Sq && it.h < p.Hq, kBoundsQRow, qrow);
      const size_t q_off = q_in ? (static_cast<size_t>(qrow) * p.Hq + it.h) * D : 0;
      // ---- this warpgroup's half of the Q row -> TMEM ----
      {
        if constexpr (C::kTF32) {
          const float4* qp = reinterpret_cast<const float4*>(
              static_cast<const float*>(p.q) + q_off + half * kHalfD);
          uint32_t big[32], small[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 x = __ldg(qp + i);
            split_tf32_alu(x.x, big[4 * i + 0], small[4 * i + 0]);
            split_tf32_alu(x.y, big[4 * i + 1], small[4 * i + 1]);
            split_tf32_alu(x.z, big[4 * i + 2], small[4 * i + 2]);
            split_tf32_alu(x.w, big[4 * i + 3], small[4 * i + 3]);
          }
          tmem_st32(tmem + lane_base + C::kColQ + half * kHalfD, big);
          tmem_st32(tmem + lane_base + C::kColQ + C::kQCols + half * kHalfD, small);
        } else {
          constexpr int kQc = D / 4;  // packed bf16 columns per warpgroup
          const uint4* qp = reinterpret_cast<const uint4*>(
              static_cast<const uint16_t*>(p.q) + q_off + half * kHalfD);
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < kQc / 4; ++i) {
            const uint4 x = __ldg(qp + i);
            w[4 * i + 0] = x.x;
            w[4 * i + 1] = x.y;
            w[4 * i + 2] = x.z;
            w[4 * i + 3] = x.w;
          }
          if constexpr (kQc == 32)
            tmem_st32(tmem + lane_base + C::kColQ + half * kQc, w);
          else
            tmem_st16(tmem + lane_base + C::kColQ + half * kQc, w);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();  // the warp's TMEM stores are complete and fenced
        if (lane == 0) mbar_arrive(q_full);
      }
      float m_run = -INFINITY;  // running max of scaled log2 scores (same in both halves)
      float l_part = 0.f;       // this half's share of the row sum
      int j = 0;
      const int q_lo = kCausal ? global_pos(it.q0, p.rank, p.Sq, p.world, p.zigzag) : 0;
      TileWalk<kN> wk;
      int v = it.v_begin;
      bool more = kCausal ? wk.begin(p, it.v_begin, it.v_end, q_lo + kM - 1)
                          : v < it.v_end;
      for (; more && ok; more = kCausal ? wk.next(p) : ++v < it.v_end) {
        int k_lo = 0;
        int cls = 1;
        if constexpr (kCausal) {
          // visible (the walk skips masked tiles): full or cut by the diagonal
          k_lo = wk.k_lo;
          cls = k_lo + kN - 1 <= q_lo ? 1 : 2;
        }
        const int b = g & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (g >> 1) & 1, st, kSiteSFull, tmo));
        if (!ok) break;
        tc_fence_after();
        const uint32_t s_tm = tmem + lane_base + (b ? C::kColS1 : C::kColS0);
        uint32_t sr[kHalfN];
#pragma unroll
        for (int c = 0; c < kHalfN; c += 32) tmem_ld32(s_tm + half * kHalfN + c, sr + c);
        tmem_ld_wait();
        if (cls == 2) {
          const int lim = q_lo + row - k_lo - half * kHalfN;  // column c visible iff c <= lim
#pragma unroll
          for (int c = 0; c < kHalfN; ++c)
            if (c > lim) sr[c] = 0xff800000u;  // -inf
        }
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = __uint_as_float(sr[i]);
#pragma unroll
        for (int c = 8; c < kHalfN; ++c) pm[c & 7] = fmaxf(pm[c & 7], __uint_as_float(sr[c]));
        const float mx_part = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                                    fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        s_xmax[g & 1][half][row] = mx_part;
        // bounded exchange (an mbarrier, not bar.sync): if the other half gave
        // up on an error this wait runs out instead of hanging
        mbar_arrive(&xbar[g & 1]);
        ok = __all_sync(0xffffffffu, mbar_wait(&xbar[g & 1], (g >> 1) & 1, st, kSiteSFull, tmo));
        if (!ok) break;
        const float mx = fmaxf(mx_part, s_xmax[g & 1][half ^ 1][row]) * sl2;
        // lazy rescale: move the reference max only when it grows by > 2^8
        // (both halves see the same mx and m_run, so they decide alike)
        const bool need = mx > m_run + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - mx);
          m_run = mx;
          l_part *= alpha;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O holds PV of earlier tiles: wait until the last PV landed, then scale rows
          ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (g - 1) & 1, st, kSitePvDone, tmo));
          if (!ok) break;
          tc_fence_after();
          const uint32_t o_tm = tmem + lane_base + C::kColO + half * kHalfD;
#pragma unroll
          for (int c = 0; c < kHalfD; c += 32) {
            uint32_t o[32];
            tmem_ld32(o_tm + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(o_tm + c, o);
          }
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        if constexpr (C::kTF32) {
          float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // partial row sums
          uint32_t pb[32], psm[32];
#pragma unroll
          for (int c = 0; c < kHalfN; c += 32) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float e = ex2_approx(fmaf(__uint_as_float(sr[c + i]), sl2, -m_use));
              ps8[i & 7] += e;
              split_tf32_alu(e, pb[i], psm[i]);
            }
            tmem_st32(s_tm + half * kHalfN + c, pb);
            tmem_st32(tmem + lane_base + (b ? C::kColPs1 : C::kColPs0) + half * kHalfN + c, psm);
          }
          l_part += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
        } else {
          // four partial sums: the bf16 d=128 instance sits at the 168-register cap
          float ps4[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < kHalfN; c += 64) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float e0 = ex2_approx(fmaf(__uint_as_float(sr[c + 2 * i]), sl2, -m_use));
              const float e1 = ex2_approx(fmaf(__uint_as_float(sr[c + 2 * i + 1]), sl2, -m_use));
              ps4[i & 3] += e0 + e1;
              pk[i] = pack_bf16x2(e0, e1);
            }
            tmem_st32(s_tm + (half * kHalfN + c) / 2, pk);
          }
          l_part += (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
        ++j;
        ++g;
      }
      if (!ok) break;
      // ---- combine the two halves' row sums ----
      s_xl[item_count & 1][half][row] = l_part;
      mbar_arrive(&lbar[item_count & 1]);
      ok = __all_sync(0xffffffffu, mbar_wait(&lbar[item_count & 1], (item_count >> 1) & 1, st,
                                             kSiteOReady, tmo));
      if (!ok) break;
      const float l_run = l_part + s_xl[item_count & 1][half ^ 1][row];
      // ---- epilogue: this half's columns of O ----
      const bool have = j > 0;
      if (have) {
        ok = __all_sync(0xffffffffu, mbar_wait(o_final, final_count & 1, st, kSiteOReady, tmo));
        ++final_count;
        if (!ok) break;
        tc_fence_after();
      }
      const uint32_t o_tm = tmem + lane_base + C::kColO + half * kHalfD;
      const float m_nat = have ? m_run * kLn2 : -INFINITY;
      // re-read here (queue slot or shared-memory work list) rather than kept live
      // across the tile loop
      const Item ie = kCausal ? s_items[slot] : work_item(p, w, tiles_total, s_work);
      const size_t r = static_cast<size_t>(ie.q0 + row) * p.Hq + ie.h;
      const bool split = ie.store >= 0;
      // (RAB_DEBUG_BOUNDS builds: an out-of-range row or record is reported, its stores skipped)
      const bool out_in = st_bounds(
          st, ie.q0 + row < p.Sq && ie.h < p.Hq &&
                  (!split || ie.store < (p.balanced ? 2 * p.n_items : p.n_items)),
          split ? kBoundsRecord : kBoundsQRow, split ? ie.store : ie.q0 + row);
      const float inv = (have && l_run > 0.f && !p.partial && !split) ? 1.f / l_run : 1.f;
      float* dst_f32 = nullptr;
      if (split)
        dst_f32 = p.split_acc + (static_cast<size_t>(ie.store) * kM + row) * D + half * kHalfD;
      else if (p.partial)
        dst_f32 = p.acc + r * D + half * kHalfD;
      else if (!p.out_bf16)
        dst_f32 = static_cast<float*>(p.out) + r * D + half * kHalfD;
#pragma unroll
      for (int c = 0; c < kHalfD; c += 32) {
        uint32_t o[32];
        if (have) {
          tmem_ld32(o_tm + c, o);
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
          uint4* d4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + r * D +
                                               half * kHalfD + c);
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
      if (half == 0 && out_in) {
        if (split) {
          p.split_m[static_cast<size_t>(ie.store) * kM + row] = m_nat;
          p.split_l[static_cast<size_t>(ie.store) * kM + row] = l_run;
        } else if (p.partial) {
          if (p.m_out) p.m_out[r] = m_nat;
          if (p.l_out) p.l_out[r] = l_run;
        } else if (p.lse != nullptr) {
          p.lse[r] = (have && l_run > 0.f) ? m_nat + logf(l_run) : -INFINITY;
        }
      }
      // all TMEM reads of this item are done before the next Q lands in TMEM
      tc_fence_before();
      if constexpr (kCausal) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&item_empty[slot]);  // queue slot free again
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (kCausal && p.dynamic && threadIdx.x == 0) {
    // Every CTA has stopped claiming items once it gets here; the last one
    // resets the claim counter for the next launch that uses this status block.
    __threadfence();
    if (atomicAdd(&st->pad[1], 1u) == gridDim.x - 1) {
      atomicExch(&st->pad[0], 0u);
      atomicExch(&st->pad[1], 0u);
    }
  }
  if (threadIdx.x == 0) finish_launch(p);  // device-side epochs: bump the call counter
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// split merge: combine the partial records of a unit
// ---------------------------------------------------------------------------
// Final (or partial-mode) write of merged row `row` of `unit`, column quad c.
template <int D>
__device__ __forceinline__ void write_merged(const FlashParams& p, int unit, int row, int c,
                                             float mx, float l, float4 a) {
  const int h = unit_head(p, unit);
  const int qrow = unit_q0(p, unit) + row;
  if (!st_bounds(p.status, qrow < p.Sq && h < p.Hq, kBoundsQRow, qrow)) return;
  const size_t r = static_cast<size_t>(qrow) * p.Hq + h;
  if (p.partial) {
    reinterpret_cast<float4*>(p.acc + r * D)[c] = a;
    if (c == 0) {
      if (p.m_out) p.m_out[r] = mx;
      if (p.l_out) p.l_out[r] = l;
    }
    return;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  a.x *= inv;
  a.y *= inv;
  a.z *= inv;
  a.w *= inv;
  if (p.out_bf16) {
    uint2 pk;
    pk.x = pack_bf16x2(a.x, a.y);
    pk.y = pack_bf16x2(a.z, a.w);
    reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + r * D)[c] = pk;
  } else {
    reinterpret_cast<float4*>(static_cast<float*>(p.out) + r * D)[c] = a;
  }
  if (c == 0 && p.lse != nullptr) p.lse[r] = l > 0.f ? mx + logf(l) : -INFINITY;
}

// Accumulate record `rec` of R rows (row `row`, column quad c) into the running
// merge relative to the reference max `mref`.
template <int D>
__device__ __forceinline__ void add_record(const FlashParams& p, size_t rec, int R, int row, int c,
                                           float mref, float& l, float4& a) {
  const size_t n_rec = p.balanced ? 2 * static_cast<size_t>(p.n_items) : p.n_items;
  if (!st_bounds(p.status, rec < n_rec, kBoundsMergeRecord, static_cast<uint32_t>(rec))) return;
  const float mk = p.split_m[rec * R + row];
  const float w = (mk == -INFINITY) ? 0.f : expf(mk - mref);
  l += w * p.split_l[rec * R + row];
  const float4 x = reinterpret_cast<const float4*>(p.split_acc + (rec * R + row) * D)[c];
  a.x += w * x.x;
  a.y += w * x.y;
  a.z += w * x.z;
  a.w += w * x.w;
}

// Equal-split schedule: unit u has records k * n_units + u, k < nsplit.
template <int D>
__global__ void split_merge_kernel(const FlashParams p) {
  constexpr int kTpr = D / 4;
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const int R = p.rows_per_unit;
  const long long rows_total = static_cast<long long>(p.n_units) * R;
  const long long urow = t / kTpr;
  const int c = static_cast<int>(t % kTpr);
  if (urow >= rows_total) return;
  const int unit = static_cast<int>(urow / R);
  const int row = static_cast<int>(urow % R);
  float mx = -INFINITY;
  for (int k = 0; k < p.nsplit; ++k)
    mx = fmaxf(mx, p.split_m[(static_cast<size_t>(k) * p.n_units + unit) * R + row]);
  const float mref = (mx == -INFINITY) ? 0.f : mx;
  float l = 0.f;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < p.nsplit; ++k)
    add_record<D>(p, static_cast<size_t>(k) * p.n_units + unit, R, row, c, mref, l, a);
  write_merged<D>(p, unit, row, c, mx, l, a);
}

// Balanced schedule: blockIdx.x = unit - full_waves * G over the units of the
// shared-out remainder, blockIdx.y = the block's kBalMergeRows rows of it.  CTA c of G owns the tiles
// [c*T/G, (c+1)*T/G), so the CTAs whose ranges meet the unit's tiles
// [u0, u1) are c_lo = owner(u0) .. c_hi = owner(u1 - 1), owner(x) =
// floor(((x + 1) G - 1) / T) (the last CTA whose range starts at or before
// x).  A unit inside one CTA's range was written whole by that CTA; otherwise
// the pieces are merged from record 2c (the unit holds the first tile of CTA
// c's range) or 2c + 1 (it holds its last) of each of those CTAs.
constexpr int kBalMergeRows = 16;  // rows of a unit per block (blockIdx.y picks them)
constexpr int kBalMaxPieces = 16;

template <int D>
__global__ void balanced_merge_kernel(const FlashParams p) {
  constexpr int kTpr = D / 4;
  const int G = p.n_items;
  const long long tt = p.kv_tiles;
  const int base = p.full_waves * G;
  const long long T = static_cast<long long>(p.n_units - base) * tt;
  const long long u0 = static_cast<long long>(blockIdx.x) * tt;
  const long long u1 = u0 + tt;
  const int c_lo = static_cast<int>(((u0 + 1) * G - 1) / T);
  const int c_hi = static_cast<int>((u1 * G - 1) / T);
  if (c_lo >= c_hi) return;  // written whole by one CTA
  const int unit = base + static_cast<int>(blockIdx.x);
  // record of the k-th CTA's piece of the unit (-1: empty range)
  auto record = [&](int c) -> long long {
    const long long s_c = balanced_start(T, G, c);
    if (balanced_start(T, G, c + 1) <= s_c) return -1;
    return 2LL * c + (s_c >= u0 ? 0 : 1);
  };
  if (c_hi - c_lo + 1 <= kBalMaxPieces) {
    // the usual case (a unit spans about tt * G / T + 1 CTAs): the records
    // once per block, not inside the row loops
    __shared__ size_t rec[kBalMaxPieces];
    __shared__ int s_n;
    if (threadIdx.x == 0) {
      int k = 0;
      for (int c = c_lo; c <= c_hi; ++c) {
        const long long r = record(c);
        if (r >= 0) rec[k++] = static_cast<size_t>(r);
      }
      s_n = k;
    }
    __syncthreads();
    const int n = s_n;
    for (int q = threadIdx.x; q < kBalMergeRows * kTpr; q += blockDim.x) {
      const int row = blockIdx.y * kBalMergeRows + q / kTpr;
      const int c = q % kTpr;
      float mx = -INFINITY;
      for (int i = 0; i < n; ++i) mx = fmaxf(mx, p.split_m[rec[i] * kM + row]);
      const float mref = (mx == -INFINITY) ? 0.f : mx;
      float l = 0.f;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int i = 0; i < n; ++i) add_record<D>(p, rec[i], kM, row, c, mref, l, a);
      write_merged<D>(p, unit, row, c, mx, l, a);
    }
    return;
  }
  // a unit cut by many CTAs (few units left over for many CTAs)
  for (int q = threadIdx.x; q < kBalMergeRows * kTpr; q += blockDim.x) {
    const int row = blockIdx.y * kBalMergeRows + q / kTpr;
    const int c = q % kTpr;
    float mx = -INFINITY;
    for (int k = c_lo; k <= c_hi; ++k) {
      const long long r = record(k);
      if (r >= 0) mx = fmaxf(mx, p.split_m[static_cast<size_t>(r) * kM + row]);
    }
    const float mref = (mx == -INFINITY) ? 0.f : mx;
    float l = 0.f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = c_lo; k <= c_hi; ++k) {
      const long long r = record(k);
      if (r >= 0) add_record<D>(p, static_cast<size_t>(r), kM, row, c, mref, l, a);
    }
    write_merged<D>(p, unit, row, c, mx, l, a);
  }
}

// ---------------------------------------------------------------------------
// ring-format preparation (3xTF32): K -> planes, V -> transposed planes
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tf32_pair(float x, float& b, float& s) {
  uint32_t bb, ss;
  split_tf32(x, bb, ss);
  b = __uint_as_float(bb);
  s = __uint_as_float(ss);
}

// One launch formats a whole fp32 ring block (the split was two launches; the
// per-step launch gap showed in the step time):
//   blocks [0, n_vt):  V [Skv][Hkv][D] -> V^T planes [2][Hkv][D][Skv], one 32x32
//                      tile each, transposed through shared memory;
//   blocks [n_vt, ..): K [Skv][Hkv][D] -> planes [2][Skv][Hkv][D], float4 grid-stride.
// Block shape (32, 8).
__global__ void __launch_bounds__(256) ring_format_f32_kernel(
    const float4* __restrict__ k, float4* __restrict__ kb, float4* __restrict__ ks, size_t n4,
    const float* __restrict__ v, float* __restrict__ vt, int Skv, int Hkv, int D, int n_vt) {
  if (static_cast<int>(blockIdx.x) < n_vt) {
    __shared__ float tile[32][33];
    const int sx = Skv / 32, dy = D / 32;
    const int hk = blockIdx.x / (sx * dy);
    const int rem = blockIdx.x - hk * (sx * dy);
    const int s0 = (rem % sx) * 32, d0 = (rem / sx) * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y)
      tile[i][threadIdx.x] = v[(static_cast<size_t>(s0 + i) * Hkv + hk) * D + d0 + threadIdx.x];
    __syncthreads();
    const size_t plane = static_cast<size_t>(Hkv) * D * Skv;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      float b, sm;
      tf32_pair(tile[threadIdx.x][i], b, sm);
      const size_t o = (static_cast<size_t>(hk) * D + d0 + i) * Skv + s0 + threadIdx.x;
      vt[o] = b;
      vt[plane + o] = sm;
    }
    return;
  }
  const size_t nb = gridDim.x - n_vt;
  const size_t t = threadIdx.y * 32 + threadIdx.x;
  for (size_t i = (blockIdx.x - n_vt) * static_cast<size_t>(256) + t; i < n4; i += nb * 256) {
    const float4 x = k[i];
    float4 b, sm;
    tf32_pair(x.x, b.x, sm.x);
    tf32_pair(x.y, b.y, sm.y);
    tf32_pair(x.z, b.z, sm.z);
    tf32_pair(x.w, b.w, sm.w);
    kb[i] = b;
    ks[i] = sm;
  }
}

template <Prec P, int D, bool kCausal>
int launch_one(const FlashParams& p, const FlashMaps& maps, int grid, bool cooperative,
               cudaStream_t stream) {
  using C = Cfg<P, D>;
  // the shared-memory opt-in is a per-device function attribute
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaFuncSetAttribute(flash_fwd_kernel<P, D, kCausal>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         C::kSmemBytes);
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  if (cooperative) {
    void* args[] = {const_cast<FlashParams*>(&p), const_cast<CUtensorMap*>(&maps.k),
                    const_cast<CUtensorMap*>(&maps.v)};
    return static_cast<int>(cudaLaunchCooperativeKernel(
        reinterpret_cast<void*>(flash_fwd_kernel<P, D, kCausal>), dim3(grid), dim3(kThreads), args,
        C::kSmemBytes, stream));
  }
  flash_fwd_kernel<P, D, kCausal><<<grid, kThreads, C::kSmemBytes, stream>>>(p, maps.k, maps.v);
  return static_cast<int>(cudaGetLastError());
}

template <Prec P, int D>
int launch_impl(const FlashParams& p, const FlashMaps& maps, int grid, bool cooperative,
                cudaStream_t stream) {
  using C = Cfg<P, D>;
  if (p.Skv % C::kN != 0)
    throw std::runtime_error("flash: keys per block must be a multiple of " +
                             std::to_string(C::kN));
  if (p.dynamic && (p.balanced || !p.causal))
    throw std::runtime_error("flash: the dynamic schedule is for causal equal-split launches");
  return p.causal ? launch_one<P, D, true>(p, maps, grid, cooperative, stream)
                  : launch_one<P, D, false>(p, maps, grid, cooperative, stream);
}

}  // namespace

int flash_sm_count() {
  // per device (a process may drive GPUs of different sizes, or MIG slices);
  // atomic because host threads of the C entry points may call this at once
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int sms = cache[dev].load(std::memory_order_relaxed);
  if (sms == 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0)
      sms = 148;  // B200 (query failed)
    cache[dev].store(sms, std::memory_order_relaxed);
  }
  return sms;
}

size_t ring_v_offset(Prec prec, int Skv, int Hkv, int D) {
  const size_t e = static_cast<size_t>(Skv) * Hkv * D;
  const size_t k_bytes = prec == Prec::kF32x3 ? 2 * e * 4 : e * 2;
  return (k_bytes + 1023) / 1024 * 1024;
}

size_t ring_block_bytes(Prec prec, int Skv, int Hkv, int D) {
  const size_t e = static_cast<size_t>(Skv) * Hkv * D;
  const size_t v_bytes = prec == Prec::kF32x3 ? 2 * e * 4 : e * 2;
  return (ring_v_offset(prec, Skv, Hkv, D) + v_bytes + 4095) / 4096 * 4096;
}

FlashMaps flash_make_maps(Prec prec, const void* k_base, const void* v_base, size_t slot_stride,
                          int nblk, int Skv, int Hkv, int D) {
  FlashMaps m;
  if (slot_stride == 0) slot_stride = ring_block_bytes(prec, Skv, Hkv, D);
  if (prec == Prec::kF32x3) {
    const uint64_t kn = 64;
    {
      uint64_t dims[5] = {(uint64_t)D, (uint64_t)Hkv, (uint64_t)Skv, 2, (uint64_t)nblk};
      uint64_t strides[4] = {(uint64_t)D * 4, (uint64_t)Hkv * D * 4, (uint64_t)Skv * Hkv * D * 4,
                             slot_stride};
      uint32_t box[5] = {32, 1, (uint32_t)kn, 2, 1};
      m.k = make_tmap(k_base, TmapDtype::kF32, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    {
      uint64_t dims[5] = {(uint64_t)Skv, (uint64_t)D, (uint64_t)Hkv, 2, (uint64_t)nblk};
      uint64_t strides[4] = {(uint64_t)Skv * 4, (uint64_t)D * Skv * 4,
                             (uint64_t)Hkv * D * Skv * 4, slot_stride};
      uint32_t box[5] = {32, (uint32_t)D, 1, 2, 1};
      m.v = make_tmap(v_base, TmapDtype::kF32, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
  } else {
    uint64_t dims[4] = {(uint64_t)D, (uint64_t)Hkv, (uint64_t)Skv, (uint64_t)nblk};
    uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)Hkv * D * 2, slot_stride};
    uint32_t box[4] = {64, 1, 128, 1};
    m.k = make_tmap(k_base, TmapDtype::kBF16, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    m.v = make_tmap(v_base, TmapDtype::kBF16, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  return m;
}

int flash_choose_split(int units, int tiles_per_unit, int sms, int overhead_tiles) {
  // Cost model fitted to B200 measurements of the fp32 kernel: a work item
  // costs its KV tiles plus a fixed overhead (pipeline fill and drain, Q
  // staging, epilogue, partial write-back) of about six 64-key tiles, and the
  // persistent grid runs ceil(items / SMs) waves.
  int best = 1;
  double best_cost = 1e300;
  for (int c = 1; c <= 16 && c <= tiles_per_unit; ++c) {
    const long long items = static_cast<long long>(units) * c;
    const long long waves = (items + sms - 1) / sms;
    const double cost = static_cast<double>(waves) *
                        (static_cast<double>(tiles_per_unit) / c + overhead_tiles);
    if (cost < best_cost * 0.995) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

bool flash_prefer_balanced(int units, int tiles_per_unit, int sms, int overhead_tiles) {
  // Balanced: floor(units / G) whole-unit waves, then the remainder's
  // ceil(R * tiles / G) tiles per CTA in at most two pieces, plus the merge
  // pass (about four tiles of either kernel on B200).  It has to beat the best
  // equal split by 2 % to be worth the partial records.
  const long long full = units / sms;
  const long long R = units - full * sms;
  if (R == 0) return false;
  const long long per = (R * tiles_per_unit + sms - 1) / sms;
  const long long pieces = (per + tiles_per_unit - 1) / tiles_per_unit + 1;
  const double bal = static_cast<double>(full * (tiles_per_unit + overhead_tiles) + per +
                                         pieces * overhead_tiles + 4);
  const int c = flash_choose_split(units, tiles_per_unit, sms, overhead_tiles);
  const long long items = static_cast<long long>(units) * c;
  const double split = static_cast<double>((items + sms - 1) / sms) *
                       (static_cast<double>(tiles_per_unit) / c + overhead_tiles);
  return bal < 0.98 * split;
}

int flash_forward_launch(Prec prec, const FlashParams& p, const FlashMaps& maps, int grid,
                         bool cooperative, cudaStream_t stream) {
  if (p.Sq % kM != 0) throw std::runtime_error("flash: query rows must be a multiple of 128");
  if (p.Hq % p.Hkv != 0) throw std::runtime_error("flash: Hq must be a multiple of Hkv");
  if (p.nblk > kMaxSlots) throw std::runtime_error("flash: too many blocks");
  if (p.balanced && (grid != p.n_items || p.causal || p.rows_per_unit != kM ||
                     p.full_waves < 0 || p.full_waves * grid > p.n_units))
    throw std::runtime_error(
        "flash: balanced schedule needs grid == n_items, full_waves * grid <= units and no "
        "causal mask");
  if (p.causal && p.zigzag && (p.Sq != p.Skv || (p.Sq / 2) % kM != 0))
    throw std::runtime_error("flash: zigzag causal needs Sq == Skv and Sq/2 a multiple of 128");
  if (prec == Prec::kF32x3) {
    if (p.D != 64) throw std::runtime_error("flash: fp32 (3xTF32) path supports head_dim 64");
    return launch_impl<Prec::kF32x3, 64>(p, maps, grid, cooperative, stream);
  }
  if (p.D == 64) return launch_impl<Prec::kBF16, 64>(p, maps, grid, cooperative, stream);
  if (p.D == 128) return launch_impl<Prec::kBF16, 128>(p, maps, grid, cooperative, stream);
  throw std::runtime_error("flash: head_dim must be 64 or 128");
}

int flash_split_merge_launch(const FlashParams& p, cudaStream_t stream) {
  if (p.balanced) {
    const int remainder = p.n_units - p.full_waves * p.n_items;  // units shared out
    if (p.n_items < 2 || remainder <= 0) return 0;
    const dim3 grid(remainder, kM / kBalMergeRows);
    const int threads = kBalMergeRows * (p.D / 4);  // one float4 of one row each
    if (p.D == 64)
      balanced_merge_kernel<64><<<grid, threads, 0, stream>>>(p);
    else
      balanced_merge_kernel<128><<<grid, threads, 0, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
  }
  const long long threads_total = static_cast<long long>(p.n_units) * p.rows_per_unit * (p.D / 4);
  const int bs = 256;
  const int blocks = static_cast<int>((threads_total + bs - 1) / bs);
  if (p.D == 64)
    split_merge_kernel<64><<<blocks, bs, 0, stream>>>(p);
  else
    split_merge_kernel<128><<<blocks, bs, 0, stream>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int ring_format_launch(Prec prec, const void* k, const void* v, void* k_dst, void* v_dst, int Skv,
                       int Hkv, int D, cudaStream_t stream) {
  const size_t e = static_cast<size_t>(Skv) * Hkv * D;
  if (prec == Prec::kBF16) {
    cudaError_t err = cudaMemcpyAsync(k_dst, k, e * 2, cudaMemcpyDeviceToDevice, stream);
    if (err == cudaSuccess)
      err = cudaMemcpyAsync(v_dst, v, e * 2, cudaMemcpyDeviceToDevice, stream);
    return static_cast<int>(err);
  }
  if (Skv % 32 != 0 || D % 32 != 0) throw std::runtime_error("ring_format: Skv, D % 32");
  const size_t n4 = e / 4;
  const long long n_vt = static_cast<long long>(Skv / 32) * (D / 32) * Hkv;
  const long long n_k = std::min<long long>((n4 + 255) / 256, 8LL * flash_sm_count());
  if (n_vt + n_k > 0x7fffffffLL) throw std::runtime_error("ring_format: block too large");
  float* kb = static_cast<float*>(k_dst);
  ring_format_f32_kernel<<<static_cast<unsigned>(n_vt + n_k), dim3(32, 8), 0, stream>>>(
      static_cast<const float4*>(k), reinterpret_cast<float4*>(kb),
      reinterpret_cast<float4*>(kb + e), n4, static_cast<const float*>(v),
      static_cast<float*>(v_dst), Skv, Hkv, D, static_cast<int>(n_vt));
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rab
