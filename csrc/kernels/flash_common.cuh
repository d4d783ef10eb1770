// flash_common.cuh - pieces shared by the sm_100a flash-attention kernels:
// work-item decomposition, causal tile classification by global position, the
// cross-GPU flag primitives and the in-kernel ring copy role of the fused mode.
#pragma once

#include <cstdint>

#include "flash.h"
#include "sm100.cuh"

namespace rab {
namespace flash_detail {

using namespace sm100;

constexpr int kM = 128;                    // rows of one query tile (TMEM lanes)
constexpr float kRescaleThreshold = 8.0f;  // lazy rescale threshold, log2 units
constexpr float kLn2 = 0.69314718055994530942f;

// One work item: query tile `unit` (head h, first row q0) against the ring's
// KV tiles [v_begin, v_end).  `store` is the index of the split partial record
// the item writes (split_acc / split_m / split_l), or -1 when the item covers
// every KV tile of its unit and writes the final result itself.
struct Item {
  int unit, h, hk, q0, v_begin, v_end, store;
};

// First query row of a work unit.  Units run head-major (all query tiles of a
// head, then the next head), so the CTAs of one wave share a head's K/V in L2.
// With a causal mask the later query tiles see more keys; they are handed out
// first (longest-processing-time-first shortens the tail of the schedule).
__device__ __forceinline__ int unit_q0(const FlashParams& p, int unit) {
  const int per_head = p.Sq / p.rows_per_unit;
  const int qt = unit % per_head;
  return (p.causal ? (per_head - 1 - qt) : qt) * p.rows_per_unit;
}

__device__ __forceinline__ int unit_head(const FlashParams& p, int unit) {
  return unit / (p.Sq / p.rows_per_unit);
}

__device__ __forceinline__ void set_unit(const FlashParams& p, int unit, Item& it) {
  it.unit = unit;
  it.h = unit_head(p, unit);
  it.hk = it.h / (p.Hq / p.Hkv);
  it.q0 = unit_q0(p, unit);
}

// Equal-split schedule: item = chunk * n_units + unit, chunk in [0, nsplit).
__device__ __forceinline__ Item make_item(const FlashParams& p, int item, int tiles_total) {
  Item it;
  const int chunk = item / p.n_units;
  set_unit(p, item - chunk * p.n_units, it);
  it.v_begin = static_cast<int>(static_cast<long long>(chunk) * tiles_total / p.nsplit);
  it.v_end = static_cast<int>(static_cast<long long>(chunk + 1) * tiles_total / p.nsplit);
  it.store = p.nsplit > 1 ? item : -1;
  return it;
}

// Balanced schedule (every KV tile costs the same, i.e. no causal mask).  The
// first full_waves * G units run whole, unit blockIdx.x + k * G in wave k (the
// head-major order of the equal-split schedule, which keeps the CTAs of a
// wave on the same heads' K/V in L2).  The remaining R < G units are shared
// out evenly: CTA c of G owns the tiles [c*T/G, (c+1)*T/G) of their (unit,
// KV tile) space, T = R * tiles_total, cut at unit boundaries into pieces.  A
// piece that is not a whole unit writes split record 2c (the piece holding
// the range's first tile) or 2c+1 (the one holding its last tile), and
// balanced_merge_kernel combines the records of each unit a CTA boundary cuts.
__device__ __forceinline__ long long balanced_start(long long T, int G, int c) {
  return static_cast<long long>(c) * T / G;
}

// Per-CTA work description, computed once by one thread into shared memory:
// [0] work items, [1] whole-unit waves, [2] pieces n, [3] first piece's unit,
// [4] rotation (1: the leading piece runs last), [5] first tile of the leading
// piece, [6] end tile of the last piece.
constexpr int kWorkWords = 7;

__device__ __forceinline__ void work_setup(const FlashParams& p, int tiles_total, int* sw) {
  if (!p.balanced) {
    sw[0] = blockIdx.x < p.n_items ? (p.n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    return;
  }
  const int G = gridDim.x;
  const int base = p.full_waves * G;
  const long long T = static_cast<long long>(p.n_units - base) * tiles_total;
  const long long s = balanced_start(T, G, blockIdx.x);
  const long long e = balanced_start(T, G, blockIdx.x + 1);
  sw[1] = p.full_waves;
  if (e <= s) {
    sw[0] = p.full_waves;
    sw[2] = 0;
    return;
  }
  const int u_lo = static_cast<int>(s / tiles_total);
  const int u_hi = static_cast<int>((e - 1) / tiles_total);
  sw[2] = u_hi - u_lo + 1;
  sw[0] = p.full_waves + sw[2];
  sw[3] = base + u_lo;
  sw[4] = (u_hi > u_lo && s % tiles_total != 0) ? 1 : 0;
  sw[5] = static_cast<int>(s - static_cast<long long>(u_lo) * tiles_total);
  sw[6] = static_cast<int>(e - static_cast<long long>(u_hi) * tiles_total);
}

// Depth of the shared-memory queue through which the TMA thread hands work
// items to the MMA and softmax roles.
constexpr int kItemSlots = 4;

// The k-th of this CTA's sw[0] work items.  In the balanced schedule the
// whole units come first; among the pieces a leading one that starts inside
// its unit runs last: in the fused ring its tiles lie in the ring blocks that
// arrive last, while every other piece starts at block 0.
__device__ __forceinline__ Item work_item(const FlashParams& p, int k, int tiles_total,
                                          const int* sw) {
  if (!p.balanced) return make_item(p, blockIdx.x + k * gridDim.x, tiles_total);
  Item it;
  if (k < sw[1]) {
    set_unit(p, blockIdx.x + k * gridDim.x, it);
    it.v_begin = 0;
    it.v_end = tiles_total;
    it.store = -1;
    return it;
  }
  const int n = sw[2];
  const int idx = (k - sw[1] + sw[4]) % n;
  set_unit(p, sw[3] + idx, it);
  it.v_begin = idx == 0 ? sw[5] : 0;
  it.v_end = idx == n - 1 ? sw[6] : tiles_total;
  const bool whole = it.v_begin == 0 && it.v_end == tiles_total;
  it.store = whole ? -1 : 2 * static_cast<int>(blockIdx.x) + (idx == 0 ? 0 : 1);
  return it;
}

// Dynamic schedule (p.dynamic): claim the next unclaimed equal-split item of
// the whole grid from a counter in the status block (pad[0]); false once all
// are taken.  A CTA that drew cheap items (short causal query tiles) takes
// more of them, and since items are claimed in order, the cheap tail of the
// longest-first unit order balances the end of the schedule.
__device__ __forceinline__ bool claim_item(const FlashParams& p, int tiles_total, Item* it) {
  const uint32_t i = atomicAdd(&p.status->pad[0], 1u);
  if (i >= static_cast<uint32_t>(p.n_items)) return false;
  *it = make_item(p, static_cast<int>(i), tiles_total);
  return true;
}

__device__ __forceinline__ int global_pos(int local, int owner, int S, int W, int zigzag) {
  if (!zigzag) return owner * S + local;
  const int C = S >> 1;
  return local < C ? owner * C + local : (2 * W - 1 - owner) * C + (local - C);
}

// Tile classification for the 128-row query tile starting at local row q0:
// 0 = skip (fully masked), 1 = full, 2 = diagonal (mask per element).
// On 0, *v_io moves to the last tile of v's key chunk: keys grow along each
// contiguous chunk of a ring block (the whole block, or each half under
// zigzag sharding), so every later tile of the chunk is masked as well and a
// loop over v continues after it.
__device__ __forceinline__ int classify(const FlashParams& p, int q0, int* v_io, int kN, int tpb,
                                        int* k_lo_out, int* q_lo_out) {
  if (!p.causal) return 1;
  const int v = *v_io;
  const int s = v / tpb, t = v - (v / tpb) * tpb;
  const int owner = ((p.rank - p.blk_offset - s) % p.world + p.world) % p.world;
  const int q_lo = global_pos(q0, p.rank, p.Sq, p.world, p.zigzag);
  const int q_hi = q_lo + kM - 1;
  const int k_lo = global_pos(t * kN, owner, p.Skv, p.world, p.zigzag);
  const int k_hi = k_lo + kN - 1;
  *k_lo_out = k_lo;
  *q_lo_out = q_lo;
  if (k_lo > q_hi) {
    const int chunk = p.zigzag ? tpb / 2 : tpb;
    *v_io = s * tpb + (t / chunk + 1) * chunk - 1;
    return 0;
  }
  if (k_hi <= q_lo) return 1;
  return 2;
}

// Causal walk over the KV tiles [v_begin, v_end) of a work item that a query
// range ending at global position q_hi can see, in ring order, with the first
// global key position of each tile.  Keys grow along each contiguous chunk of
// a ring block (the whole block, or each half under zigzag sharding), so the
// visible tiles of a chunk are a prefix of it: the walk steps tile by tile
// with one compare and jumps to the next chunk at the first masked tile.  The
// owner of a block (a modulo) is computed once per block, not per tile.
// Every role of a CTA walks the same sequence.
template <int kN>
struct TileWalk {
  int v, v_end;   // current tile (ring tile index) and end of the range
  int k_lo;       // first global key position of tile v
  int t;          // tile within its block
  int chunk_end;  // tile (within the block) where the current chunk ends
  int q_hi;       // last global query position the walk serves
  // (tiles per block, p.Skv / kN, is recomputed where needed: one register
  // fewer in the softmax, which runs at its register cap)

  // position the walk at tile `v_new` (no visibility check)
  __device__ __forceinline__ void seek(const FlashParams& p, int v_new) {
    v = v_new;
    if (v >= v_end) return;
    const int tpb = p.Skv / kN;
    const int s = v / tpb;
    t = v - s * tpb;
    const int tpc = p.zigzag ? tpb / 2 : tpb;
    const int c = t >= tpc ? 1 : 0;
    const int owner = ((p.rank - p.blk_offset - s) % p.world + p.world) % p.world;
    k_lo = global_pos(c * tpc * kN, owner, p.Skv, p.world, p.zigzag) + (t - c * tpc) * kN;
    chunk_end = (c + 1) * tpc;
  }
  // skip masked tiles from the current one (the rest of their chunk); false
  // at the end of the range
  __device__ __forceinline__ bool settle(const FlashParams& p) {
    while (v < v_end && k_lo > q_hi) seek(p, v - t + chunk_end);
    return v < v_end;
  }
  __device__ __forceinline__ bool begin(const FlashParams& p, int v_begin, int v_end_, int q_hi_) {
    v_end = v_end_;
    q_hi = q_hi_;
    seek(p, v_begin);
    return settle(p);
  }
  // advance to the next visible tile; false at the end of the range
  __device__ __forceinline__ bool next(const FlashParams& p) {
    ++v;
    ++t;
    if (v >= v_end) return false;
    if (t == chunk_end)
      seek(p, v);  // next chunk or next block
    else
      k_lo += kN;
    return settle(p);
  }
};

__device__ __forceinline__ uint64_t ld_acquire_gpu(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded poll of a 64-bit flag until it reaches `target`.
__device__ __forceinline__ bool wait_flag(const uint64_t* flag, uint64_t target, bool sys,
                                          DeviceStatus* st, uint32_t where, uint32_t detail,
                                          uint64_t timeout_ns) {
  if ((sys ? ld_acquire_sys(flag) : ld_acquire_gpu(flag)) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if ((sys ? ld_acquire_sys(flag) : ld_acquire_gpu(flag)) >= target) return true;
    if (st_read_error(st) != 0) return false;
    if (globaltimer_ns() - t0 > timeout_ns) {
      st_record_timeout(st, where, detail);
      return false;
    }
  }
}

// Overlap trace (p.stamps != nullptr): see FlashParams::stamps.
__device__ __forceinline__ void trace_stamp(const FlashParams& p, int slot, int which,
                                            uint64_t t) {
  if (p.stamps != nullptr)
    p.stamps[(static_cast<size_t>(blockIdx.x) * kMaxSlots + slot) * 2 + which] = t;
}

// Epoch of this launch and the cumulative flag values it waits for: from the
// launch parameters, or (device-side epochs) from the engine's call counter,
// which only the previous launch's last CTA wrote.  Every launch of an engine
// has the same grid: each CTA adds one slice per ring block to the arrival
// flags, and every peer reads one slice per CTA of this rank's slot 0.
struct RingTargets {
  uint64_t epoch, arrive, reads;
};

__device__ __forceinline__ RingTargets ring_targets(const FlashParams& p) {
  if (p.call_counter == nullptr) return {p.epoch, p.arrive_target, p.reads_target};
  const uint64_t e = *reinterpret_cast<volatile const uint64_t*>(p.call_counter) + 1;
  return {e, e * gridDim.x, e * static_cast<uint64_t>(p.world - 1) * gridDim.x};
}

// Device-side epochs: called by one thread of every CTA after the CTA's last
// use of the epoch; the last CTA of the launch to get here bumps the call
// counter for the next launch and clears the exit count.
__device__ __forceinline__ void finish_launch(const FlashParams& p) {
  if (p.call_counter == nullptr) return;
  unsigned long long* exits = reinterpret_cast<unsigned long long*>(p.call_counter + 1);
  __threadfence();
  if (atomicAdd(exits, 1ull) == gridDim.x - 1) {
    atomicExch(exits, 0ull);
    atomicAdd(reinterpret_cast<unsigned long long*>(p.call_counter), 1ull);
    __threadfence();
  }
}

// The TMA thread's wait for ring block s to be present locally (fused mode),
// with the overlap trace.
__device__ __forceinline__ bool wait_block(const FlashParams& p, int s) {
  const uint64_t t0 = p.stamps != nullptr ? globaltimer_ns() : 0;
  const bool ok = wait_flag(p.flags_local + kFlagArrivedBase + s, ring_targets(p).arrive, false,
                            p.status, kSiteBlockReady, s, p.timeout_ns);
  if (p.stamps != nullptr) {
    trace_stamp(p, s, 0, t0);
    trace_stamp(p, s, 1, globaltimer_ns());
  }
  return ok;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// The fused mode's copy role, run by 64 threads (two warps) of every CTA:
// slice blockIdx.x of every ring block 1..nblk-1 is pulled from peer memory
// into this rank's slot; see FlashParams for the flag protocol.  `s_copy_ok`
// is a shared word that makes each go / no-go decision uniform across the 64
// threads before the named barrier they share.
__device__ __forceinline__ void ring_copy_role(const FlashParams& p, int ct, int* s_copy_ok) {
  DeviceStatus* st = p.status;
  const uint64_t tmo = p.timeout_ns;
  const RingTargets tg = ring_targets(p);
  if (blockIdx.x == 0 && ct == 0) st_release_sys(p.flags_local + kFlagSlot0Ready, tg.epoch);
  const int left = (p.rank - 1 + p.world) % p.world;
  const size_t n16 = p.slot_bytes / 16;
  const size_t per = (n16 + gridDim.x - 1) / gridDim.x;
  const size_t beg = per * blockIdx.x;
  const size_t end = beg + per < n16 ? beg + per : n16;
  bool ok = true;
  for (int s = 1; s < p.nblk && ok; ++s) {
    const uint4* src;
    uint64_t* src_flags;
    if (p.ring_chain) {
      src = reinterpret_cast<const uint4*>(p.peer_slots[left] + (size_t)(s - 1) * p.slot_bytes);
      src_flags = p.flags_peer[left];
    } else {
      const int origin = ((p.rank - s) % p.world + p.world) % p.world;
      src = reinterpret_cast<const uint4*>(p.peer_slots[origin]);
      src_flags = p.flags_peer[origin];
    }
    if (ct == 0) {
      bool w;
      if (p.ring_chain && s > 1)
        w = wait_flag(src_flags + kFlagArrivedBase + (s - 1), tg.arrive, true, st,
                      kSitePeerReady, s, tmo);
      else
        w = wait_flag(src_flags + kFlagSlot0Ready, tg.epoch, true, st, kSitePeerReady, s, tmo);
      *s_copy_ok = (w && st_read_error(st) == 0) ? 1 : 0;
    }
    named_bar_sync(1, 64);
    ok = *s_copy_ok != 0;  // one decision for all 64 copy threads
    if (!ok) break;
    uint4* dst = reinterpret_cast<uint4*>(p.local_slots + (size_t)s * p.slot_bytes);
    size_t i = beg + ct;
    constexpr int U = 8;
    for (; i + (U - 1) * 64 < end; i += U * 64) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) r[u] = __ldcg(src + i + u * 64);
#pragma unroll
      for (int u = 0; u < U; ++u) __stcg(dst + i + u * 64, r[u]);
    }
    for (; i < end; i += 64) __stcg(dst + i, __ldcg(src + i));
    fence_proxy_async_global();
    __threadfence_system();
    named_bar_sync(1, 64);
    if (ct == 0) {
      red_add_release_sys(p.flags_local + kFlagArrivedBase + s, 1);
      red_add_release_sys(src_flags + kFlagReads, 1);
    }
  }
  // this rank's slots must outlive every peer's reads of this launch
  if (ok && blockIdx.x == 0 && ct == 0)
    wait_flag(p.flags_local + kFlagReads, tg.reads, true, st, kSitePeerConsumed, 0, tmo);
}

}  // namespace flash_detail
}  // namespace rab
