// flash_host.cpp - host planning of the flash forward: work split, grid,
// workspace and cached tensor maps.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <queue>
#include <stdexcept>
#include <tuple>
#include <utility>
#include <vector>

#include "flash.h"

namespace rab {

namespace {

using MapKey = std::tuple<int, const void*, const void*, size_t, int, int, int, int, int>;

const FlashMaps& cached_maps(Prec prec, const void* k, const void* v, size_t stride, int nblk,
                             int Skv, int Hkv, int D) {
  static std::mutex mu;
  static std::map<MapKey, FlashMaps> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key{static_cast<int>(prec), k, v, stride, nblk, Skv, Hkv, D, dev};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cache.size() > 256) cache.clear();
  return cache.emplace(key, flash_make_maps(prec, k, v, stride, nblk, Skv, Hkv, D)).first->second;
}

// Dynamic claiming of work items (causal one-tile launches) is on unless
// RAB_FLASH_DYNAMIC=0.
bool dynamic_enabled() {
  const char* e = std::getenv("RAB_FLASH_DYNAMIC");
  return e == nullptr || std::strcmp(e, "0") != 0;
}

// Two-query-tile bf16 kernel: RAB_FLASH_2Q=1 forces it (where the query rows
// split into 256-row units), RAB_FLASH_2Q=0 disables it.  By default every
// causal bf16 launch uses it, and a non-causal one when its 256-row units fill
// at least two waves of the GPU (measured on B200: 4-10 % above the one-tile
// kernel there); small non-causal problems keep the one-tile kernel's
// balanced schedule.
bool use_two_tile(const FlashArgs& a, int sms) {
  if (a.prec != Prec::kBF16 || a.Sq % 256 != 0 || a.nsplit < 0) return false;
  const char* e = std::getenv("RAB_FLASH_2Q");
  if (e != nullptr && std::strcmp(e, "1") == 0) return true;
  if (e != nullptr && std::strcmp(e, "0") == 0) return false;
  // causal: measured on B200 (16k tokens x 32 heads d=128: 900 vs 796 TFLOP/s; 64k GQA:
  // 1013 vs 882), its dynamic claiming keeps small problems balanced
  return a.causal || static_cast<long long>(a.Hq) * (a.Sq / 256) >= 2LL * sms;
}

// CTA-pair kernel (bf16, d = 128, 512-row units): RAB_FLASH_2SM=1 selects it
// where the shape allows it (and =0 never does).
bool use_pair(const FlashArgs& a) {
  if (a.prec != Prec::kBF16 || a.D != 128 || a.Sq % 512 != 0 || a.Skv % 128 != 0) return false;
  if (a.causal && a.zigzag && (a.Sq / 2) % 512 != 0) return false;
  if (a.nsplit < 0) return false;  // the balanced schedule is one-tile only
  const char* e = std::getenv("RAB_FLASH_2SM");
  return e != nullptr && std::strcmp(e, "1") == 0;
}

// Visible KV tiles of the 128-row query tile at local row q0, as ranges of
// ring tile indices: keys grow along each contiguous chunk of a ring block
// (the whole block, or each half under zigzag), so each chunk contributes the
// run of tiles from its start up to the last one whose first key is <= the
// tile's last query position (the same rule as the kernel's classify()).
std::vector<std::pair<int, int>> visible_ranges(const FlashArgs& a, int kN, int q0) {
  auto gpos = [&](int local, int owner, int S) -> long long {
    if (!a.zigzag) return static_cast<long long>(owner) * S + local;
    const int Ch = S / 2;
    return local < Ch ? static_cast<long long>(owner) * Ch + local
                      : static_cast<long long>(2 * a.world - 1 - owner) * Ch + (local - Ch);
  };
  const long long q_hi = gpos(q0, a.rank, a.Sq) + 127;
  const int tpb = a.Skv / kN;
  const int chunks = a.zigzag ? 2 : 1;
  const int tpc = tpb / chunks;
  std::vector<std::pair<int, int>> r;
  for (int s = 0; s < a.nblk; ++s) {
    const int owner = ((a.rank - a.blk_offset - s) % a.world + a.world) % a.world;
    for (int c = 0; c < chunks; ++c) {
      const long long k0 = gpos(c * tpc * kN, owner, a.Skv);
      if (k0 > q_hi) continue;
      const long long n = std::min<long long>((q_hi - k0) / kN + 1, tpc);
      const int beg = s * tpb + c * tpc;
      r.emplace_back(beg, beg + static_cast<int>(n));
    }
  }
  return r;
}

// Fused ring launches: the copy warps pull the other ranks' blocks in ring
// order, block s landing about s copy intervals after the launch.  Measured on
// B200 with 8 ranks: 268 MB bf16 blocks every 0.9 ms (~300 GB/s per GPU while
// the tensor cores run).  The tile time converts that interval into the
// planner's unit, one 128-row x kN-key tile on one SM, at the kernels'
// measured rates (two-tile bf16 ~1.1 PFLOP/s, 3xTF32 ~0.24 PFLOP/s per GPU).
constexpr double kRingCopyBytesPerS = 300e9;
constexpr double kHbmBytesPerS = 6.5e12;

double tile_seconds(const FlashArgs& a, int kN, int sms) {
  const double rate = a.prec == Prec::kF32x3 ? 0.24e15 : 1.1e15;
  return 4.0 * 128 * kN * a.D / (rate / sms);
}

// nsplit by simulation, for a causal launch with dynamic claiming and for any
// fused ring launch of several blocks: simulate the CTAs claiming items in
// kernel order (chunk-major, then head-major units, under a causal mask with
// the last query tiles first) and keep the split with the shortest makespan.
// A unit of `rows` query rows works on every KV tile visible to its last
// 128-row tile (every tile without a mask), once per 128-row tile; an item
// costs that work plus `overhead`, and a split adds one merge pass.  (The
// non-causal static order hands equal items round-robin, which the claim
// simulation reproduces.)  In a fused ring launch an item walks its chunk's ring
// blocks in order and cannot start on block s before the block has landed, so
// every CTA would wait for each block in turn when all items span the whole
// ring; a split whose chunks follow the blocks lets the early items run on the
// blocks already present.  There the merge pass is charged by its traffic
// (every split's partial records read once).
int simulated_split(const FlashArgs& a, int kN, int rows, int units, int tiles, int sms,
                    int overhead) {
  static std::mutex mu;
  static std::map<std::vector<long long>, int> cache;
  const std::vector<long long> key{a.Sq,     a.Skv,    a.nblk, a.Hq,  a.Hkv, a.D,
                                   a.world,  a.rank,   a.blk_offset, a.zigzag, a.fused ? 1 : 0,
                                   a.causal,
                                   static_cast<long long>(a.prec), kN, rows, sms, overhead};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int per_head = a.Sq / rows;
  const int weight = rows / 128;
  std::vector<std::vector<std::pair<int, int>>> vis(per_head);
  const int tpb = tiles / std::max(1, a.nblk);
  for (int qt = 0; qt < per_head; ++qt) {
    if (a.causal) {
      vis[qt] = visible_ranges(a, kN, qt * rows + rows - 128);
    } else {
      for (int s = 0; s < a.nblk; ++s) vis[qt].emplace_back(s * tpb, (s + 1) * tpb);
    }
  }
  // fused ring: arrival of block s, and the merge pass per split, in tile units
  const bool ring = a.fused && a.nblk > 1;
  double interval = 0.0, merge_per_split = 0.0;
  if (ring) {
    const double tile_s = tile_seconds(a, kN, sms);
    interval = static_cast<double>(ring_block_bytes(a.prec, a.Skv, a.Hkv, a.D)) /
               kRingCopyBytesPerS / tile_s;
    merge_per_split = static_cast<double>(a.Sq) * a.Hq * (a.D + 2) * 4 / kHbmBytesPerS / tile_s;
  }
  int best = 1;
  double best_span = 1e300;
  for (int ns = 1; ns <= 16 && ns <= tiles; ++ns) {
    const long long items = static_cast<long long>(units) * ns;
    const int G = static_cast<int>(std::min<long long>(items, sms));
    std::priority_queue<double, std::vector<double>, std::greater<double>> load;
    for (int i = 0; i < G; ++i) load.push(0.0);
    double span = 0.0;
    for (int c = 0; c < ns; ++c) {
      const int vb = static_cast<int>(static_cast<long long>(c) * tiles / ns);
      const int ve = static_cast<int>(static_cast<long long>(c + 1) * tiles / ns);
      for (int u = 0; u < units; ++u) {
        const int qt = per_head - 1 - u % per_head;  // the kernel's unit order
        double t = load.top();
        for (const auto& r : vis[qt]) {  // ranges lie inside one ring block, in ring order
          const int n = std::max(0, std::min(r.second, ve) - std::max(r.first, vb));
          if (n == 0) continue;
          if (ring) t = std::max(t, (r.first / tpb) * interval);
          t += static_cast<double>(weight) * n;
        }
        t += overhead;
        load.pop();
        load.push(t);
        span = std::max(span, t);
      }
    }
    if (ns > 1) span += ring ? 4 + ns * merge_per_split : 4;  // merge pass
    if (span < best_span * 0.995) {
      best_span = span;
      best = ns;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 256) cache.clear();
  cache[key] = best;
  return best;
}

int tiles_of(const FlashArgs& a) { return a.nblk * (a.Skv / (a.prec == Prec::kF32x3 ? 64 : 128)); }

}  // namespace

std::vector<std::pair<int, int>> flash_visible_ranges(const FlashArgs& a, int q0) {
  return visible_ranges(a, a.prec == Prec::kF32x3 ? 64 : 128, q0);
}

FlashPlan flash_plan(const FlashArgs& a) {
  if (a.Sq <= 0 || a.Sq % 128 != 0) throw std::runtime_error("flash: Sq must be a positive multiple of 128");
  FlashPlan pl{};
  const int sm_total = a.sms > 0 ? a.sms : flash_sm_count();
  const bool pair = use_pair(a);
  // the pair kernel's workers are CTA pairs (as many as are resident at once)
  const int pair_grid = pair ? (a.sms > 0 ? (a.sms / 2) * 2 : flash_pair_max_grid()) : 0;
  const int sms = pair ? pair_grid / 2 : sm_total;
  // bf16 may use the two-query-tile kernel when the rows split into 256-row units
  pl.rows_per_unit = pair ? 512 : (use_two_tile(a, sms) ? 256 : 128);
  pl.n_units = a.Hq * (a.Sq / pl.rows_per_unit);
  const int tiles = tiles_of(a);
  // per-item overhead in tiles: ~6 of the fp32 kernel's 64-key tiles, ~3 of 128-key bf16 tiles
  const int overhead = a.prec == Prec::kF32x3 ? 6 : 3;
  // the balanced schedule needs equal-cost tiles (no causal mask) and 128-row units
  const bool can_balance = !a.causal && pl.rows_per_unit == 128;
  if (a.nsplit < 0 && !can_balance)
    throw std::runtime_error("flash: the balanced schedule needs causal=0 and 128-row units");
  pl.balanced = (a.nsplit < 0 ||
                 (a.nsplit == 0 && can_balance &&
                  flash_prefer_balanced(pl.n_units, tiles, sms, overhead)))
                    ? 1
                    : 0;
  if (pl.balanced) {
    pl.nsplit = 1;
    pl.grid = a.grid > 0 ? a.grid : sms;
    pl.n_items = pl.grid;  // one balanced range per CTA
    pl.full_waves = pl.n_units / pl.grid;
    pl.merge_kernel = 1;
    pl.workspace_bytes = static_cast<size_t>(2 * pl.grid) * 128 * (a.D + 2) * sizeof(float);
    return pl;
  }
  const bool dyn = a.causal && dynamic_enabled();
  if (a.nsplit > 0)
    pl.nsplit = a.nsplit;
  else if (dyn || (a.fused && a.nblk > 1))
    pl.nsplit = simulated_split(a, a.prec == Prec::kF32x3 ? 64 : 128, pl.rows_per_unit,
                                pl.n_units, tiles, sms, overhead);
  else
    pl.nsplit = flash_choose_split(pl.n_units, tiles, sms, overhead);
  if (pl.nsplit > tiles) pl.nsplit = tiles > 0 ? tiles : 1;
  pl.n_items = pl.n_units * pl.nsplit;
  pl.grid = a.grid > 0 ? a.grid : std::min(pl.n_items, sms);
  if (a.fused) pl.grid = a.grid > 0 ? a.grid : sms;  // every CTA also copies a slice
  if (pair) pl.grid = 2 * (a.fused ? sms : std::min(pl.n_items, sms));  // two CTAs per worker
  pl.merge_kernel = pl.nsplit > 1 ? 1 : 0;
  pl.workspace_bytes = pl.nsplit > 1 ? static_cast<size_t>(pl.n_items) * pl.rows_per_unit *
                                           (a.D + 2) * sizeof(float)
                                     : 0;
  // causal items differ in cost: claim them dynamically
  pl.dynamic = dyn ? 1 : 0;
  return pl;
}

int flash_run(const FlashArgs& a, const FlashPlan& pl, cudaStream_t stream) {
  const bool records = pl.nsplit > 1 || pl.balanced;
  if (records && (a.workspace == nullptr || a.workspace_bytes < pl.workspace_bytes))
    throw std::runtime_error("flash: split workspace missing or too small");
  FlashParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = a.q;
  p.Sq = a.Sq;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.D = a.D;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.nblk = a.nblk;
  p.Skv = a.Skv;
  p.causal = a.causal;
  p.zigzag = a.zigzag;
  p.world = a.world;
  p.rank = a.rank;
  p.blk_offset = a.blk_offset;
  p.nsplit = pl.nsplit;
  p.balanced = pl.balanced;
  p.full_waves = pl.balanced ? pl.full_waves : 0;
  p.dynamic = pl.dynamic;
  p.kv_tiles = tiles_of(a);
  p.rows_per_unit = pl.rows_per_unit;
  p.n_units = pl.n_units;
  p.n_items = pl.n_items;
  p.out = a.out;
  p.out_bf16 = a.out_bf16 ? 1 : 0;
  p.lse = a.lse;
  p.partial = a.partial ? 1 : 0;
  p.acc = a.acc;
  p.m_out = a.m;
  p.l_out = a.l;
  if (records) {
    // nsplit > 1: one record per item; balanced: two per CTA (n_items == CTAs)
    const size_t rec_rows =
        static_cast<size_t>(pl.balanced ? 2 * pl.n_items : pl.n_items) * pl.rows_per_unit;
    float* ws = static_cast<float*>(a.workspace);
    p.split_acc = ws;
    p.split_m = ws + rec_rows * a.D;
    p.split_l = p.split_m + rec_rows;
  }
  p.fused = a.fused ? 1 : 0;
  p.ring_chain = a.ring_chain ? 1 : 0;
  p.local_slots = a.local_slots;
  for (int r = 0; r < kMaxRanks; ++r) {
    p.peer_slots[r] = a.peer_slots[r];
    p.flags_peer[r] = a.flags_peer[r];
  }
  p.flags_local = a.flags_local;
  p.slot_bytes = a.slot_bytes;
  p.epoch = a.epoch;
  p.arrive_target = a.arrive_target;
  p.reads_target = a.reads_target;
  p.call_counter = a.fused ? a.call_counter : nullptr;
  p.status = a.status;
  p.timeout_ns = static_cast<uint64_t>(a.timeout_s * 1e9);
  p.stamps = a.stamps;
  if (p.status == nullptr) throw std::runtime_error("flash: a device status word is required");
  const FlashMaps& maps =
      cached_maps(a.prec, a.k_base, a.v_base, a.slot_stride, a.nblk, a.Skv, a.Hkv, a.D);
  int err;
  if (pl.rows_per_unit == 512) {
    const CUtensorMap tq = flash_make_q_map(a.q, a.Sq, a.Hq, a.D);
    err = flash_forward_2sm_launch(p, tq, a.k_base, a.v_base, a.slot_stride, pl.grid, a.fused,
                                   stream);
  } else if (pl.rows_per_unit == 256) {
    const CUtensorMap tq = flash_make_q_map(a.q, a.Sq, a.Hq, a.D);
    err = flash_forward_2q_launch(p, tq, maps, pl.grid, a.fused, stream);
  } else {
    err = flash_forward_launch(a.prec, p, maps, pl.grid, a.fused, stream);
  }
  if (err != 0) return err;
  if (records && pl.merge_kernel) err = flash_split_merge_launch(p, stream);
  return err;
}

}  // namespace rab
