// flash.h - parameters and host API of the sm_100a flash-attention forward
// kernel, used both per ring step (unfused baselines) and as the fused ring
// kernel (`b200_fused`: K/V blocks of the other ranks are pulled over NVLink
// from inside the kernel while the tensor cores work on the blocks already
// present).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <utility>
#include <vector>

#include "host_comm.h"
#include "status.h"

namespace rab {

enum class Prec : int {
  kBF16 = 0,   // bf16 Q/K/V, fp32 accumulation (kind::f16)
  kF32x3 = 1,  // fp32 Q/K/V, 3xTF32 split products (kind::tf32), fp32-level accuracy
};

// Flag words (uint64) at the start of each rank's arena used by the fused kernel.
enum FusedFlag : int {
  kFlagSlot0Ready = 0,  // epoch whose slot-0 block is published
  kFlagReads = 1,       // slices of this rank's slots read by peers (cumulative)
  kFlagCalls = 2,       // device-side epochs: launches completed by this engine
  kFlagExit = 3,        // device-side epochs: CTAs of the running launch that finished
  kFlagArrivedBase = 8, // + s: slices of slot s landed locally (cumulative)
  kMaxSlots = 64,
};

struct FlashParams {
  // ---- queries ----
  const void* q;        // [Sq, Hq, D] bf16 or fp32
  int Sq, Hq, Hkv, D;
  float scale_log2;     // softmax scale * log2(e)
  // ---- key/value blocks (ring slots), described by the tensor maps ----
  int nblk;             // blocks to attend to, in ring order (block s from rank - s)
  int Skv;              // keys per block
  // ---- masking ----
  int causal;           // 0/1
  int zigzag;           // 1: rank r holds global chunks r and 2W-1-r; 0: contiguous shards
  int world, rank;
  int blk_offset;       // block s holds the keys of rank (rank - blk_offset - s) mod world
  // ---- work split ----
  int nsplit;           // KV chunks per (head, q tile) unit (equal-split schedule)
  int balanced;         // 1: balanced schedule: full_waves waves of whole units, then the
                        //    remaining units' (unit, KV tile) space shared out evenly, CTA c
                        //    owning tiles [c*T/G, (c+1)*T/G); needs causal == 0, 128-row units
  int full_waves;       // balanced: whole-unit waves before the shared-out remainder
  int dynamic;          // 1: CTAs claim equal-split items from a counter in the status block
  int kv_tiles;         // KV tiles of one unit over the whole ring (nblk * Skv / tile keys)
  int rows_per_unit;    // query rows of one work unit (128, or 256 for the two-tile bf16 kernel)
  int n_units;          // heads * Sq / rows_per_unit
  int n_items;          // n_units * nsplit; balanced: the number of CTAs G
  // ---- outputs ----
  void* out;            // final O [Sq, Hq, D] (nsplit == 1 and !partial)
  int out_bf16;
  float* lse;           // [Sq, Hq] natural-log LSE (optional)
  int partial;          // 1: write unnormalised acc + natural-log m + l (reference partial semantics)
  float* acc;           // partial acc [Sq, Hq, D]     (partial, nsplit == 1)
  float* m_out;         // partial m [Sq, Hq]
  float* l_out;         // partial l [Sq, Hq]
  float* split_acc;     // nsplit > 1: [n_items][128][D]; balanced: [2 * G][128][D]
  float* split_m;       // [records][128] (natural log)
  float* split_l;       // [records][128]
  // ---- fused ring transfer ----
  int fused;            // 1: copy blocks 1..nblk-1 from peers inside the kernel
  int ring_chain;       // 0: pull block s from its origin's slot 0; 1: from the left neighbour's slot s-1
  uint8_t* local_slots;               // this rank's slot 0 (slot s at + s * slot_bytes)
  const uint8_t* peer_slots[kMaxRanks];  // every rank's slot 0 (peer-mapped)
  uint64_t* flags_local;
  uint64_t* flags_peer[kMaxRanks];
  size_t slot_bytes;    // bytes of one ring-format block
  uint64_t epoch;
  uint64_t arrive_target;  // value of flag kFlagArrivedBase+s once this launch copied slot s
  uint64_t reads_target;   // value of kFlagReads once every peer finished this launch's reads
  // Device-side epochs (nullptr: epoch and targets above, set by the host per
  // launch): this launch's epoch is *call_counter + 1, the targets follow from
  // it and the grid, and the launch's last CTA to finish bumps the counter, so
  // the launch parameters stay the same from call to call (a captured CUDA
  // graph can replay them).  Points at flag word kFlagCalls; kFlagExit follows.
  uint64_t* call_counter;
  // ---- diagnostics ----
  DeviceStatus* status;
  uint64_t timeout_ns;
  // optional overlap trace, [grid][kMaxSlots][2] globaltimer ns per CTA:
  // [c][0] = (TMA role start, TMA role end), [c][s] = (first wait for ring
  // block s, block s present); nullptr: off
  uint64_t* stamps;
};

// Host side: tensor maps for the K/V slots.  For kBF16 the slots hold K and V
// as [Skv, Hkv, D] bf16 each (V read MN-major by the MMA).  For kF32x3 a slot
// holds K as two tf32 planes [2][Skv][Hkv][D] and V transposed as two planes
// [2][Hkv][D][Skv] (both K-major for the MMA).
struct FlashMaps {
  CUtensorMap k;
  CUtensorMap v;
};

// Build tensor maps over `nblk` consecutive slots starting at `k_base` /
// `v_base` with `slot_stride` bytes between slots (0 for a single block).
FlashMaps flash_make_maps(Prec prec, const void* k_base, const void* v_base, size_t slot_stride,
                          int nblk, int Skv, int Hkv, int D);

// Pick nsplit for `units` work units of `tiles_per_unit` KV tiles on `sms` SMs,
// with a fixed per-item overhead equivalent to `overhead_tiles` tiles.
int flash_choose_split(int units, int tiles_per_unit, int sms, int overhead_tiles);

// True when the balanced schedule is expected to beat the best equal split
// (same cost model; only valid without a causal mask).
bool flash_prefer_balanced(int units, int tiles_per_unit, int sms, int overhead_tiles);

int flash_forward_launch(Prec prec, const FlashParams& p, const FlashMaps& maps, int grid,
                         bool cooperative, cudaStream_t stream);

// Two-query-tile bf16 kernel (256-row work units); q map from flash_make_q_map.
CUtensorMap flash_make_q_map(const void* q, int Sq, int Hq, int D);
int flash_forward_2q_launch(const FlashParams& p, const CUtensorMap& tmq, const FlashMaps& maps,
                            int grid, bool cooperative, cudaStream_t stream);

// bf16 d=128 kernel on CTA pairs (clusters of two, tcgen05 cta_group::2):
// 512-row work units; each CTA loads half of every K/V tile.  k_base/v_base
// and slot_stride describe the ring slots as for flash_make_maps.  `grid` must
// be even and at most flash_pair_max_grid() when every CTA has to be resident
// (fused mode).
int flash_forward_2sm_launch(const FlashParams& p, const CUtensorMap& tq, const void* k_base,
                             const void* v_base, size_t slot_stride, int grid, bool cooperative,
                             cudaStream_t stream);
int flash_pair_max_grid();  // CTAs (an even number) of the pairs resident at once

// Merge the split partials (nsplit > 1: every unit; balanced: the units a CTA
// boundary cuts) into the final output (and LSE), or into acc/m/l when partial.
int flash_split_merge_launch(const FlashParams& p, cudaStream_t stream);

// Ring-format preparation of one block: kF32x3 -> tf32 planes, V transposed.
// kBF16 -> plain copy (skipped by callers when the data already sits in the slot).
int ring_format_launch(Prec prec, const void* k, const void* v, void* k_dst, void* v_dst, int Skv,
                       int Hkv, int D, cudaStream_t stream);

size_t ring_block_bytes(Prec prec, int Skv, int Hkv, int D);  // K + V bytes of one slot
size_t ring_v_offset(Prec prec, int Skv, int Hkv, int D);     // V offset inside a slot

int flash_sm_count();

}  // namespace rab

namespace rab {

// Everything one forward call needs, in raw pointers.  Shared by the torch
// bindings and the native benchmark drivers.
struct FlashArgs {
  Prec prec = Prec::kBF16;
  const void* q = nullptr;
  int Sq = 0, Hq = 1, Hkv = 1, D = 64;
  float scale = 1.f;                 // softmax scale (natural units)
  const void* k_base = nullptr;      // ring-format K of block 0
  const void* v_base = nullptr;      // ring-format V of block 0
  size_t slot_stride = 0;            // bytes between consecutive blocks
  int nblk = 1, Skv = 0;
  int causal = 0, zigzag = 0, world = 1, rank = 0;
  int blk_offset = 0;                // first block is ring step blk_offset
  void* out = nullptr;
  bool out_bf16 = false;
  float* lse = nullptr;
  bool partial = false;
  float* acc = nullptr;
  float* m = nullptr;
  float* l = nullptr;
  int nsplit = 0;                    // > 0: equal split; 0: choose; -1: balanced schedule
  void* workspace = nullptr;         // split partials (see flash_workspace_bytes)
  size_t workspace_bytes = 0;
  int grid = 0;                      // <= 0: min(items, SMs)
  int sms = 0;                       // > 0: plan for this many SMs (default: the current device's)
  DeviceStatus* status = nullptr;
  double timeout_s = 10.0;
  // fused ring transfer
  bool fused = false;
  bool ring_chain = false;
  uint8_t* local_slots = nullptr;
  const uint8_t* peer_slots[kMaxRanks] = {};
  uint64_t* flags_local = nullptr;
  uint64_t* flags_peer[kMaxRanks] = {};
  size_t slot_bytes = 0;
  uint64_t epoch = 0;
  uint64_t arrive_target = 0;
  uint64_t reads_target = 0;
  uint64_t* call_counter = nullptr;  // device-side epochs (FlashParams::call_counter)
  uint64_t* stamps = nullptr;        // optional overlap trace (FlashParams::stamps)
};

struct FlashPlan {
  int rows_per_unit;  // 128 (one query tile per CTA), 256 (two-tile bf16 kernel) or
                      // 512 (bf16 d=128 kernel on CTA pairs)
  int nsplit;         // equal-split chunks per unit; 1 under the balanced schedule
  int balanced;       // 1: balanced schedule (n_items == grid == CTAs)
  int full_waves;     // balanced: whole-unit waves before the shared-out remainder
  int dynamic;        // 1: dynamic claiming of equal-split items (causal launches)
  int n_units;
  int n_items;
  int grid;
  int merge_kernel;   // 1: a merge launch follows the attention kernel (split records)
  size_t workspace_bytes;
};

FlashPlan flash_plan(const FlashArgs& a);

// Visible KV tiles of the 128-row query tile at local row q0 under the causal
// mask, as [begin, end) ranges of ring tile indices (the planner's closed form).
std::vector<std::pair<int, int>> flash_visible_ranges(const FlashArgs& a, int q0);
int flash_run(const FlashArgs& a, const FlashPlan& plan, cudaStream_t stream);

}  // namespace rab
