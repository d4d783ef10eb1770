// drivers.h - native benchmark drivers: the comm-only ring loop and the ring
// attention schedules of the reference benchmark, re-expressed on the native
// runtime (RingContext), plus the fused `b200_fused` backend.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "flash.h"
#include "ring_context.h"

namespace rab {

// Flag-word layout (uint64 indices into RingContext::flags_*) besides the
// fused-attention words of flash.h (0..71).
enum RuntimeFlag : int {
  kFlagRingArrived = 1024,  // [kMaxSlices] comm-only ring: slices landed
  kFlagRingSent = 2048,     // [kMaxSlices] comm-only ring: slices sent
  kMaxSlices = 512,
};

struct RingCopyParams {
  uint8_t* buf[2];          // this rank's two shard buffers
  uint8_t* right_buf[2];    // the right neighbour's two buffers (peer-mapped)
  uint8_t* left_buf[2];     // the left neighbour's two buffers (peer-mapped; pull mode)
  uint64_t* arrived_local;  // [slices] written by the left neighbour
  uint64_t* arrived_right;  // the right neighbour's arrived[] (peer-mapped)
  uint64_t* sent_local;     // [slices] this rank's progress
  uint64_t* sent_right;     // the right neighbour's sent[] (peer-mapped)
  uint64_t* sent_left;      // the left neighbour's sent[] (peer-mapped; pull mode)
  size_t bytes;
  int nsteps;
  int first_step;           // ring step index of this launch's first step (buffer parity)
  uint64_t base;            // steps completed by earlier launches
  DeviceStatus* status;
  uint64_t timeout_ns;
  int mode;                 // 0: 16-byte vector stores, 1: TMA bulk copies through shared
                            // memory, 2: 32-byte vector loads and stores, 3: pull (16-byte
                            // loads of the left neighbour's buffer, local stores)
};
int p2p_ring_launch(const RingCopyParams& p, int slices, cudaStream_t stream);

// ---------------------------------------------------------------------------
// comm-only ring (reference: src/loop/ring_loop_<backend>.cu)
// ---------------------------------------------------------------------------
struct CommOptions {
  std::string backend;   // staged | staged_Isendrecv | cuda_aware | cuda_aware_Isendrecv | nccl | b200_fused
  size_t bytes = 262144;
  int warmup = 10;
  int iters = 100;
  int slices = 0;        // b200_fused CTAs (0: default)
  int p2p_mode = 0;      // b200_fused copy engine: 0 vector stores, 1 TMA bulk, 2 32-byte vectors,
                         // 3 pull
  bool precheck = true;
};

// Averages over `iters` timed repetitions of the per-rank maxima (ms), the
// same reduction as the reference (MPI_Reduce(MAX) per repetition, then mean).
struct CommResult {
  std::map<std::string, double> avg_ms;  // d2h, mpi, h2d, nccl, p2p, total
  bool precheck_ok = true;
  std::string precheck_msg;
};

CommResult run_comm_bench(RingContext& ctx, const CommOptions& opt);

// Buffers the comm bench needs in the symmetric arena.
size_t comm_arena_bytes(size_t bytes);

// ---------------------------------------------------------------------------
// FusedRing: the `b200_fused` ring attention engine.  Owns `world` ring slots
// in the symmetric arena; forward() formats the local K/V into slot 0 and
// launches one persistent kernel that pulls the other ranks' blocks over
// NVLink into slots 1..world-1 while it computes, keeping the online-softmax
// state on chip across the whole ring.
// ---------------------------------------------------------------------------
class FusedRing {
 public:
  // device_epochs: the fused kernel takes its epoch from a call counter in
  // device memory instead of the launch parameters, so a call's launches are
  // the same every time and can be captured in a CUDA graph and replayed
  // (every rank must replay in step: each replay is one ring call).
  FusedRing(RingContext& ctx, Prec prec, int seq, int heads, int heads_kv, int dim, bool causal,
            bool zigzag, bool ring_chain, double timeout_s, bool device_epochs = false);
  ~FusedRing();
  FusedRing(const FusedRing&) = delete;
  FusedRing& operator=(const FusedRing&) = delete;

  static size_t arena_bytes(Prec prec, int seq, int heads_kv, int dim, int world);

  // q [seq, heads, dim]; k, v [seq, heads_kv, dim] (bf16 or fp32 per `prec`);
  // out [seq, heads, dim] (fp32 or bf16); lse [seq, heads] (optional).  When
  // `k` already points at slot 0 (see slot0_k) the formatting copy is skipped.
  void forward(const void* q, const void* k, const void* v, void* out, bool out_bf16, float* lse,
               float scale, cudaStream_t stream);
  // Split for timing: prepare() formats slot 0, attend() runs the fused kernel.
  void prepare(const void* k, const void* v, cudaStream_t stream);
  void attend(const void* q, void* out, bool out_bf16, float* lse, float scale,
              cudaStream_t stream);
  // Reads (and clears) the device status word; throws RankFailure after a timeout.
  void check();
  uint8_t* slot0_k() const;  // bf16: raw K layout; write inputs here to skip the copy
  uint8_t* slot0_v() const;
  int grid() const { return plan_.grid; }
  int nsplit() const { return plan_.balanced ? -1 : plan_.nsplit; }  // -1: balanced schedule
  int merge_launches() const { return plan_.merge_kernel; }  // merge launches per call
  const FlashArgs& args() const { return args_; }  // shapes and precision of the engine
  uint64_t launches() const { return epoch_; }  // attend() calls (a graph replay adds none)
  bool device_epochs() const { return device_epochs_; }
  // Overlap trace of the following launches (FlashParams::stamps), one
  // [grid][kMaxSlots][2] globaltimer record per launch, cleared before each.
  void set_trace(bool on);
  // copy of the last traced launch's stamps into host memory of trace_words() uint64
  void read_trace(uint64_t* host) const;
  size_t trace_words() const { return static_cast<size_t>(plan_.grid) * kMaxSlots * 2; }

 private:
  RingContext& ctx_;
  FlashArgs args_;
  FlashPlan plan_;
  size_t slots_off_ = 0;
  size_t slot_bytes_ = 0;
  void* workspace_ = nullptr;
  uint64_t* stamps_ = nullptr;
  bool trace_ = false;
  bool device_epochs_ = false;
  uint64_t epoch_ = 0;
  uint64_t arrive_total_ = 0;
  uint64_t reads_total_ = 0;
};

// ---------------------------------------------------------------------------
// ring attention (reference: src/attention/ring_attention_<backend>_gpu_bench.cu)
// ---------------------------------------------------------------------------
struct AttnOptions {
  std::string backend;    // the 7 reference schedules + b200_fused
  Prec prec = Prec::kF32x3;
  int seq = 1024;         // tokens per rank
  int heads = 1, heads_kv = 1, dim = 64;
  float scale = 1.f;
  bool kv_shared = false; // K and V are one buffer (reference-compatible data)
  bool causal = false, zigzag = false;
  std::string kernel = "tcgen05";  // partial-attention kernel of the unfused schedules: tcgen05 | simt
  bool ring_chain = false;         // b200_fused: forward along the ring instead of pulling from origin
  int warmup = 10, iters = 50;
  double timeout_s = 10.0;
  bool keep_output = true;
};

struct AttnResult {
  std::map<std::string, double> avg_ms;  // total, D2H, MPI, H2D, NCCL, CUDA-aware, attn, merge, final
  std::vector<double> step_ms;           // per-iteration total (max over ranks)
};

class AttnBench {
 public:
  AttnBench(RingContext& ctx, const AttnOptions& opt);
  ~AttnBench();
  // Copies this rank's inputs into the benchmark buffers (host pointers,
  // contiguous [seq, heads, dim] / [seq, heads_kv, dim], dtype of `prec`).
  void set_inputs(const void* q, const void* k, const void* v);
  AttnResult run();
  // The final normalised output [seq, heads, dim] (fp32 for fp32 inputs, bf16 otherwise).
  void copy_output(void* host_dst) const;
  size_t output_bytes() const;
  static size_t arena_bytes(const AttnOptions& opt, int world);

 private:
  struct Impl;
  Impl* impl_;
};

}  // namespace rab
