// fused_ring.cpp - host side of the `b200_fused` ring attention engine.  It
// replaces the reference's per-step ring loop (send/recv of the K/V shard, then
// attention and merge of the current block; src/attention/
// ring_attention_nccl_gpu_bench.cu:331-367) with one fused kernel launch per call.
#include <cstdint>
#include <stdexcept>

#include "drivers.h"
#include "strfmt.h"
#include "trace.h"

namespace rab {

size_t FusedRing::arena_bytes(Prec prec, int seq, int heads_kv, int dim, int world) {
  return static_cast<size_t>(world) * ring_block_bytes(prec, seq, heads_kv, dim) + 4096;
}

FusedRing::FusedRing(RingContext& ctx, Prec prec, int seq, int heads, int heads_kv, int dim,
                     bool causal, bool zigzag, bool ring_chain, double timeout_s,
                     bool device_epochs)
    : ctx_(ctx), device_epochs_(device_epochs) {
  const int np = ctx.world();
  if (np > kMaxSlots) throw std::runtime_error("FusedRing: too many ranks");
  if (np > 1 && !ctx.peers_open())
    throw std::runtime_error("FusedRing: peer buffers must be mapped first");
  if (np > 1 && !ctx.devices_unique())
    throw std::runtime_error(
        "FusedRing: ranks spin on each other inside the kernel and need one GPU each");
  // the flag words (and, with device-side epochs, the call counter) count
  // launches of this engine from zero on every rank
  ctx.reset_flags();
  slot_bytes_ = ring_block_bytes(prec, seq, heads_kv, dim);
  slots_off_ = ctx.arena_alloc(static_cast<size_t>(np) * slot_bytes_, 4096);
  FlashArgs& a = args_;
  a.prec = prec;
  a.Sq = seq;
  a.Hq = heads;
  a.Hkv = heads_kv;
  a.D = dim;
  a.Skv = seq;
  a.nblk = np;
  a.causal = causal ? 1 : 0;
  a.zigzag = zigzag ? 1 : 0;
  a.world = np;
  a.rank = ctx.rank();
  a.k_base = ctx.local(slots_off_);
  a.v_base = ctx.local(slots_off_ + ring_v_offset(prec, seq, heads_kv, dim));
  a.slot_stride = slot_bytes_;
  a.status = ctx.status_dev();
  a.timeout_s = timeout_s;
  a.fused = np > 1;
  a.ring_chain = ring_chain;
  a.local_slots = ctx.local(slots_off_);
  a.slot_bytes = slot_bytes_;
  a.flags_local = ctx.flags_local();
  for (int r = 0; r < np; ++r) {
    a.peer_slots[r] = np > 1 ? ctx.peer(r, slots_off_) : ctx.local(slots_off_);
    a.flags_peer[r] = np > 1 ? ctx.flags_peer(r) : ctx.flags_local();
  }
  plan_ = flash_plan(a);
  if (plan_.workspace_bytes > 0)
    cuda_check(cudaMalloc(&workspace_, plan_.workspace_bytes), "cudaMalloc(workspace)");
  a.workspace = workspace_;
  a.workspace_bytes = plan_.workspace_bytes;
}

FusedRing::~FusedRing() {
  if (workspace_) cudaFree(workspace_);
  if (stamps_) cudaFree(stamps_);
}

void FusedRing::set_trace(bool on) {
  if (on && stamps_ == nullptr)
    cuda_check(cudaMalloc(&stamps_, trace_words() * sizeof(uint64_t)), "cudaMalloc(trace)");
  trace_ = on;
}

void FusedRing::read_trace(uint64_t* host) const {
  if (stamps_ == nullptr) throw std::runtime_error("FusedRing: tracing was never enabled");
  cuda_check(cudaMemcpy(host, stamps_, trace_words() * sizeof(uint64_t), cudaMemcpyDeviceToHost),
             "read trace");
}

uint8_t* FusedRing::slot0_k() const { return ctx_.local(slots_off_); }
uint8_t* FusedRing::slot0_v() const {
  return ctx_.local(slots_off_ + ring_v_offset(args_.prec, args_.Skv, args_.Hkv, args_.D));
}

void FusedRing::prepare(const void* k, const void* v, cudaStream_t stream) {
  if (k == slot0_k() && v == slot0_v() && args_.prec == Prec::kBF16) return;
  TraceRange range("rab.ring_format");
  const int err = ring_format_launch(args_.prec, k, v, slot0_k(), slot0_v(), args_.Skv, args_.Hkv,
                                     args_.D, stream);
  cuda_check(static_cast<cudaError_t>(err), "ring_format");
}

void FusedRing::attend(const void* q, void* out, bool out_bf16, float* lse, float scale,
                       cudaStream_t stream) {
  TraceRange range("rab.fused_attention");
  FlashArgs a = args_;
  a.q = q;
  a.out = out;
  a.out_bf16 = out_bf16;
  a.lse = lse;
  a.scale = scale;
  ++epoch_;
  if (a.fused && device_epochs_) {
    // the kernel reads its epoch from the call counter (flag word kFlagCalls)
    a.call_counter = ctx_.flags_local() + kFlagCalls;
  } else if (a.fused) {
    arrive_total_ += static_cast<uint64_t>(plan_.grid);
    reads_total_ += static_cast<uint64_t>(a.world - 1) * plan_.grid;
    a.epoch = epoch_;
    a.arrive_target = arrive_total_;
    a.reads_target = reads_total_;
  }
  if (trace_) {
    cuda_check(cudaMemsetAsync(stamps_, 0, trace_words() * sizeof(uint64_t), stream),
               "clear trace");
    a.stamps = stamps_;
  }
  const int err = flash_run(a, plan_, stream);
  cuda_check(static_cast<cudaError_t>(err), "fused ring attention launch");
}

void FusedRing::forward(const void* q, const void* k, const void* v, void* out, bool out_bf16,
                        float* lse, float scale, cudaStream_t stream) {
  const bool aligned =
      reinterpret_cast<uintptr_t>(k) % 16 == 0 && reinterpret_cast<uintptr_t>(v) % 16 == 0;
  if (!args_.fused && args_.prec == Prec::kBF16 && aligned) {
    // one rank, bf16: the ring slot would only be a copy of K/V in the same
    // layout; the kernel reads the caller's K and V directly
    TraceRange range("rab.fused_attention");
    FlashArgs a = args_;
    a.q = q;
    a.k_base = k;
    a.v_base = v;
    a.slot_stride = 0;
    a.out = out;
    a.out_bf16 = out_bf16;
    a.lse = lse;
    a.scale = scale;
    const int err = flash_run(a, plan_, stream);
    cuda_check(static_cast<cudaError_t>(err), "ring attention launch");
    return;
  }
  prepare(k, v, stream);
  attend(q, out, out_bf16, lse, scale, stream);
}

void FusedRing::check() {
  const DeviceStatus s = ctx_.read_status(true);
  if (s.code != 0) {
    const std::string msg =
        strfmt("rank %d: fused ring attention wait timed out (site %u, block %u, detail %u)",
               ctx_.rank(), s.where, s.block, s.detail);
    ctx_.host().abort(msg);
    throw RankFailure(msg);
  }
}

}  // namespace rab
