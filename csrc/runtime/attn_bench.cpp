// attn_bench.cpp - ring attention benchmark schedules
// (reference: src/attention/ring_attention_<backend>_gpu_bench.cu).
//
// Every schedule keeps the reference's structure and phase timers:
//   staged                        blocking: local attn+merge, then per step
//                                 D2H -> host exchange -> H2D -> attn -> merge
//                                 (…staged_gpu_bench.cu:361-426)
//   staged_Isendrecv(_overlap)    async D2H on the comm stream || attn+merge on
//                                 the compute stream; the host exchange runs
//                                 once the D2H lands, then async H2D
//                                 (…staged_Isendrecv_gpu_bench.cu:333-395; the
//                                 two reference programs run the same schedule)
//   cuda_aware                    blocking device-to-device exchange, then
//                                 attn+merge (…cuda_aware_gpu_bench.cu:310-343)
//   cuda_aware_Isendrecv          posted exchange || attn+merge; the exchange
//                                 timer runs until both finish (…:333-370)
//   cuda_aware_Isendrecv_overlap  same, the exchange timer stops at its own
//                                 completion (…overlap_gpu_bench.cu:338-359)
//   nccl                          ncclSend/Recv on the comm stream || attn+merge
//                                 on the compute stream, event timers
//                                 (…nccl_gpu_bench.cu:331-383)
//   b200_fused                    one kernel: K/V blocks move over NVLink inside
//                                 the tcgen05 attention kernel (FusedRing)
// The unfused schedules compute each block with the tcgen05 partial kernel (or
// the exact-order CUDA-core kernel, `kernel=simt`) and merge with merge_lse;
// normalisation runs on the device (the reference does it on the host).
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cstring>
#include <memory>
#include "strfmt.h"
#include <stdexcept>
#include <vector>

#include "drivers.h"
#include "trace.h"
#include "launchers.h"

namespace rab {

namespace {

double wall_ms() {
  return std::chrono::duration<double, std::milli>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

bool known_backend(const std::string& b) {
  return b == "staged" || b == "staged_Isendrecv" || b == "staged_Isendrecv_overlap" ||
         b == "cuda_aware" || b == "cuda_aware_Isendrecv" || b == "cuda_aware_Isendrecv_overlap" ||
         b == "nccl" || b == "b200_fused";
}

float ev_ms(cudaEvent_t a, cudaEvent_t b) {
  float ms = 0.f;
  cuda_check(cudaEventElapsedTime(&ms, a, b), "cudaEventElapsedTime");
  return ms;
}

}  // namespace

struct AttnBench::Impl {
  RingContext& ctx;
  AttnOptions o;
  int np, rank;
  size_t esize, q_bytes, kv_bytes, shard_bytes, out_bytes;
  size_t rows;  // seq * heads
  size_t off_shard[2] = {0, 0};
  std::unique_ptr<FusedRing> fused;
  void* q_dev = nullptr;
  void* out_dev = nullptr;
  float *acc_run = nullptr, *m_run = nullptr, *l_run = nullptr;
  float *acc_new = nullptr, *m_new = nullptr, *l_new = nullptr;
  void* prep_slot = nullptr;
  void* ws = nullptr;
  FlashArgs pa;
  FlashPlan pplan{};
  std::vector<uint8_t> h_shard, h_q;
  std::vector<float> h_minit;
  void* h_send = nullptr;
  void* h_recv = nullptr;
  cudaEvent_t e_a0, e_a1, e_m1, e_c0, e_c1, e_d2h, e_h2d, e_x;

  Impl(RingContext& c, const AttnOptions& opt) : ctx(c), o(opt) {
    np = ctx.world();
    rank = ctx.rank();
    if (!known_backend(o.backend)) throw std::runtime_error("unknown attention backend " + o.backend);
    if (o.kernel == "simt" && o.prec != Prec::kF32x3)
      throw std::runtime_error("the CUDA-core kernel is fp32 only");
    if (o.kernel == "simt" && o.causal)
      throw std::runtime_error("the CUDA-core kernel has no causal mask; use kernel=tcgen05");
    if (o.kv_shared && o.heads_kv != o.heads && o.heads_kv != 1)
      throw std::runtime_error("kv_shared needs one K/V buffer");
    const bool needs_peers = o.backend.rfind("cuda_aware", 0) == 0 || o.backend == "b200_fused";
    if (np > 1 && needs_peers && !ctx.peers_open())
      throw std::runtime_error(o.backend + " needs peer-mapped buffers");
    if (np > 1 && o.backend == "nccl" && !ctx.has_nccl())
      throw std::runtime_error("nccl backend: communicator not initialised");
    cuda_check(cudaSetDevice(ctx.device()), "cudaSetDevice");
    esize = o.prec == Prec::kF32x3 ? 4 : 2;
    rows = static_cast<size_t>(o.seq) * o.heads;
    q_bytes = rows * o.dim * esize;
    kv_bytes = static_cast<size_t>(o.seq) * o.heads_kv * o.dim * esize;
    shard_bytes = o.kv_shared ? kv_bytes : 2 * kv_bytes;
    out_bytes = rows * o.dim * esize;
    ctx.arena_reset();
    if (o.backend == "b200_fused") {
      fused = std::make_unique<FusedRing>(ctx, o.prec, o.seq, o.heads, o.heads_kv, o.dim, o.causal,
                                          o.zigzag, o.ring_chain, o.timeout_s);
    } else {
      ctx.reset_flags();
      off_shard[0] = ctx.arena_alloc(shard_bytes, 4096);
      off_shard[1] = ctx.arena_alloc(shard_bytes, 4096);
    }
    cuda_check(cudaMalloc(&q_dev, q_bytes), "cudaMalloc(q)");
    cuda_check(cudaMalloc(&out_dev, out_bytes), "cudaMalloc(out)");
    if (o.backend != "b200_fused") {
      const size_t st = rows * sizeof(float);
      cuda_check(cudaMalloc(&acc_run, rows * o.dim * sizeof(float)), "cudaMalloc");
      cuda_check(cudaMalloc(&acc_new, rows * o.dim * sizeof(float)), "cudaMalloc");
      cuda_check(cudaMalloc(&m_run, st), "cudaMalloc");
      cuda_check(cudaMalloc(&l_run, st), "cudaMalloc");
      cuda_check(cudaMalloc(&m_new, st), "cudaMalloc");
      cuda_check(cudaMalloc(&l_new, st), "cudaMalloc");
      h_minit.assign(rows, -FLT_MAX);
      if (o.kernel == "tcgen05") {
        if (o.prec == Prec::kF32x3)
          cuda_check(cudaMalloc(&prep_slot, ring_block_bytes(o.prec, o.seq, o.heads_kv, o.dim)),
                     "cudaMalloc(prep slot)");
        pa.prec = o.prec;
        pa.Sq = o.seq;
        pa.Hq = o.heads;
        pa.Hkv = o.heads_kv;
        pa.D = o.dim;
        pa.Skv = o.seq;
        pa.nblk = 1;
        pa.scale = o.scale;
        pa.causal = o.causal;
        pa.zigzag = o.zigzag;
        pa.world = np;
        pa.rank = rank;
        pa.partial = true;
        pa.acc = acc_new;
        pa.m = m_new;
        pa.l = l_new;
        pa.status = ctx.status_dev();
        pa.timeout_s = o.timeout_s;
        pplan = flash_plan(pa);
        if (pplan.workspace_bytes)
          cuda_check(cudaMalloc(&ws, pplan.workspace_bytes), "cudaMalloc(ws)");
        pa.workspace = ws;
        pa.workspace_bytes = pplan.workspace_bytes;
      }
      if (o.backend.rfind("staged", 0) == 0) {
        cuda_check(cudaMallocHost(&h_send, shard_bytes), "cudaMallocHost");
        cuda_check(cudaMallocHost(&h_recv, shard_bytes), "cudaMallocHost");
      }
    }
    for (cudaEvent_t* e : {&e_a0, &e_a1, &e_m1, &e_c0, &e_c1, &e_d2h, &e_h2d, &e_x})
      cuda_check(cudaEventCreate(e), "cudaEventCreate");
  }

  ~Impl() {
    cudaSetDevice(ctx.device());
    cudaDeviceSynchronize();
    for (void* p : {q_dev, out_dev, static_cast<void*>(acc_run), static_cast<void*>(acc_new),
                    static_cast<void*>(m_run), static_cast<void*>(l_run),
                    static_cast<void*>(m_new), static_cast<void*>(l_new), prep_slot, ws})
      if (p) cudaFree(p);
    if (fused == nullptr || o.prec != Prec::kBF16) {
      if (raw_k) cudaFree(raw_k);
      if (raw_v) cudaFree(raw_v);
    }
    if (h_send) cudaFreeHost(h_send);
    if (h_recv) cudaFreeHost(h_recv);
    for (cudaEvent_t e : {e_a0, e_a1, e_m1, e_c0, e_c1, e_d2h, e_h2d, e_x}) cudaEventDestroy(e);
  }

  uint8_t* shard_k(size_t off) { return ctx.local(off); }
  uint8_t* shard_v(size_t off) { return ctx.local(off) + (o.kv_shared ? 0 : kv_bytes); }

  void check_dev(const char* what) {
    const DeviceStatus s = ctx.read_status(true);
    if (s.code != 0) {
      const std::string msg = strfmt("rank %d: %s: device wait timed out (site %u, block %u)",
                                     rank, what, s.where, s.block);
      ctx.host().abort(msg);
      throw RankFailure(msg);
    }
  }

  // Partial attention of the local Q against the shard at `off` (ring step s)
  // and the merge into the running state, on `stream`, bracketed by events.
  void attn_merge(size_t off, int s, cudaStream_t stream) {
    cuda_check(cudaEventRecord(e_a0, stream), "event");
    const void* K = shard_k(off);
    const void* V = shard_v(off);
    if (o.kernel == "simt") {
      cuda_check(static_cast<cudaError_t>(simt_partial_attention_launch(
                     static_cast<const float*>(q_dev), static_cast<const float*>(K),
                     static_cast<const float*>(V), o.seq, o.seq, o.heads, o.heads_kv, o.dim,
                     o.scale, -1, acc_new, m_new, l_new, false, stream)),
                 "simt attention");
    } else {
      FlashArgs a = pa;
      a.q = q_dev;
      a.blk_offset = s;
      if (o.prec == Prec::kF32x3) {
        uint8_t* slot = static_cast<uint8_t*>(prep_slot);
        cuda_check(static_cast<cudaError_t>(ring_format_launch(
                       o.prec, K, V, slot, slot + ring_v_offset(o.prec, o.seq, o.heads_kv, o.dim),
                       o.seq, o.heads_kv, o.dim, stream)),
                   "ring_format");
        a.k_base = slot;
        a.v_base = slot + ring_v_offset(o.prec, o.seq, o.heads_kv, o.dim);
      } else {
        a.k_base = K;  // bf16 blocks are read in place
        a.v_base = V;
      }
      cuda_check(static_cast<cudaError_t>(flash_run(a, pplan, stream)), "flash partial");
    }
    cuda_check(cudaEventRecord(e_a1, stream), "event");
    cuda_check(static_cast<cudaError_t>(merge_lse_launch(m_run, l_run, acc_run, m_new, l_new,
                                                         acc_new, static_cast<int>(rows), o.dim,
                                                         stream)),
               "merge");
    cuda_check(cudaEventRecord(e_m1, stream), "event");
  }

  void reset_iteration() {
    if (o.backend == "b200_fused") return;  // inputs are formatted from the input buffers each step
    cuda_check(cudaMemcpy(ctx.local(off_shard[0]), h_shard.data(), shard_bytes,
                          cudaMemcpyHostToDevice),
               "H2D reset");
    cuda_check(cudaMemset(ctx.local(off_shard[1]), 0, shard_bytes), "memset");
    cuda_check(cudaMemcpy(m_run, h_minit.data(), rows * sizeof(float), cudaMemcpyHostToDevice),
               "reset m");
    cuda_check(cudaMemset(l_run, 0, rows * sizeof(float)), "reset l");
    cuda_check(cudaMemset(acc_run, 0, rows * o.dim * sizeof(float)), "reset acc");
    // peers write into our receive buffer once the next barrier releases them
    cuda_check(cudaDeviceSynchronize(), "reset sync");
  }

  // device-to-device step through the IPC mapping (see comm_bench.cpp)
  uint64_t ca_post(size_t cur, size_t next) {
    HostComm& h = ctx.host();
    const uint64_t q = ctx.next_xfer();
    h.publish(h.ready_words()[rank].v, q);
    h.wait_at_least(h.ready_words()[ctx.right()].v, q, "receive-buffer ready", ctx.right());
    cuda_check(cudaEventRecord(e_c0, ctx.comm_stream()), "event");
    cuda_check(cudaMemcpyAsync(ctx.peer(ctx.right(), next), ctx.local(cur), shard_bytes,
                               cudaMemcpyDeviceToDevice, ctx.comm_stream()),
               "peer copy");
    cuda_check(cudaEventRecord(e_c1, ctx.comm_stream()), "event");
    return q;
  }
  void ca_finish(uint64_t q) {
    HostComm& h = ctx.host();
    cuda_check(cudaEventSynchronize(e_c1), "event sync");
    h.publish(h.delivered_words()[ctx.right()].v, q);
    h.wait_at_least(h.delivered_words()[rank].v, q, "delivery", ctx.left());
  }

  // Poll an event without blocking the host thread's progress loop.
  static bool done(cudaEvent_t e) {
    const cudaError_t r = cudaEventQuery(e);
    if (r == cudaSuccess) return true;
    if (r != cudaErrorNotReady) cuda_check(r, "cudaEventQuery");
    return false;
  }

  AttnResult run() {
    AttnResult res;
    const std::string& b = o.backend;
    cudaStream_t cs = ctx.compute_stream(), ms = ctx.comm_stream();
    std::map<std::string, double> sum;
    for (int it = 0; it < o.warmup + o.iters; ++it) {
      TraceRange range(it < o.warmup ? "rab.attn_warmup" : "rab.attn_iter");
      reset_iteration();
      double t_d2h = 0, t_mpi = 0, t_h2d = 0, t_nccl = 0, t_ca = 0, t_attn = 0, t_merge = 0,
             t_final = 0, t_prep = 0;
      ctx.host().barrier();
      const double t0 = wall_ms();
      size_t cur = off_shard[0], next = off_shard[1];
      if (b == "b200_fused") {
        cuda_check(cudaEventRecord(e_a0, cs), "event");
        fused->prepare(shard_k_input(), shard_v_input(), cs);
        cuda_check(cudaEventRecord(e_a1, cs), "event");
        fused->attend(q_dev, out_dev, o.prec == Prec::kBF16, nullptr, o.scale, cs);
        cuda_check(cudaEventRecord(e_m1, cs), "event");
        cuda_check(cudaStreamSynchronize(cs), "sync");
        t_prep = ev_ms(e_a0, e_a1);
        t_attn = ev_ms(e_a1, e_m1);
      } else if (b == "staged" || b == "cuda_aware") {
        attn_merge(cur, 0, cs);
        cuda_check(cudaStreamSynchronize(cs), "sync");
        t_attn += ev_ms(e_a0, e_a1);
        t_merge += ev_ms(e_a1, e_m1);
        for (int s = 0; s < np - 1; ++s) {
          if (b == "staged") {
            const double t1 = wall_ms();
            cuda_check(cudaMemcpy(h_send, ctx.local(cur), shard_bytes, cudaMemcpyDeviceToHost), "D2H");
            const double t2 = wall_ms();
            ctx.host().ring_sendrecv(h_send, h_recv, shard_bytes);
            const double t3 = wall_ms();
            cuda_check(cudaMemcpy(ctx.local(next), h_recv, shard_bytes, cudaMemcpyHostToDevice), "H2D");
            t_d2h += t2 - t1;
            t_mpi += t3 - t2;
            t_h2d += wall_ms() - t3;
          } else {
            const double t1 = wall_ms();
            ca_finish(ca_post(cur, next));
            t_mpi += wall_ms() - t1;
          }
          attn_merge(next, s + 1, cs);
          cuda_check(cudaStreamSynchronize(cs), "sync");
          t_attn += ev_ms(e_a0, e_a1);
          t_merge += ev_ms(e_a1, e_m1);
          std::swap(cur, next);
        }
      } else {
        // overlapped schedules: transfer of `cur` || compute on `cur`
        for (int s = 0; s < np - 1; ++s) {
          if (b == "nccl") {
            cuda_check(cudaEventRecord(e_c0, ms), "event");
            nccl_check(ncclGroupStart(), "ncclGroupStart");
            nccl_check(ncclSend(ctx.local(cur), shard_bytes / esize,
                                esize == 4 ? ncclFloat : ncclBfloat16, ctx.right(), ctx.nccl(), ms),
                       "ncclSend");
            nccl_check(ncclRecv(ctx.local(next), shard_bytes / esize,
                                esize == 4 ? ncclFloat : ncclBfloat16, ctx.left(), ctx.nccl(), ms),
                       "ncclRecv");
            nccl_check(ncclGroupEnd(), "ncclGroupEnd");
            cuda_check(cudaEventRecord(e_c1, ms), "event");
            attn_merge(cur, s, cs);
            cuda_check(cudaEventSynchronize(e_m1), "sync");
            cuda_check(cudaEventSynchronize(e_c1), "sync");
            t_nccl += ev_ms(e_c0, e_c1);
          } else if (b == "staged_Isendrecv" || b == "staged_Isendrecv_overlap") {
            const double t1 = wall_ms();
            cuda_check(cudaMemcpyAsync(h_send, ctx.local(cur), shard_bytes, cudaMemcpyDeviceToHost, ms),
                       "D2H async");
            cuda_check(cudaEventRecord(e_d2h, ms), "event");
            attn_merge(cur, s, cs);
            // host progress loop: exchange as soon as the D2H landed, then H2D
            while (!done(e_d2h)) ctx.host().check_abort();
            const double t2 = wall_ms();
            ctx.host().ring_sendrecv(h_send, h_recv, shard_bytes);
            const double t3 = wall_ms();
            cuda_check(cudaMemcpyAsync(ctx.local(next), h_recv, shard_bytes, cudaMemcpyHostToDevice, ms),
                       "H2D async");
            cuda_check(cudaEventRecord(e_h2d, ms), "event");
            while (!(done(e_m1) && done(e_h2d))) ctx.host().check_abort();
            t_d2h += t2 - t1;
            t_mpi += t3 - t2;
            t_h2d += wall_ms() - t3;
          } else {  // cuda_aware_Isendrecv(_overlap)
            const double t1 = wall_ms();
            const uint64_t q = ca_post(cur, next);
            attn_merge(cur, s, cs);
            if (b == "cuda_aware_Isendrecv") {
              while (!(done(e_c1) && done(e_m1))) ctx.host().check_abort();
              ca_finish(q);
              t_ca += wall_ms() - t1;
            } else {
              ca_finish(q);
              t_ca += wall_ms() - t1;
              cuda_check(cudaEventSynchronize(e_m1), "sync");
            }
          }
          t_attn += ev_ms(e_a0, e_a1);
          t_merge += ev_ms(e_a1, e_m1);
          std::swap(cur, next);
        }
        attn_merge(cur, np - 1, cs);  // the last received block
        cuda_check(cudaStreamSynchronize(cs), "sync");
        t_attn += ev_ms(e_a0, e_a1);
        t_merge += ev_ms(e_a1, e_m1);
      }
      if (b != "b200_fused") {
        const double tf = wall_ms();
        cuda_check(static_cast<cudaError_t>(normalize_launch(acc_run, m_run, l_run, out_dev,
                                                             o.prec == Prec::kBF16, nullptr,
                                                             static_cast<int>(rows), o.dim, cs)),
                   "normalize");
        cuda_check(cudaStreamSynchronize(cs), "sync");
        t_final = wall_ms() - tf;
      }
      ctx.host().barrier();
      const double t_total = wall_ms() - t0;
      check_dev(b.c_str());
      const std::vector<double> mx = ctx.host().reduce_max(
          {t_total, t_d2h, t_mpi, t_h2d, t_nccl, t_ca, t_attn, t_merge, t_final, t_prep});
      if (it >= o.warmup) {
        static const char* names[] = {"total", "D2H", "MPI", "H2D", "NCCL",
                                      "CUDA-aware", "attn", "merge", "final", "prep"};
        for (int i = 0; i < 10; ++i) sum[names[i]] += mx[i];
        res.step_ms.push_back(mx[0]);
      }
    }
    const double n = o.iters > 0 ? o.iters : 1;
    for (auto& kv : sum) res.avg_ms[kv.first] = kv.second / n;
    return res;
  }

  // inputs of the fused engine: raw K/V live outside the arena for fp32 (the
  // formatter reads them); bf16 inputs are written straight into slot 0
  void* raw_k = nullptr;
  void* raw_v = nullptr;
  const void* shard_k_input() { return raw_k; }
  const void* shard_v_input() { return raw_v; }
};

AttnBench::AttnBench(RingContext& ctx, const AttnOptions& opt) : impl_(new Impl(ctx, opt)) {}
AttnBench::~AttnBench() { delete impl_; }

size_t AttnBench::arena_bytes(const AttnOptions& o, int world) {
  const size_t es = o.prec == Prec::kF32x3 ? 4 : 2;
  const size_t kv = static_cast<size_t>(o.seq) * o.heads_kv * o.dim * es;
  const size_t shard = o.kv_shared ? kv : 2 * kv;
  const size_t unfused = 2 * ((shard + 4095) / 4096 * 4096) + 8192;
  const size_t f = FusedRing::arena_bytes(o.prec, o.seq, o.heads_kv, o.dim, world);
  return std::max(unfused, f);
}

void AttnBench::set_inputs(const void* q, const void* k, const void* v) {
  Impl& m = *impl_;
  cuda_check(cudaSetDevice(m.ctx.device()), "cudaSetDevice");
  cuda_check(cudaMemcpy(m.q_dev, q, m.q_bytes, cudaMemcpyHostToDevice), "H2D q");
  if (m.o.backend == "b200_fused") {
    if (m.o.prec == Prec::kBF16) {
      m.raw_k = m.fused->slot0_k();
      m.raw_v = m.fused->slot0_v();
    } else {
      if (!m.raw_k) cuda_check(cudaMalloc(&m.raw_k, m.kv_bytes), "cudaMalloc(k)");
      if (!m.raw_v) cuda_check(cudaMalloc(&m.raw_v, m.kv_bytes), "cudaMalloc(v)");
    }
    cuda_check(cudaMemcpy(m.raw_k, k, m.kv_bytes, cudaMemcpyHostToDevice), "H2D k");
    cuda_check(cudaMemcpy(m.raw_v, v, m.kv_bytes, cudaMemcpyHostToDevice), "H2D v");
    return;
  }
  m.h_shard.resize(m.shard_bytes);
  std::memcpy(m.h_shard.data(), k, m.kv_bytes);
  if (!m.o.kv_shared) std::memcpy(m.h_shard.data() + m.kv_bytes, v, m.kv_bytes);
}

AttnResult AttnBench::run() { return impl_->run(); }

size_t AttnBench::output_bytes() const { return impl_->out_bytes; }

void AttnBench::copy_output(void* host_dst) const {
  cuda_check(cudaSetDevice(impl_->ctx.device()), "cudaSetDevice");
  cuda_check(cudaDeviceSynchronize(), "sync");
  cuda_check(cudaMemcpy(host_dst, impl_->out_dev, impl_->out_bytes, cudaMemcpyDeviceToHost),
             "D2H out");
}

}  // namespace rab
