// comm_bench.cpp - comm-only ring benchmark (reference: src/loop/ring_loop_*.cu).
//
// Loop structure kept from the reference (src/loop/ring_loop_staged.cu:162-231):
// per repetition the send buffer is reset from the host init pattern and the
// receive buffer zeroed, all ranks meet in a barrier, the shard rotates np-1
// times to the right neighbour with per-phase host timers, and the per-rank
// phase times are max-reduced; repetitions after `warmup` are averaged.  An
// untimed precheck ring first verifies that every step delivered the shard of
// rank (rank - step - 1) mod np (reference C15, :122-155).
//
// Transports (native re-expressions of the reference's backends):
//   staged               D2H -> host ring exchange through shared-memory
//                        mailboxes (copy-in/copy-out, like MPI's shm path) -> H2D
//   staged_Isendrecv     same data path, both directions progressed together
//   cuda_aware           device-to-device copy into the right neighbour's
//                        receive buffer through the CUDA IPC mapping (what a
//                        CUDA-aware MPI does inside a node), blocking
//   cuda_aware_Isendrecv posted copy + completion poll
//   nccl                 ncclGroupStart / ncclSend / ncclRecv / ncclGroupEnd
//   b200_fused           one kernel for all np-1 steps, NVLink peer stores,
//                        per-slice flags (p2p_ring.cu)
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "drivers.h"
#include "flash.h"
#include "strfmt.h"
#include "trace.h"

namespace rab {

namespace {

double wall_ms() {
  return std::chrono::duration<double, std::milli>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

struct PinnedBuf {
  void* p = nullptr;
  explicit PinnedBuf(size_t n) { cuda_check(cudaMallocHost(&p, n), "cudaMallocHost"); }
  ~PinnedBuf() {
    if (p) cudaFreeHost(p);
  }
};

bool is_backend(const std::string& b) {
  return b == "staged" || b == "staged_Isendrecv" || b == "cuda_aware" ||
         b == "cuda_aware_Isendrecv" || b == "nccl" || b == "b200_fused";
}

}  // namespace

size_t comm_arena_bytes(size_t bytes) { return 2 * ((bytes + 4095) / 4096 * 4096) + 8192; }

// One blocking device-to-device ring step through the IPC mapping: wait until
// the right neighbour's receive buffer is free, copy into it, publish
// delivery, wait for the left neighbour's delivery into ours.
static void cuda_aware_step(RingContext& ctx, size_t cur_off, size_t next_off, size_t bytes,
                            cudaEvent_t done, bool wait_copy) {
  HostComm& h = ctx.host();
  const uint64_t q = ctx.next_xfer();
  const int me = ctx.rank(), right = ctx.right(), left = ctx.left();
  h.publish(h.ready_words()[me].v, q);  // our `next` is free for step q
  h.wait_at_least(h.ready_words()[right].v, q, "receive-buffer ready", right);
  cuda_check(cudaMemcpyAsync(ctx.peer(right, next_off), ctx.local(cur_off), bytes,
                             cudaMemcpyDeviceToDevice, ctx.comm_stream()),
             "cudaMemcpyAsync(peer)");
  cuda_check(cudaEventRecord(done, ctx.comm_stream()), "event");
  if (wait_copy) {
    cuda_check(cudaEventSynchronize(done), "event sync");
    h.publish(h.delivered_words()[right].v, q);
    h.wait_at_least(h.delivered_words()[me].v, q, "delivery", left);
  }
}

CommResult run_comm_bench(RingContext& ctx, const CommOptions& o) {
  if (!is_backend(o.backend)) throw std::runtime_error("unknown comm backend: " + o.backend);
  if (o.bytes == 0 || o.bytes % 4 != 0)
    throw std::runtime_error("kv_size_bytes must be a positive multiple of 4");
  const int np = ctx.world(), rank = ctx.rank();
  const bool device_path = o.backend == "cuda_aware" || o.backend == "cuda_aware_Isendrecv" ||
                           o.backend == "b200_fused";
  if (np > 1 && device_path && !ctx.peers_open())
    throw std::runtime_error(o.backend + " needs peer-mapped buffers (open_peers)");
  if (np > 1 && o.backend == "b200_fused" && !ctx.devices_unique())
    throw std::runtime_error(
        "b200_fused spins on peer flags inside a kernel and needs one GPU per rank");
  if (np > 1 && o.backend == "nccl" && !ctx.has_nccl())
    throw std::runtime_error("nccl backend: communicator not initialised");
  cuda_check(cudaSetDevice(ctx.device()), "cudaSetDevice");
  ctx.reset_flags();
  ctx.arena_reset();
  const size_t off1 = ctx.arena_alloc(o.bytes, 4096);
  const size_t off2 = ctx.arena_alloc(o.bytes, 4096);
  uint8_t* d1 = ctx.local(off1);
  uint8_t* d2 = ctx.local(off2);
  const size_t n_floats = o.bytes / 4;
  std::vector<float> h_init(n_floats);
  for (size_t i = 0; i < n_floats; ++i) h_init[i] = rank * 1000.0f + static_cast<float>(i);
  PinnedBuf h_send(o.bytes), h_recv(o.bytes);
  cudaStream_t cs = ctx.comm_stream();
  cudaEvent_t ev0, ev1, done;
  cuda_check(cudaEventCreate(&ev0), "event");
  cuda_check(cudaEventCreate(&ev1), "event");
  cuda_check(cudaEventCreate(&done), "event");
  // default: one CTA per SM
  const int slices = std::min(o.slices > 0 ? o.slices : flash_sm_count(), static_cast<int>(kMaxSlices));

  RingCopyParams rp;
  std::memset(&rp, 0, sizeof(rp));
  if (np > 1 && o.backend == "b200_fused") {
    rp.buf[0] = d1;
    rp.buf[1] = d2;
    rp.right_buf[0] = ctx.peer(ctx.right(), off1);
    rp.right_buf[1] = ctx.peer(ctx.right(), off2);
    rp.left_buf[0] = ctx.peer(ctx.left(), off1);
    rp.left_buf[1] = ctx.peer(ctx.left(), off2);
    rp.arrived_local = ctx.flags_local() + kFlagRingArrived;
    rp.arrived_right = ctx.flags_peer(ctx.right()) + kFlagRingArrived;
    rp.sent_local = ctx.flags_local() + kFlagRingSent;
    rp.sent_right = ctx.flags_peer(ctx.right()) + kFlagRingSent;
    rp.sent_left = ctx.flags_peer(ctx.left()) + kFlagRingSent;
    rp.bytes = o.bytes;
    rp.status = ctx.status_dev();
    rp.timeout_ns = static_cast<uint64_t>(ctx.host().timeout_s() * 1e9);
    rp.mode = o.p2p_mode;
  }
  auto check_dev_status = [&](const char* what) {
    const DeviceStatus s = ctx.read_status(true);
    if (s.code != 0) {
      const std::string msg =
          strfmt("rank %d: %s: device wait timed out (site %u, block %u, detail %u)", rank, what,
                 s.where, s.block, s.detail);
      ctx.host().abort(msg);
      throw RankFailure(msg);
    }
  };

  // One ring step on the chosen transport; buffers named by arena offset.
  auto step = [&](size_t cur_off, size_t next_off, int s, double* t_d2h, double* t_mpi,
                  double* t_h2d) {
    if (o.backend == "staged" || o.backend == "staged_Isendrecv") {
      const double t1 = wall_ms();
      cuda_check(cudaMemcpy(h_send.p, ctx.local(cur_off), o.bytes, cudaMemcpyDeviceToHost), "D2H");
      const double t2 = wall_ms();
      ctx.host().ring_sendrecv(h_send.p, h_recv.p, o.bytes);
      const double t3 = wall_ms();
      cuda_check(cudaMemcpy(ctx.local(next_off), h_recv.p, o.bytes, cudaMemcpyHostToDevice), "H2D");
      const double t4 = wall_ms();
      *t_d2h += t2 - t1;
      *t_mpi += t3 - t2;
      *t_h2d += t4 - t3;
    } else if (o.backend == "cuda_aware" || o.backend == "cuda_aware_Isendrecv") {
      const double t1 = wall_ms();
      cuda_aware_step(ctx, cur_off, next_off, o.bytes, done, true);
      *t_mpi += wall_ms() - t1;
    } else if (o.backend == "nccl") {
      const double t1 = wall_ms();
      nccl_check(ncclGroupStart(), "ncclGroupStart");
      nccl_check(ncclSend(ctx.local(cur_off), n_floats, ncclFloat, ctx.right(), ctx.nccl(), cs),
                 "ncclSend");
      nccl_check(ncclRecv(ctx.local(next_off), n_floats, ncclFloat, ctx.left(), ctx.nccl(), cs),
                 "ncclRecv");
      nccl_check(ncclGroupEnd(), "ncclGroupEnd");
      cuda_check(cudaStreamSynchronize(cs), "stream sync");
      *t_mpi += wall_ms() - t1;
    } else {  // b200_fused, one step per launch (precheck path)
      rp.nsteps = 1;
      rp.first_step = s;
      rp.base = ctx.take_steps(1);
      const double t1 = wall_ms();
      cuda_check(static_cast<cudaError_t>(p2p_ring_launch(rp, slices, cs)), "p2p ring launch");
      cuda_check(cudaStreamSynchronize(cs), "stream sync");
      *t_mpi += wall_ms() - t1;
      check_dev_status("b200_fused precheck");
    }
  };

  CommResult res;
  // ---- precheck: one untimed ring, check the first float of every step ----
  if (o.precheck && np > 1) {
    cuda_check(cudaMemcpy(d1, h_init.data(), o.bytes, cudaMemcpyHostToDevice), "H2D init");
    cuda_check(cudaMemset(d2, 0, o.bytes), "memset");
    cuda_check(cudaDeviceSynchronize(), "reset sync");  // peers may write d2 after the barrier
    ctx.host().barrier();
    size_t cur = off1, next = off2;
    double a = 0, b = 0, c = 0;
    for (int s = 0; s < np - 1; ++s) {
      step(cur, next, s, &a, &b, &c);
      float first = 0.f;
      cuda_check(cudaMemcpy(&first, ctx.local(next), 4, cudaMemcpyDeviceToHost), "D2H check");
      const int src = ((rank - s - 1) % np + np) % np;
      if (first != src * 1000.0f && res.precheck_ok) {
        res.precheck_ok = false;
        res.precheck_msg = strfmt("rank %d step %d: received %g, expected %g", rank, s,
                                  static_cast<double>(first), src * 1000.0);
      }
      std::swap(cur, next);
    }
    ctx.host().barrier();
    if (!res.precheck_ok) {
      ctx.host().abort(res.precheck_msg);
      throw RankFailure("precheck failed: " + res.precheck_msg);
    }
  }

  // ---- timed repetitions ----
  double sum[6] = {0, 0, 0, 0, 0, 0};  // d2h, mpi, h2d, total, p2p(kernel), spare
  for (int rep = 0; rep < o.warmup + o.iters; ++rep) {
    TraceRange range(rep < o.warmup ? "rab.comm_warmup" : "rab.comm_rep");
    cuda_check(cudaMemcpy(d1, h_init.data(), o.bytes, cudaMemcpyHostToDevice), "H2D reset");
    cuda_check(cudaMemset(d2, 0, o.bytes), "memset");
    cuda_check(cudaDeviceSynchronize(), "reset sync");
    double t_d2h = 0, t_mpi = 0, t_h2d = 0, t_kernel = 0;
    ctx.host().barrier();
    const double t0 = wall_ms();
    if (o.backend == "b200_fused") {
      if (np > 1) {
        rp.nsteps = np - 1;
        rp.first_step = 0;
        rp.base = ctx.take_steps(np - 1);
        cuda_check(cudaEventRecord(ev0, cs), "event");
        cuda_check(static_cast<cudaError_t>(p2p_ring_launch(rp, slices, cs)), "p2p ring launch");
        cuda_check(cudaEventRecord(ev1, cs), "event");
        cuda_check(cudaStreamSynchronize(cs), "stream sync");
        float k = 0.f;
        cuda_check(cudaEventElapsedTime(&k, ev0, ev1), "elapsed");
        t_kernel = k;
        t_mpi = wall_ms() - t0;
      }
    } else {
      size_t cur = off1, next = off2;
      for (int s = 0; s < np - 1; ++s) {
        step(cur, next, s, &t_d2h, &t_mpi, &t_h2d);
        std::swap(cur, next);
      }
    }
    const double t_total = wall_ms() - t0;
    if (o.backend == "b200_fused" && np > 1) check_dev_status("b200_fused ring");
    const std::vector<double> mx = ctx.host().reduce_max({t_d2h, t_mpi, t_h2d, t_total, t_kernel});
    if (rep >= o.warmup)
      for (int i = 0; i < 5; ++i) sum[i] += mx[i];
  }
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  cudaEventDestroy(done);
  // Full-content check of the last repetition (the precheck, like the
  // reference's, looks at one float per step): after np-1 steps this rank
  // holds the whole shard of rank (rank + 1) mod np.  Every rank takes part in
  // the reduction, so all of them fail together.
  if (o.precheck && np > 1 && o.warmup + o.iters > 0) {
    std::vector<float> got(n_floats);
    cuda_check(cudaMemcpy(got.data(), (np - 1) & 1 ? d2 : d1, o.bytes, cudaMemcpyDeviceToHost),
                          "D2H final check");
    const int src = (rank + 1) % np;
    size_t bad = n_floats;
    for (size_t i = 0; i < n_floats; ++i)
      if (got[i] != src * 1000.0f + static_cast<float>(i)) {
        bad = i;
        break;
      }
    const double any_bad = ctx.host().reduce_max({bad < n_floats ? 1.0 : 0.0})[0];
    if (any_bad > 0.0) {
      res.precheck_ok = false;
      res.precheck_msg =
          bad < n_floats
              ? strfmt("rank %d: final buffer differs at float %zu: got %g, expected %g", rank,
                       bad, static_cast<double>(got[bad]),
                       static_cast<double>(src * 1000.0f + static_cast<float>(bad)))
              : strfmt("rank %d: another rank's final buffer is wrong", rank);
      throw RankFailure("final content check failed: " + res.precheck_msg);
    }
  }
  const double n = o.iters > 0 ? o.iters : 1;
  res.avg_ms["d2h"] = sum[0] / n;
  res.avg_ms["mpi"] = sum[1] / n;
  res.avg_ms["h2d"] = sum[2] / n;
  res.avg_ms["total"] = sum[3] / n;
  res.avg_ms["kernel"] = sum[4] / n;
  return res;
}

}  // namespace rab
