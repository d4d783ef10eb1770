// p2p_ring.cu - comm-only ring rotation over NVLink peer memory, all np-1 steps
// in one launch (the `b200_fused` comm backend).
//
// Same data movement as the reference loops (src/loop/ring_loop_*.cu: every
// step sends the current shard to rank+1 and receives the next one from
// rank-1, two buffers swapped per step) but with no library call: CTA c of
// every rank owns byte slice c of the shard, pushes it into the right
// neighbour's receive buffer with 16-byte stores through the peer mapping, and
// hands over with two monotonically increasing flags per slice:
//   arrived[c] (in the receiver's memory)  step n of slice c has landed
//   sent[c]    (in the sender's memory)    the sender finished reading slice c of step n
// so each slice runs its own pipeline and no grid-wide barrier is needed.  All
// waits are bounded and report through the status word.
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>

#include "drivers.h"
#include "status.h"

namespace rab {



namespace {

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ bool wait_ge(const uint64_t* flag, uint64_t target, DeviceStatus* st, uint32_t detail,
                        uint64_t timeout_ns) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t t0 = now_ns();
  while (true) {
    __nanosleep(32);
    if (ld_acquire_sys(flag) >= target) return true;
    if (st_read_error(st) != 0) return false;
    if (now_ns() - t0 > timeout_ns) {
      st_record_timeout(st, kSiteRingFlag, detail);
      return false;
    }
  }
}

__global__ void __launch_bounds__(512) p2p_ring_kernel(const RingCopyParams p) {
  const int c = blockIdx.x;
  const size_t n16 = p.bytes / 16;
  const size_t per = (n16 + gridDim.x - 1) / gridDim.x;
  const size_t beg = per * c;
  const size_t end = beg + per < n16 ? beg + per : n16;
  __shared__ int s_ok;
  for (int s = 0; s < p.nsteps; ++s) {
    const uint64_t seq = p.base + s;  // steps completed before this one
    const int sg = p.first_step + s;  // ring step index
    if (threadIdx.x == 0) {
      bool ok = true;
      if (sg > 0) ok = wait_ge(p.arrived_local + c, seq, p.status, (uint32_t)s, p.timeout_ns);
      if (ok) ok = wait_ge(p.sent_right + c, seq, p.status, 0x10000u | (uint32_t)s, p.timeout_ns);
      s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const uint4* src = reinterpret_cast<const uint4*>(p.buf[sg & 1]);
    uint4* dst = reinterpret_cast<uint4*>(p.right_buf[(sg + 1) & 1]);
    constexpr int U = 4;
    size_t i = beg + threadIdx.x;
    for (; i + (U - 1) * blockDim.x < end; i += U * blockDim.x) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) r[u] = __ldcg(src + i + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < U; ++u) dst[i + u * blockDim.x] = r[u];
    }
    for (; i < end; i += blockDim.x) dst[i] = __ldcg(src + i);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.arrived_right + c)
                   : "memory");
      asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.sent_local + c), "l"(seq + 1)
                   : "memory");
    }
  }
}

}  // namespace

int p2p_ring_launch(const RingCopyParams& p, int slices, cudaStream_t stream) {
  if (p.bytes % 16 != 0) throw std::runtime_error("p2p ring: bytes must be a multiple of 16");
  if (p.nsteps <= 0) return 0;
  void* args[] = {const_cast<RingCopyParams*>(&p)};
  // cooperative launch: every slice's CTA must be resident at once
  return static_cast<int>(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(p2p_ring_kernel),
                                                      dim3(slices), dim3(512), args, 0, stream));
}

}  // namespace rab
