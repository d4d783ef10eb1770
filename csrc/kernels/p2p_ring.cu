// p2p_ring.cu - comm-only ring rotation over NVLink peer memory, all np-1 steps
// in one launch (the `b200_fused` comm backend).
//
// Same data movement as the reference loops (src/loop/ring_loop_*.cu: every
// step sends the current shard to rank+1 and receives the next one from
// rank-1, two buffers swapped per step) but with no library call.  The shard
// is cut into 8 KiB chunks dealt round-robin to the CTAs (CTA c of G owns
// chunks c, c+G, c+2G, ...: at any moment the G CTAs write neighbouring
// addresses, which measured ~5 % faster over NVLink on B200 than one
// contiguous slice per CTA, and no CTA holds more than one chunk over
// another).  Each CTA pushes its chunks into the right neighbour's receive
// buffer and hands over with two monotonically increasing flags per CTA:
//   arrived[c] (in the receiver's memory)  step n of CTA c's chunks has landed
//   sent[c]    (in the sender's memory)    the sender finished reading them
// so each CTA runs its own pipeline and no grid-wide barrier is needed.  All
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

constexpr int kVecThreads = 512;
constexpr int kVecUnroll = 4;                                   // chunks in flight per thread
constexpr size_t kVecChunk16 = static_cast<size_t>(kVecThreads);  // one vector per thread

// 16-byte (uint4) or 32-byte (sm_100 256-bit ld/st) vectors
struct alignas(32) Vec32 {
  uint32_t w[8];
};

__device__ __forceinline__ uint4 ld_vec(const uint4* p) { return __ldcg(p); }
__device__ __forceinline__ void st_vec(uint4* p, const uint4& v) { *p = v; }
__device__ __forceinline__ Vec32 ld_vec(const Vec32* p) {
  Vec32 r;
  asm volatile("ld.global.cg.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]), "=r"(r.w[4]),
                 "=r"(r.w[5]), "=r"(r.w[6]), "=r"(r.w[7])
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_vec(Vec32* p, const Vec32& v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]),
               "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]),
               "r"(v.w[7])
               : "memory");
}

// Chunks of kVecThreads vectors (8 KiB with 16-byte vectors, 16 KiB with 32-byte ones).
//
// kPull: the rank reads the left neighbour's buffer over NVLink and writes its
// own (instead of writing the right neighbour's), and both flags of a step
// live in the waiting rank's memory, so every poll is a local load:
//   arrived[c]  bumped by the left neighbour once its buffer holds the data
//               this rank pulls next (it finished its own previous step)
//   sent[c]     bumped by the right neighbour once it finished reading the
//               buffer this rank is about to overwrite
// The counts match the push protocol's, step for step.
template <typename V, bool kPull>
__global__ void __launch_bounds__(kVecThreads) p2p_ring_kernel(const RingCopyParams p) {
  const int c = blockIdx.x;
  const size_t n16 = p.bytes / sizeof(V);
  const size_t stride16 = kVecChunk16 * gridDim.x;
  __shared__ int s_ok;
  for (int s = 0; s < p.nsteps; ++s) {
    const uint64_t seq = p.base + s;  // steps completed before this one
    const int sg = p.first_step + s;  // ring step index
    if (threadIdx.x == 0) {
      bool ok = true;
      if (sg > 0) ok = wait_ge(p.arrived_local + c, seq, p.status, (uint32_t)s, p.timeout_ns);
      if (ok)
        ok = wait_ge(kPull ? p.sent_local + c : p.sent_right + c, seq, p.status,
                     0x10000u | (uint32_t)s, p.timeout_ns);
      s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const V* src = reinterpret_cast<const V*>(kPull ? p.left_buf[sg & 1] : p.buf[sg & 1]);
    V* dst = reinterpret_cast<V*>(kPull ? p.buf[(sg + 1) & 1] : p.right_buf[(sg + 1) & 1]);
    // chunks c, c + G, c + 2G, ... (one vector per thread), kVecUnroll of them
    // in flight; the CTAs' shares differ by one chunk at most
    size_t base = kVecChunk16 * c;
    for (; base + (kVecUnroll - 1) * stride16 + kVecChunk16 <= n16; base += kVecUnroll * stride16) {
      const size_t i = base + threadIdx.x;
      V r[kVecUnroll];
#pragma unroll
      for (int u = 0; u < kVecUnroll; ++u) r[u] = ld_vec(src + i + u * stride16);
#pragma unroll
      for (int u = 0; u < kVecUnroll; ++u) st_vec(dst + i + u * stride16, r[u]);
    }
    for (; base < n16; base += stride16) {
      const size_t i = base + threadIdx.x;
      if (i < n16) st_vec(dst + i, ld_vec(src + i));
    }
    // The barrier orders every thread's stores before thread 0's system-scope
    // release, and release is cumulative, so the neighbour that acquires
    // arrived[c] sees the whole chunk set.  (A per-thread system fence here
    // measured 9-13 us slower per 64 MiB launch on B200.)
    __syncthreads();
    if (threadIdx.x == 0) {
      // push: the data landed in the right neighbour's buffer, and this rank
      // finished reading its own; pull: this rank's buffer holds the right
      // neighbour's next data, and the left neighbour's buffer was read
      asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.arrived_right + c)
                   : "memory");
      if constexpr (kPull)
        asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.sent_left + c)
                     : "memory");
      else
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.sent_local + c), "l"(seq + 1)
                     : "memory");
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk variant: one elected thread per CTA streams its chunks through a
// 4-stage shared-memory ring with the TMA bulk engine: bulk loads of the local
// buffer into shared memory run up to four chunks ahead (completion on an
// mbarrier per stage), each landed chunk is bulk-stored into the right
// neighbour's buffer, and a stage is refilled once its store has read it.
// Only stores touch peer memory; loads read this GPU's own buffer.
// ---------------------------------------------------------------------------
constexpr int kBulkStages = 4;
constexpr uint32_t kBulkChunk = 32768;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, DeviceStatus* st,
                                         uint64_t timeout_ns) {
  const uint64_t t0 = now_ns();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (st_read_error(st) != 0) return false;
    if (now_ns() - t0 > timeout_ns) {
      st_record_timeout(st, kSiteCopySlice, 0);
      return false;
    }
  }
}

__device__ __forceinline__ void bulk_load(uint8_t* sdst, const uint8_t* gsrc, uint32_t n,
                                          uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(n)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(sdst)),
      "l"(gsrc), "r"(n), "r"(smem_addr(bar))
      : "memory");
}

__global__ void __launch_bounds__(32) p2p_ring_bulk_kernel(const RingCopyParams p) {
  extern __shared__ __align__(128) uint8_t stage_buf[];
  __shared__ __align__(8) uint64_t bars[kBulkStages];
  if (threadIdx.x != 0) return;
  const size_t c = blockIdx.x;
  const size_t G = gridDim.x;
  const size_t n_chunks = (p.bytes + kBulkChunk - 1) / kBulkChunk;
  // this CTA's chunks: c, c + G, ...
  const int mine = c < n_chunks ? static_cast<int>((n_chunks - 1 - c) / G + 1) : 0;
  auto chunk_off = [&](int k) { return (c + static_cast<size_t>(k) * G) * kBulkChunk; };
  auto chunk_len = [&](int k) {
    const size_t off = chunk_off(k);
    return static_cast<uint32_t>(p.bytes - off < kBulkChunk ? p.bytes - off : kBulkChunk);
  };
  for (int i = 0; i < kBulkStages; ++i)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bars[i])) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  uint32_t uses[kBulkStages] = {0, 0, 0, 0};
  for (int s = 0; s < p.nsteps; ++s) {
    const uint64_t seq = p.base + s;
    const int sg = p.first_step + s;
    if (sg > 0 && !wait_ge(p.arrived_local + c, seq, p.status, (uint32_t)s, p.timeout_ns)) return;
    if (!wait_ge(p.sent_right + c, seq, p.status, 0x10000u | (uint32_t)s, p.timeout_ns)) return;
    // data this rank received last step (written by the peer's bulk stores) is
    // read below by the bulk engine: order it after the flag acquire
    asm volatile("fence.proxy.async.global;" ::: "memory");
    const uint8_t* src = p.buf[sg & 1];
    uint8_t* dst = p.right_buf[(sg + 1) & 1];
    int loaded = 0;
    for (; loaded < kBulkStages && loaded < mine; ++loaded)
      bulk_load(stage_buf + loaded * kBulkChunk, src + chunk_off(loaded), chunk_len(loaded),
                &bars[loaded]);
    for (int k = 0; k < mine; ++k) {
      const int st = k % kBulkStages;
      uint8_t* sb = stage_buf + st * kBulkChunk;
      if (!bar_wait(&bars[st], uses[st] & 1, p.status, p.timeout_ns)) {
        // unwind: let this CTA's bulk stores finish and give the loads still in
        // flight a bounded chance to land before shared memory is released
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        for (int j = k; j < loaded; ++j) {
          const int sj = j % kBulkStages;
          bar_wait(&bars[sj], uses[sj] & 1, nullptr, 100000000ull);
          ++uses[sj];
        }
        return;
      }
      ++uses[st];
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                       dst + chunk_off(k)),
                   "r"(smem_addr(sb)), "r"(chunk_len(k))
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      if (loaded < mine) {
        // refill this stage once the store just issued has read it
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        bulk_load(sb, src + chunk_off(loaded), chunk_len(loaded), &bars[st]);
        ++loaded;
      }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence_system();
    asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.arrived_right + c) : "memory");
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.sent_local + c), "l"(seq + 1)
                 : "memory");
  }
}

}  // namespace

int p2p_ring_launch(const RingCopyParams& p, int slices, cudaStream_t stream) {
  if (p.bytes % 16 != 0) throw std::runtime_error("p2p ring: bytes must be a multiple of 16");
  if (p.nsteps <= 0) return 0;
  // Slice c only waits on slice c of the neighbours, so the CTAs need not be
  // co-resident: a regular launch cannot deadlock.
  if (p.mode == 1) {
    const int smem = kBulkStages * kBulkChunk;
    // the attribute is per device; set it on every launch (a cheap host call)
    const cudaError_t e = cudaFuncSetAttribute(
        p2p_ring_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    p2p_ring_bulk_kernel<<<slices, 32, smem, stream>>>(p);
  } else if (p.mode == 2 && p.bytes % 32 == 0) {
    p2p_ring_kernel<Vec32, false><<<slices, kVecThreads, 0, stream>>>(p);
  } else if (p.mode == 3) {
    p2p_ring_kernel<uint4, true><<<slices, kVecThreads, 0, stream>>>(p);
  } else {
    p2p_ring_kernel<uint4, false><<<slices, kVecThreads, 0, stream>>>(p);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rab
