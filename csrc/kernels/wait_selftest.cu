// wait_selftest.cu - exercises the bounded-wait path on the GPU without any
// fault: one thread waits for a flag word that nothing ever sets, gives up after
// `timeout_ns` of globaltimer time, records the timeout in the status word and
// returns normally.  The host then reads the status and keeps using the context.
#include <cuda_runtime.h>

#include <cstdint>

#include "status.h"

namespace rab {

namespace {

__global__ void wait_selftest_kernel(const volatile uint64_t* flag, uint64_t target,
                                     uint64_t timeout_ns, DeviceStatus* st) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (*flag < target) {
    __nanosleep(1000);
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > timeout_ns) {
      st_record_timeout(st, kSiteTest, 0);
      return;
    }
  }
}

}  // namespace

int wait_selftest_launch(const uint64_t* flag, uint64_t target, uint64_t timeout_ns,
                         DeviceStatus* st, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 1, 0, stream>>>(flag, target, timeout_ns, st);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rab
