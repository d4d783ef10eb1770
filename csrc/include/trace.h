// trace.h - NVTX ranges around the host-side phases (ring-format, fused
// launch, comm repetitions, attention iterations), so a timeline profiler
// shows them next to the kernels.  NVTX v3 is header-only: without a profiler
// attached each range costs a few nanoseconds and nothing is recorded.
// Build with -DRAB_NO_NVTX to compile the ranges out.
#pragma once

#ifndef RAB_NO_NVTX
#include <nvtx3/nvToolsExt.h>
#endif

namespace rab {

class TraceRange {
 public:
  explicit TraceRange(const char* name) {
#ifndef RAB_NO_NVTX
    nvtxRangePushA(name);
#else
    (void)name;
#endif
  }
  ~TraceRange() {
#ifndef RAB_NO_NVTX
    nvtxRangePop();
#endif
  }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

}  // namespace rab
