// status.h - device status word shared by every kernel that waits on anything.
//
// Waits in this code base are bounded: when a wait runs out it records an error
// code, the wait site and the block/rank that gave up, then the kernel unwinds
// normally.  The host reads the word after the launch and raises a clean error;
// the CUDA context stays usable.  No kernel traps.
#pragma once

#include <cstdint>

namespace rab {

enum StatusCode : uint32_t {
  kStatusOk = 0,
  kStatusTimeout = 1,     // a bounded wait ran out
  kStatusBadArgs = 2,     // device-side argument check failed
  kStatusBounds = 3,      // DEBUG_BOUNDS index check failed
  kStatusPeerError = 4,   // a peer rank published an error flag
};

// Wait-site identifiers (reported as `where`).
enum WaitSite : uint32_t {
  kSiteNone = 0,
  kSiteQFull = 1,
  kSiteKFull = 2,
  kSiteVFull = 3,
  kSiteKEmpty = 4,
  kSiteVEmpty = 5,
  kSiteSFull = 6,
  kSitePFull = 7,
  kSiteOReady = 8,
  kSiteBlockReady = 9,     // waiting for a ring block to land in local memory
  kSitePeerReady = 10,     // waiting for a peer's published epoch
  kSitePeerConsumed = 11,  // waiting for peers to finish reading our buffers
  kSiteCopySlice = 12,
  kSiteRingFlag = 13,      // comm-only ring copy flag
  kSiteTest = 14,          // deliberately unsatisfiable wait used by tests
  kSitePvDone = 15,
  kSiteItemQueue = 16,     // flash kernel's in-CTA work-item queue
};

// Sites of the RAB_DEBUG_BOUNDS index checks (reported as `where` with kStatusBounds).
enum BoundsSite : uint32_t {
  kBoundsQRow = 101,       // query row of a work item (Q load, output write)
  kBoundsRecord = 102,     // split partial record written by a work item
  kBoundsMergeRecord = 103,  // split partial record read by a merge kernel
};

struct DeviceStatus {
  uint32_t code;       // StatusCode, first error wins
  uint32_t where;      // WaitSite of the first error
  uint32_t block;      // blockIdx.x that recorded it
  uint32_t detail;     // site-specific (step, tile, peer...)
  uint32_t n_errors;   // how many threads/blocks hit an error
  // [0] work-item claim counter and [1] finished-CTA counter of the flash
  // kernel's dynamic schedule; zero between launches (the last CTA resets
  // them), so one status block serves one launch at a time.
  uint32_t pad[3];
};

#ifdef __CUDACC__
__device__ __forceinline__ uint32_t st_read_error(DeviceStatus* st) {
  if (st == nullptr) return 0;
  return *reinterpret_cast<volatile uint32_t*>(&st->code);
}

__device__ __forceinline__ void st_record(DeviceStatus* st, uint32_t code, uint32_t where,
                                          uint32_t detail = 0) {
  if (st == nullptr) return;
  atomicAdd(&st->n_errors, 1u);
  if (atomicCAS(&st->code, 0u, code) == 0u) {
    st->where = where;
    st->block = blockIdx.x;
    st->detail = detail;
    __threadfence_system();
  }
}

__device__ __forceinline__ void st_record_timeout(DeviceStatus* st, uint32_t where,
                                                  uint32_t detail = 0) {
  st_record(st, kStatusTimeout, where, detail);
}

// Index check of a computed global access.  Builds with RAB_DEBUG_BOUNDS
// evaluate `ok`; when it is false they record kStatusBounds (`where` = the
// BoundsSite, `detail` = the offending index) and return false so the caller
// skips the access.  Default builds compile the check to `true`.
__device__ __forceinline__ bool st_bounds(DeviceStatus* st, bool ok, uint32_t where,
                                          uint32_t detail) {
#ifdef RAB_DEBUG_BOUNDS
  if (!ok) st_record(st, kStatusBounds, where, detail);
  return ok;
#else
  (void)st, (void)ok, (void)where, (void)detail;
  return true;
#endif
}
#endif

}  // namespace rab
