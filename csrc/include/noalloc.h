// noalloc.h - allocation-free C entry point of the bf16 flash-attention forward.
//
// This entry point has no counterpart in the reference benchmark suite; it is
// an addition of this library.
//
// Who needs it: callers that may not allocate device memory at the point they
// run attention - for example a plugin running inside another runtime's
// enqueue/execute callback with a fixed memory budget, or C code without a
// device allocator of its own.  The regular entry points take their split-KV
// workspace from the caller's allocator; this one uses a fixed scratch array
// compiled into the library instead (a file-scope __device__ array of
// RAB_NOALLOC_SCRATCH_BYTES bytes, held on every GPU that loads the library
// until the process exits).
//
// Contract:
//  * inputs and outputs stay the caller's: q [Sq, Hq, D], k / v [Skv, Hkv, D],
//    out [Sq, Hq, D], all bf16, contiguous, on the current device; lse
//    [Sq, Hq] fp32 or NULL.  D is 64 or 128, Sq a multiple of 128, Skv a
//    multiple of 128, Hq a multiple of Hkv.
//  * nsplit = 0 picks an equal KV split from the wave cost model (the
//    regular entry point may pick its balanced or causal-aware schedule
//    instead; the results agree within bf16 rounding).  A problem whose split
//    workspace exceeds the scratch array is rejected with
//    RAB_NOALLOC_ERR_TOO_LARGE and a message in `err` - it is not shrunk.
//  * no cudaMalloc, cudaFree or allocating library call is made.  The first
//    call on a device resolves the scratch array's device address once
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before capturing a stream.
//  * every call shares the one scratch array.  Calls whose kernels overlap on
//    the GPU (different streams, no ordering between them) race on it; order
//    them on one stream or with events.
//  * the launch is asynchronous on `stream`; 0 means the work was queued.
//    Every wait inside the kernel is bounded: if one runs out, the kernel
//    records the error in a status word (also in the scratch array) and
//    returns, leaving `out` undefined.  Check it with
//    rab_flash_attention_noalloc_status once the work is due: it waits for
//    `stream` and returns RAB_NOALLOC_ERR_DEVICE (with the wait site in `err`
//    and, when `info` is not NULL, code / site / block / detail in info[0..3])
//    if the last call on this device failed on the GPU.  The status word is
//    cleared at the start of every call, so read it before the next one.
//  * rab_flash_attention_noalloc_wait_selftest runs one bounded wait on a
//    flag that nothing sets against the same status word, so a caller can see
//    how a device-side timeout surfaces (the status call then reports it);
//    timeout_s is in (0, 5].
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#define RAB_NOALLOC_SCRATCH_BYTES (32u << 20) /* 32 MiB */

#define RAB_NOALLOC_OK 0
#define RAB_NOALLOC_ERR_ARGS (-1)
#define RAB_NOALLOC_ERR_TOO_LARGE (-2)
#define RAB_NOALLOC_ERR_CUDA (-3)
#define RAB_NOALLOC_ERR_DEVICE (-4) /* the kernel reported an error in its status word */

#ifdef __cplusplus
extern "C" {
#endif

int rab_flash_attention_noalloc(const void* q, const void* k, const void* v, void* out,
                                float* lse, int Sq, int Skv, int Hq, int Hkv, int D, float scale,
                                int causal, int nsplit, cudaStream_t stream, char* err,
                                size_t err_len);

int rab_flash_attention_noalloc_status(cudaStream_t stream, unsigned int* info, char* err,
                                       size_t err_len);

int rab_flash_attention_noalloc_wait_selftest(double timeout_s, cudaStream_t stream, char* err,
                                              size_t err_len);

#ifdef __cplusplus
}
#endif
