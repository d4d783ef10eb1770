// noalloc_entry.cu - allocation-free C entry point of the bf16 flash forward
// (declared and documented in noalloc.h; no counterpart in the reference).
//
// The split-KV partials and the device status word live in one file-scope
// __device__ array.  Host code must not pass the array's name to a kernel (in
// host code it is only a stand-in symbol, not a device address); the device
// address is resolved once per device with cudaGetSymbolAddress and cached.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>
#include <mutex>

#include "flash.h"
#include "noalloc.h"

namespace rab {
int wait_selftest_launch(const uint64_t* flag, uint64_t target, uint64_t timeout_ns,
                         DeviceStatus* st, cudaStream_t stream);
}

namespace {

// [0, 32): DeviceStatus of the last call; [64, 72): the flag word of the
// bounded-wait self-test (nothing ever sets it); [256, end): split partials
// (acc [items][128][D], then m [items][128], then l [items][128]).
static __device__ __align__(256) unsigned char g_noalloc_scratch[RAB_NOALLOC_SCRATCH_BYTES];
constexpr size_t kStatusBytes = 256;
constexpr size_t kSelftestFlag = 64;
constexpr int kMaxDevices = 64;

void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

void set_err(char* err, size_t len, const char* fmt, ...) {
  if (err == nullptr || len == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, len, fmt, ap);
  va_end(ap);
}

// Device address of the scratch array on the current device, resolved once
// per device with that device current (host code only holds a stand-in for
// the symbol).  RAB_NOALLOC_OK or an error code with the message in `err`.
int scratch_base(void** base, char* err, size_t err_len) {
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_err(err, err_len, "no usable current device (%s)", cudaGetErrorString(ce));
    return RAB_NOALLOC_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    ce = cudaGetSymbolAddress(&g_scratch_addr[dev], g_noalloc_scratch);
    if (ce != cudaSuccess) {
      g_scratch_addr[dev] = nullptr;
      set_err(err, err_len, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(ce));
      return RAB_NOALLOC_ERR_CUDA;
    }
  }
  *base = g_scratch_addr[dev];
  return RAB_NOALLOC_OK;
}

const char* code_name(uint32_t code) {
  switch (code) {
    case rab::kStatusTimeout: return "a bounded wait timed out";
    case rab::kStatusBadArgs: return "the kernel refused its arguments";
    case rab::kStatusBounds: return "an index check failed";
    case rab::kStatusPeerError: return "a peer reported an error";
    default: return "unknown error";
  }
}

}  // namespace

extern "C" int rab_flash_attention_noalloc(const void* q, const void* k, const void* v, void* out,
                                           float* lse, int Sq, int Skv, int Hq, int Hkv, int D,
                                           float scale, int causal, int nsplit,
                                           cudaStream_t stream, char* err, size_t err_len) {
  using namespace rab;
  if (err != nullptr && err_len > 0) err[0] = '\0';
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) {
    set_err(err, err_len, "q, k, v and out must be device pointers");
    return RAB_NOALLOC_ERR_ARGS;
  }
  if ((D != 64 && D != 128) || Sq <= 0 || Sq % 128 != 0 || Skv <= 0 || Skv % 128 != 0 ||
      Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || nsplit < 0 || (causal && Sq != Skv)) {
    set_err(err, err_len,
            "unsupported shape: D=%d (64|128), Sq=%d and Skv=%d (multiples of 128, equal when "
            "causal), Hq=%d a multiple of Hkv=%d, nsplit=%d >= 0",
            D, Sq, Skv, Hq, Hkv, nsplit);
    return RAB_NOALLOC_ERR_ARGS;
  }
  void* base = nullptr;
  const int rb = scratch_base(&base, err, err_len);  // once per device: the symbol's address
  if (rb != RAB_NOALLOC_OK) return rb;
  cudaError_t ce = cudaSuccess;

  const int sms = flash_sm_count();
  const int units = Hq * (Sq / 128);
  const int tiles = Skv / 128;
  int ns = nsplit > 0 ? nsplit : flash_choose_split(units, tiles, sms, 3);
  if (ns > tiles) ns = tiles;
  const int items = units * ns;
  const size_t need = ns > 1 ? static_cast<size_t>(items) * 128 * (D + 2) * sizeof(float) : 0;
  const size_t have = RAB_NOALLOC_SCRATCH_BYTES - kStatusBytes;
  if (need > have) {
    set_err(err, err_len,
            "problem needs %zu bytes of split-KV scratch (nsplit=%d, %d work items) but the "
            "static scratch array holds %zu bytes; use the allocating entry point or a smaller "
            "problem",
            need, ns, items, have);
    return RAB_NOALLOC_ERR_TOO_LARGE;
  }

  try {
    const FlashMaps maps = flash_make_maps(Prec::kBF16, k, v, 0, 1, Skv, Hkv, D);
    FlashParams p;
    std::memset(&p, 0, sizeof(p));
    p.q = q;
    p.Sq = Sq;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.D = D;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.nblk = 1;
    p.Skv = Skv;
    p.causal = causal ? 1 : 0;
    p.world = 1;
    p.nsplit = ns;
    p.rows_per_unit = 128;  // one query tile per work unit
    p.n_units = units;
    p.n_items = items;
    p.out = out;
    p.out_bf16 = 1;
    p.lse = lse;
    unsigned char* b = static_cast<unsigned char*>(base);
    p.status = reinterpret_cast<DeviceStatus*>(b);
    if (ns > 1) {
      float* ws = reinterpret_cast<float*>(b + kStatusBytes);
      p.split_acc = ws;
      p.split_m = ws + static_cast<size_t>(items) * 128 * D;
      p.split_l = p.split_m + static_cast<size_t>(items) * 128;
    }
    p.timeout_ns = 10ull * 1000000000ull;
    // the status word must start at zero; the partials are fully rewritten
    ce = cudaMemsetAsync(p.status, 0, sizeof(DeviceStatus), stream);
    if (ce != cudaSuccess) {
      set_err(err, err_len, "cudaMemsetAsync(status) failed: %s", cudaGetErrorString(ce));
      return RAB_NOALLOC_ERR_CUDA;
    }
    int rc = flash_forward_launch(Prec::kBF16, p, maps, items < sms ? items : sms, false, stream);
    if (rc == 0 && ns > 1) rc = flash_split_merge_launch(p, stream);
    if (rc != 0) {
      set_err(err, err_len, "launch failed: %s", cudaGetErrorString(static_cast<cudaError_t>(rc)));
      return RAB_NOALLOC_ERR_CUDA;
    }
  } catch (const std::exception& e) {
    set_err(err, err_len, "%s", e.what());
    return RAB_NOALLOC_ERR_ARGS;
  }
  return RAB_NOALLOC_OK;
}

extern "C" int rab_flash_attention_noalloc_status(cudaStream_t stream, unsigned int* info,
                                                  char* err, size_t err_len) {
  using namespace rab;
  if (err != nullptr && err_len > 0) err[0] = '\0';
  void* base = nullptr;
  const int rb = scratch_base(&base, err, err_len);
  if (rb != RAB_NOALLOC_OK) return rb;
  DeviceStatus s;
  std::memset(&s, 0, sizeof(s));
  // 32 bytes into this stack copy: the driver stages pageable copies through
  // its own buffers, nothing is allocated here
  cudaError_t ce = cudaMemcpyAsync(&s, base, sizeof(s), cudaMemcpyDeviceToHost, stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(stream);
  if (ce != cudaSuccess) {
    set_err(err, err_len, "reading the status word failed: %s", cudaGetErrorString(ce));
    return RAB_NOALLOC_ERR_CUDA;
  }
  if (info != nullptr) {
    info[0] = s.code;
    info[1] = s.where;
    info[2] = s.block;
    info[3] = s.detail;
  }
  if (s.code != kStatusOk) {
    set_err(err, err_len,
            "device error %u (%s) at wait site %u, block %u, detail %u; the output of that call "
            "is not valid",
            s.code, code_name(s.code), s.where, s.block, s.detail);
    return RAB_NOALLOC_ERR_DEVICE;
  }
  return RAB_NOALLOC_OK;
}

extern "C" int rab_flash_attention_noalloc_wait_selftest(double timeout_s, cudaStream_t stream,
                                                         char* err, size_t err_len) {
  using namespace rab;
  if (err != nullptr && err_len > 0) err[0] = '\0';
  if (!(timeout_s > 0.0 && timeout_s <= 5.0)) {
    set_err(err, err_len, "timeout_s must be in (0, 5] (got %g)", timeout_s);
    return RAB_NOALLOC_ERR_ARGS;
  }
  void* base = nullptr;
  const int rb = scratch_base(&base, err, err_len);
  if (rb != RAB_NOALLOC_OK) return rb;
  // status and flag start at zero; the flag stays zero, so the wait runs out
  cudaError_t ce = cudaMemsetAsync(base, 0, kStatusBytes, stream);
  if (ce != cudaSuccess) {
    set_err(err, err_len, "cudaMemsetAsync(status) failed: %s", cudaGetErrorString(ce));
    return RAB_NOALLOC_ERR_CUDA;
  }
  unsigned char* b = static_cast<unsigned char*>(base);
  const int rc = wait_selftest_launch(reinterpret_cast<const uint64_t*>(b + kSelftestFlag), 1,
                                      static_cast<uint64_t>(timeout_s * 1e9),
                                      reinterpret_cast<DeviceStatus*>(b), stream);
  if (rc != 0) {
    set_err(err, err_len, "launch failed: %s", cudaGetErrorString(static_cast<cudaError_t>(rc)));
    return RAB_NOALLOC_ERR_CUDA;
  }
  return RAB_NOALLOC_OK;
}
