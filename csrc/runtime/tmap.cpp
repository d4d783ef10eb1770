// tmap.cpp - TMA tensor-map encoding via cudaGetDriverEntryPoint.
#include "tmap.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>
#include "strfmt.h"
#include <stdexcept>

namespace rab {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      fn = nullptr;
      return;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (fn == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
  return fn;
}

}  // namespace

std::string tmap_describe(int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                          const uint32_t* box) {
  std::string s = strfmt("rank=%d dims=[", rank);
  for (int i = 0; i < rank; ++i) s += strfmt(i ? ",%llu" : "%llu", (unsigned long long)dims[i]);
  s += "] strides=[";
  for (int i = 0; i + 1 < rank; ++i)
    s += strfmt(i ? ",%llu" : "%llu", (unsigned long long)strides_bytes[i]);
  s += "] box=[";
  for (int i = 0; i < rank; ++i) s += strfmt(i ? ",%u" : "%u", box[i]);
  return s + "]";
}

CUtensorMap make_tmap(const void* base, TmapDtype dtype, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  if (rank < 1 || rank > 5) throw std::runtime_error("make_tmap: rank must be 1..5");
  const uint32_t esize = dtype == TmapDtype::kBF16 ? 2u : 4u;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    throw std::runtime_error("make_tmap: base address not 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0)
      throw std::runtime_error("make_tmap: stride not a multiple of 16 bytes: " +
                               tmap_describe(rank, dims, strides_bytes, box));
  if ((box[0] * esize) % 16 != 0)
    throw std::runtime_error("make_tmap: inner box extent not a multiple of 16 bytes");
  if (swizzle == CU_TENSOR_MAP_SWIZZLE_128B && box[0] * esize > 128)
    throw std::runtime_error("make_tmap: inner box wider than the 128-byte swizzle span");

  cuuint64_t gdims[5];
  cuuint64_t gstrides[4];
  cuuint32_t bdims[5];
  cuuint32_t estrides[5];
  for (int i = 0; i < rank; ++i) {
    gdims[i] = dims[i];
    bdims[i] = box[i];
    estrides[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstrides[i] = strides_bytes[i];

  CUtensorMap map;
  CUresult res = get_encode_fn()(
      &map,
      dtype == TmapDtype::kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
      static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdims, gstrides, bdims, estrides,
      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) {
    throw std::runtime_error(strfmt("cuTensorMapEncodeTiled failed (%d): %s",
                                    static_cast<int>(res),
                                    tmap_describe(rank, dims, strides_bytes, box).c_str()));
  }
  return map;
}

}  // namespace rab
