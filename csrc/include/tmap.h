// tmap.h - host-side creation of TMA tensor maps (CUtensorMap) through the
// driver entry point, so the extension does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cstdint>
#include <string>

namespace rab {

enum class TmapDtype { kBF16, kF32 };

// Encode a tiled tensor map of rank `rank` (1..5).  dims[0] is the innermost
// (contiguous) dimension.  strides_bytes has rank-1 entries: the byte stride of
// dims[1..rank-1].  box[i] elements are copied per load along dims[i].
// Throws std::runtime_error with the driver's message on failure.  Checks the
// rules the driver does not: the innermost box extent times the element size
// must be a multiple of 16 bytes and, for 128-byte swizzle, exactly 128 bytes
// or less.
CUtensorMap make_tmap(const void* base, TmapDtype dtype, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

std::string tmap_describe(int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                          const uint32_t* box);

}  // namespace rab
