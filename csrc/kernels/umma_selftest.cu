// umma_selftest.cu - one-tile tcgen05 GEMMs that exercise every operand
// arrangement the attention kernels use, so descriptor or layout mistakes show
// up as a clean numerical mismatch in a unit test instead of inside the fused
// kernel:
//   * A from shared memory, K-major, 128-byte swizzle (Q in QK^T)
//   * A from tensor memory (P in PV, Q when staged in TMEM)
//   * B K-major (K in QK^T) and B MN-major (V in PV)
//   * kind::f16 with bf16 inputs and kind::tf32 with fp32 inputs
// D (128 x N, fp32) is read back from TMEM with tcgen05.ld.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100.cuh"
#include "tmap.h"

namespace rab {

using namespace sm100;

namespace {

constexpr int kM = 128;
constexpr int kMaxN = 128;
constexpr int kMaxK = 128;

// smem: A up to 128 x 128 x 4 = 64 KB, B up to 128 x 128 x 4 = 64 KB
constexpr int kSmemA = kM * kMaxK * 4;
constexpr int kSmemB = kMaxN * kMaxK * 4;
constexpr int kSmemBytes = kSmemA + kSmemB + 1024 /*align*/ + 64;

template <bool kTF32>
__global__ void __launch_bounds__(128, 1)
    umma_selftest_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB, const uint32_t* a_rows,
                         float* d_out, int N, int K, int a_in_tmem, int b_mn_major,
                         DeviceStatus* st) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kSmemA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kSmemB);  // [0] tma, [1] mma
  __shared__ uint32_t tmem_base_slot;

  constexpr uint32_t esize = kTF32 ? 4 : 2;
  constexpr uint32_t elems128 = 128 / esize;  // elements per 128-byte row
  const uint32_t warp = warp_id();
  const uint32_t tid = threadIdx.x;

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base_slot, 256);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_slot;
  const uint32_t d_col = 0;       // D: columns [0, N)
  const uint32_t a_col = kMaxN;   // A (TMEM variant): columns [128, 128 + K*esize/4)

  // --- stage A in TMEM (each thread owns row tid) ---
  if (a_in_tmem) {
    const int ncols = K * esize / 4;
    const uint32_t* row = a_rows + static_cast<size_t>(tid) * ncols;
    uint32_t v[16];
    for (int c = 0; c < ncols; c += 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = row[c + i];
      tmem_st16(tmem_addr(tmem, warp * 32, a_col + c), v);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // --- TMA loads + MMAs from one thread ---
  if (tid == 0) {
    const uint32_t a_sub = K / elems128;  // 128-byte K subtiles of A (and K-major B)
    uint32_t bytes = 0;
    if (!a_in_tmem) bytes += kM * K * esize;
    bytes += N * K * esize;
    mbar_arrive_expect_tx(&bars[0], bytes);
    if (!a_in_tmem) {
      for (uint32_t s = 0; s < a_sub; ++s)
        tma_load_3d(sA + s * kM * 128, &tmA, &bars[0], s * elems128, 0, 0);
    }
    if (!b_mn_major) {
      for (uint32_t s = 0; s < a_sub; ++s)
        tma_load_3d(sB + s * N * 128, &tmB, &bars[0], s * elems128, 0, 0);
    } else {
      const uint32_t n_sub = N / elems128;  // 128-byte N blocks
      for (uint32_t s = 0; s < n_sub; ++s)
        tma_load_3d(sB + s * K * 128, &tmB, &bars[0], s * elems128, 0, 0);
    }
  }
  if (!mbar_wait(&bars[0], 0, st, kSiteTest, 2000000000ull)) goto done;

  if (tid == 0) {
    tc_fence_after();
    const uint32_t idesc = make_idesc(kTF32 ? kFmtTF32 : kFmtBF16, kTF32 ? kFmtTF32 : kFmtBF16,
                                      kM, N, kMajorK, b_mn_major ? kMajorMN : kMajorK);
    const uint32_t ksteps = K * esize / 32;  // each MMA consumes 32 bytes of K
    for (uint32_t ks = 0; ks < ksteps; ++ks) {
      const uint32_t kbyte = ks * 32;
      const uint32_t sub = kbyte / 128, inner = kbyte % 128;
      uint64_t bdesc;
      if (!b_mn_major) {
        bdesc = make_sdesc(smem_u32(sB) + sub * N * 128 + inner, 16, 1024);
      } else {
        const uint32_t rows_per_step = 32 / esize;  // K rows consumed by one MMA
        bdesc = make_sdesc(smem_u32(sB) + ks * rows_per_step * 128, K * 128, 1024);
      }
      if (a_in_tmem) {
        mma_ts<kTF32>(tmem + d_col, tmem + a_col + ks * 8, bdesc, idesc, ks > 0 ? 1u : 0u);
      } else {
        const uint64_t adesc = make_sdesc(smem_u32(sA) + sub * kM * 128 + inner, 16, 1024);
        mma_ss<kTF32>(tmem + d_col, adesc, bdesc, idesc, ks > 0 ? 1u : 0u);
      }
    }
    mma_commit(&bars[1]);
  }
  if (!mbar_wait(&bars[1], 0, st, kSiteTest, 2000000000ull)) goto done;
  tc_fence_after();
  {
    uint32_t r[16];
    for (int c = 0; c < N; c += 16) {
      tmem_ld16(tmem_addr(tmem, warp * 32, d_col + c), r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i)
        d_out[static_cast<size_t>(tid) * N + c + i] = __uint_as_float(r[i]);
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace

// A: [128, K] row-major (bf16 or fp32), B: K-major [N, K] or MN-major [K, N].
// D: [128, N] fp32.  Returns a cudaError_t; shape errors throw.
int umma_selftest_launch(const void* A, const void* B, float* D, int N, int K, bool tf32,
                         bool a_in_tmem, bool b_mn_major, DeviceStatus* st,
                         cudaStream_t stream) {
  const uint32_t esize = tf32 ? 4 : 2;
  const uint32_t elems128 = 128 / esize;
  if (N % 16 != 0 || N < 16 || N > kMaxN) throw std::runtime_error("umma_selftest: bad N");
  if (K % elems128 != 0 || K > kMaxK || K < static_cast<int>(elems128))
    throw std::runtime_error("umma_selftest: K must be a multiple of the 128-byte row");
  if (b_mn_major && N % elems128 != 0)
    throw std::runtime_error("umma_selftest: MN-major B needs N a multiple of the 128-byte row");
  const TmapDtype dt = tf32 ? TmapDtype::kF32 : TmapDtype::kBF16;
  CUtensorMap tmA{}, tmB{};
  {
    uint64_t dims[3] = {static_cast<uint64_t>(K), 128, 1};
    uint64_t strides[2] = {static_cast<uint64_t>(K) * esize, 128ull * K * esize};
    uint32_t box[3] = {elems128, 128, 1};
    tmA = make_tmap(A, dt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (!b_mn_major) {
    uint64_t dims[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N), 1};
    uint64_t strides[2] = {static_cast<uint64_t>(K) * esize, static_cast<uint64_t>(N) * K * esize};
    uint32_t box[3] = {elems128, static_cast<uint32_t>(N), 1};
    tmB = make_tmap(B, dt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    uint64_t dims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K), 1};
    uint64_t strides[2] = {static_cast<uint64_t>(N) * esize, static_cast<uint64_t>(N) * K * esize};
    uint32_t box[3] = {elems128, static_cast<uint32_t>(K), 1};
    tmB = make_tmap(B, dt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const uint32_t* a_rows = static_cast<const uint32_t*>(A);
  if (tf32) {
    cudaFuncSetAttribute(umma_selftest_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBytes);
    umma_selftest_kernel<true><<<1, 128, kSmemBytes, stream>>>(
        tmA, tmB, a_rows, D, N, K, a_in_tmem ? 1 : 0, b_mn_major ? 1 : 0, st);
  } else {
    cudaFuncSetAttribute(umma_selftest_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBytes);
    umma_selftest_kernel<false><<<1, 128, kSmemBytes, stream>>>(
        tmA, tmB, a_rows, D, N, K, a_in_tmem ? 1 : 0, b_mn_major ? 1 : 0, st);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rab
