// elementwise.cu - the memory-bound hot ops around the attention kernels:
//   * merge_lse:   online-softmax merge of a running (acc, m, l) with a new
//                  partial block (reference C17: merge_online_softmax,
//                  src/attention/ring_attention_staged_gpu_bench.cu:171-192)
//   * normalize:   out = acc / l and lse = m + log(l) (reference C19 does this
//                  on the host, src/attention/ring_attention_staged_gpu_bench.cu:428-437)
//   * cast:        fp32 <-> bf16
//   * split_tf32:  fp32 -> (big, small) tf32 planes for the 3xTF32 tensor-core
//                  path (Ootomo & Yokota, 2022)
// All of them move 16-byte vectors; rows are [rows, D] with D % 4 == 0.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <stdexcept>

#include "flash.h"

namespace rab {

namespace {

// One group of D/4 threads per row, each thread owns one float4 of the row.
template <int D>
__global__ void merge_lse_kernel(float* __restrict__ m_run, float* __restrict__ l_run,
                                 float* __restrict__ acc_run, const float* __restrict__ m_new,
                                 const float* __restrict__ l_new,
                                 const float* __restrict__ acc_new, int rows) {
  constexpr int kTpr = D / 4;  // threads per row
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = t / kTpr;
  const int c = t % kTpr;
  if (row >= rows) return;
  const float mo = m_run[row];
  const float mn = m_new[row];
  const float mx = fmaxf(mo, mn);
  const float so = expf(mo - mx);
  const float sn = expf(mn - mx);
  float4* ar = reinterpret_cast<float4*>(acc_run + static_cast<size_t>(row) * D) + c;
  const float4 an = reinterpret_cast<const float4*>(acc_new + static_cast<size_t>(row) * D)[c];
  float4 a = *ar;
  a.x = so * a.x + sn * an.x;
  a.y = so * a.y + sn * an.y;
  a.z = so * a.z + sn * an.z;
  a.w = so * a.w + sn * an.w;
  *ar = a;
  if (c == 0) {
    l_run[row] = so * l_run[row] + sn * l_new[row];
    m_run[row] = mx;
  }
}

template <int D, bool kBF16Out>
__global__ void normalize_kernel(const float* __restrict__ acc, const float* __restrict__ m,
                                 const float* __restrict__ l, void* __restrict__ out,
                                 float* __restrict__ lse, int rows) {
  constexpr int kTpr = D / 4;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = t / kTpr;
  const int c = t % kTpr;
  if (row >= rows) return;
  const float lv = l[row];
  const float inv = 1.0f / lv;
  float4 a = reinterpret_cast<const float4*>(acc + static_cast<size_t>(row) * D)[c];
  a.x *= inv;
  a.y *= inv;
  a.z *= inv;
  a.w *= inv;
  if constexpr (kBF16Out) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(a.z, a.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + static_cast<size_t>(row) * D)[c] =
        packed;
  } else {
    reinterpret_cast<float4*>(static_cast<float*>(out) + static_cast<size_t>(row) * D)[c] = a;
  }
  if (lse != nullptr && c == 0) lse[row] = m[row] + logf(lv);
}

__global__ void cast_f32_bf16_kernel(const float4* __restrict__ in, uint2* __restrict__ out,
                                     size_t n4) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 a = in[i];
    __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(a.z, a.w);
    uint2 p;
    p.x = *reinterpret_cast<uint32_t*>(&lo);
    p.y = *reinterpret_cast<uint32_t*>(&hi);
    out[i] = p;
  }
}

__global__ void cast_bf16_f32_kernel(const uint2* __restrict__ in, float4* __restrict__ out,
                                     size_t n4) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint2 p = in[i];
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&p.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&p.y);
    const float2 a = __bfloat1622float2(lo);
    const float2 b = __bfloat1622float2(hi);
    out[i] = make_float4(a.x, a.y, b.x, b.y);
  }
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// big = rna_tf32(x), small = rna_tf32(x - big); both land in separate planes.
__global__ void split_tf32_kernel(const float4* __restrict__ in, float4* __restrict__ big,
                                  float4* __restrict__ small, size_t n4) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 a = in[i];
    float4 b, s;
    b.x = __uint_as_float(to_tf32(a.x));
    b.y = __uint_as_float(to_tf32(a.y));
    b.z = __uint_as_float(to_tf32(a.z));
    b.w = __uint_as_float(to_tf32(a.w));
    s.x = __uint_as_float(to_tf32(a.x - b.x));
    s.y = __uint_as_float(to_tf32(a.y - b.y));
    s.z = __uint_as_float(to_tf32(a.z - b.z));
    s.w = __uint_as_float(to_tf32(a.w - b.w));
    big[i] = b;
    small[i] = s;
  }
}

int grid_for(size_t n, int block) {
  size_t g = (n + block - 1) / block;
  const size_t cap = 16 * static_cast<size_t>(flash_sm_count());
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace

int merge_lse_launch(float* m_run, float* l_run, float* acc_run, const float* m_new,
                     const float* l_new, const float* acc_new, int rows, int D,
                     cudaStream_t stream) {
  const int threads = 256;
  const size_t total = static_cast<size_t>(rows) * (D / 4);
  const int blocks = static_cast<int>((total + threads - 1) / threads);
  if (blocks == 0) return 0;
  if (D == 64)
    merge_lse_kernel<64><<<blocks, threads, 0, stream>>>(m_run, l_run, acc_run, m_new, l_new,
                                                         acc_new, rows);
  else if (D == 128)
    merge_lse_kernel<128><<<blocks, threads, 0, stream>>>(m_run, l_run, acc_run, m_new, l_new,
                                                          acc_new, rows);
  else
    throw std::runtime_error("merge_lse: head_dim must be 64 or 128");
  return static_cast<int>(cudaGetLastError());
}

int normalize_launch(const float* acc, const float* m, const float* l, void* out, bool bf16_out,
                     float* lse, int rows, int D, cudaStream_t stream) {
  const int threads = 256;
  const size_t total = static_cast<size_t>(rows) * (D / 4);
  const int blocks = static_cast<int>((total + threads - 1) / threads);
  if (blocks == 0) return 0;
#define RAB_NORM(DD, BF)                                                                      \
  normalize_kernel<DD, BF><<<blocks, threads, 0, stream>>>(acc, m, l, out, lse, rows)
  if (D == 64) {
    if (bf16_out) RAB_NORM(64, true); else RAB_NORM(64, false);
  } else if (D == 128) {
    if (bf16_out) RAB_NORM(128, true); else RAB_NORM(128, false);
  } else {
    throw std::runtime_error("normalize: head_dim must be 64 or 128");
  }
#undef RAB_NORM
  return static_cast<int>(cudaGetLastError());
}

int cast_f32_bf16_launch(const float* in, void* out, size_t n, cudaStream_t stream) {
  if (n % 4 != 0) throw std::runtime_error("cast_f32_bf16: element count must be a multiple of 4");
  const size_t n4 = n / 4;
  if (n4 == 0) return 0;
  cast_f32_bf16_kernel<<<grid_for(n4, 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(in), static_cast<uint2*>(out), n4);
  return static_cast<int>(cudaGetLastError());
}

int cast_bf16_f32_launch(const void* in, float* out, size_t n, cudaStream_t stream) {
  if (n % 4 != 0) throw std::runtime_error("cast_bf16_f32: element count must be a multiple of 4");
  const size_t n4 = n / 4;
  if (n4 == 0) return 0;
  cast_bf16_f32_kernel<<<grid_for(n4, 256), 256, 0, stream>>>(
      static_cast<const uint2*>(in), reinterpret_cast<float4*>(out), n4);
  return static_cast<int>(cudaGetLastError());
}

int split_tf32_launch(const float* in, float* big, float* small, size_t n, cudaStream_t stream) {
  if (n % 4 != 0) throw std::runtime_error("split_tf32: element count must be a multiple of 4");
  const size_t n4 = n / 4;
  if (n4 == 0) return 0;
  split_tf32_kernel<<<grid_for(n4, 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(in), reinterpret_cast<float4*>(big),
      reinterpret_cast<float4*>(small), n4);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rab
