// simt_attention.cu - fp32 CUDA-core partial attention that reproduces the
// reference benchmark's arithmetic exactly where it matters.
//
// Reference semantics (src/attention/ring_attention_staged_gpu_bench.cu:78-143,
// the C16 kernel, and its CPU statement at :41-77): for query row i against one
// K/V block, s_j = sum_d Q[i,d] * K[j,d] accumulated sequentially over d,
// m = max_j s_j, w_j = expf(s_j - m), l = sum_j w_j, acc[i,:] = sum_j w_j V[j,:]
// (unnormalised).  The reference-compatible inputs produce scores near 1.6e7
// whose neighbours differ by ~1.3, so the dot product must run in the same
// order with the same fused multiply-adds or the softmax picks different keys.
// This kernel keeps that order (one thread per query row, d ascending, fmaf) and
// computes the exact row max in a first pass, like the reference.  Unlike the
// reference it needs no atomics and is deterministic: keys are visited in
// ascending order in both passes.
//
// Layout: Q [seq_q, heads, D], K/V [seq_k, heads_kv, D] (row-major, D
// contiguous), acc [seq_q, heads, D], m/l [seq_q, heads].  Query head h reads
// key/value head h / (heads / heads_kv).
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <stdexcept>

namespace rab {

namespace {

constexpr int kRows = 128;     // query rows per CTA (one per thread)
constexpr int kKeyTile = 32;   // keys staged in shared memory per iteration

template <int D>
__global__ void __launch_bounds__(kRows)
    simt_partial_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                        const float* __restrict__ V, int seq_q, int seq_k, int heads,
                        int heads_kv, float scale, int causal_offset, float* __restrict__ acc_out,
                        float* __restrict__ m_out, float* __restrict__ l_out, int normalize) {
  __shared__ float sK[kKeyTile][D];
  __shared__ float sV[kKeyTile][D];
  const int h = blockIdx.y;
  const int hk = h / (heads / heads_kv);
  const int i = blockIdx.x * kRows + threadIdx.x;
  const bool active = i < seq_q;
  const int row = active ? i : 0;

  float q[D];
#pragma unroll
  for (int d = 0; d < D; ++d) q[d] = Q[(static_cast<size_t>(row) * heads + h) * D + d];

  // causal_offset < 0 disables masking; otherwise key j is visible to query i
  // when j <= i + causal_offset (positions in a common frame).
  const int kmax = (causal_offset >= 0) ? min(seq_k, row + causal_offset + 1) : seq_k;

  // ---- pass 1: exact row max ----
  float m = -FLT_MAX;
  for (int j0 = 0; j0 < seq_k; j0 += kKeyTile) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kKeyTile * D; idx += kRows) {
      const int jj = idx / D, d = idx % D;
      const int j = j0 + jj;
      sK[jj][d] = j < seq_k ? K[(static_cast<size_t>(j) * heads_kv + hk) * D + d] : 0.f;
    }
    __syncthreads();
    const int jend = min(kKeyTile, kmax - j0);
    for (int jj = 0; jj < jend; ++jj) {
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < D; ++d) s = fmaf(q[d], sK[jj][d], s);
      if (scale != 1.0f) s *= scale;
      if (m < s) m = s;
    }
  }

  // ---- pass 2: weights, row sum, unnormalised accumulator ----
  float a[D];
#pragma unroll
  for (int d = 0; d < D; ++d) a[d] = 0.f;
  float l = 0.f;
  for (int j0 = 0; j0 < seq_k; j0 += kKeyTile) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kKeyTile * D; idx += kRows) {
      const int jj = idx / D, d = idx % D;
      const int j = j0 + jj;
      const size_t off = (static_cast<size_t>(j) * heads_kv + hk) * D + d;
      sK[jj][d] = j < seq_k ? K[off] : 0.f;
      sV[jj][d] = j < seq_k ? V[off] : 0.f;
    }
    __syncthreads();
    const int jend = min(kKeyTile, kmax - j0);
    for (int jj = 0; jj < jend; ++jj) {
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < D; ++d) s = fmaf(q[d], sK[jj][d], s);
      if (scale != 1.0f) s *= scale;
      const float w = expf(s - m);
      l += w;
#pragma unroll
      for (int d = 0; d < D; ++d) a[d] = fmaf(w, sV[jj][d], a[d]);
    }
  }
  if (!active) return;
  const size_t r = static_cast<size_t>(i) * heads + h;
  if (normalize) {
    const float inv = 1.0f / l;
#pragma unroll
    for (int d = 0; d < D; ++d) acc_out[r * D + d] = a[d] * inv;
  } else {
#pragma unroll
    for (int d = 0; d < D; ++d) acc_out[r * D + d] = a[d];
  }
  if (m_out) m_out[r] = m;
  if (l_out) l_out[r] = l;
}

}  // namespace

int simt_partial_attention_launch(const float* Q, const float* K, const float* V, int seq_q,
                                  int seq_k, int heads, int heads_kv, int D, float scale,
                                  int causal_offset, float* acc, float* m, float* l,
                                  bool normalize, cudaStream_t stream) {
  if (heads_kv <= 0 || heads % heads_kv != 0)
    throw std::runtime_error("simt_partial_attention: heads must be a multiple of heads_kv");
  dim3 grid((seq_q + kRows - 1) / kRows, heads);
  if (D == 64) {
    simt_partial_kernel<64><<<grid, kRows, 0, stream>>>(Q, K, V, seq_q, seq_k, heads, heads_kv,
                                                        scale, causal_offset, acc, m, l,
                                                        normalize ? 1 : 0);
  } else if (D == 128) {
    simt_partial_kernel<128><<<grid, kRows, 0, stream>>>(Q, K, V, seq_q, seq_k, heads, heads_kv,
                                                         scale, causal_offset, acc, m, l,
                                                         normalize ? 1 : 0);
  } else {
    throw std::runtime_error("simt_partial_attention: head_dim must be 64 or 128");
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rab
