// launchers.h - host entry points of the CUDA kernels (raw pointers + stream).
// The torch bindings in csrc/bindings.cpp wrap these; the native benchmark
// drivers call them directly.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "status.h"

namespace rab {

int umma_selftest_launch(const void* A, const void* B, float* D, int N, int K, bool tf32,
                         bool a_in_tmem, bool b_mn_major, DeviceStatus* st, cudaStream_t stream);

int simt_partial_attention_launch(const float* Q, const float* K, const float* V, int seq_q,
                                  int seq_k, int heads, int heads_kv, int D, float scale,
                                  int causal_offset, float* acc, float* m, float* l,
                                  bool normalize, cudaStream_t stream);

int merge_lse_launch(float* m_run, float* l_run, float* acc_run, const float* m_new,
                     const float* l_new, const float* acc_new, int rows, int D,
                     cudaStream_t stream);

int normalize_launch(const float* acc, const float* m, const float* l, void* out, bool bf16_out,
                     float* lse, int rows, int D, cudaStream_t stream);

int cast_f32_bf16_launch(const float* in, void* out, size_t n, cudaStream_t stream);
int cast_bf16_f32_launch(const void* in, float* out, size_t n, cudaStream_t stream);
int wait_selftest_launch(const uint64_t* flag, uint64_t target, uint64_t timeout_ns,
                         DeviceStatus* st, cudaStream_t stream);

int split_tf32_launch(const float* in, float* big, float* small, size_t n, cudaStream_t stream);

}  // namespace rab
