// bindings.cpp - torch/pybind11 surface of the native extension.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>

#include "launchers.h"
#include "bind_util.h"
#include "strfmt.h"

namespace rab {
namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const torch::Tensor& t, const char* name) {
  RAB_CHECK(t.is_cuda(), "%s must be a CUDA tensor", name);
  RAB_CHECK(t.is_contiguous(), "%s must be contiguous", name);
}

void check_launch(int err, const char* what) {
  RAB_CHECK(err == 0, "%s launch failed: %s", what, cudaGetErrorString(static_cast<cudaError_t>(err)));
}

DeviceStatus* status_ptr(const c10::optional<torch::Tensor>& status) {
  if (!status.has_value()) return nullptr;
  const auto& s = *status;
  check_cuda(s, "status");
  RAB_CHECK(s.scalar_type() == torch::kInt32 && s.numel() >= 8, "status must be int32[8]");
  return reinterpret_cast<DeviceStatus*>(s.data_ptr());
}

void umma_selftest(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool a_in_tmem,
                   bool b_mn_major, c10::optional<torch::Tensor> status) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(D, "D");
  const bool tf32 = A.scalar_type() == torch::kFloat32;
  RAB_CHECK(tf32 || A.scalar_type() == torch::kBFloat16, "A must be fp32 or bf16");
  RAB_CHECK(B.scalar_type() == A.scalar_type(), "A and B must share a dtype");
  RAB_CHECK(A.dim() == 2 && A.size(0) == 128, "A must be [128, K]");
  const int K = static_cast<int>(A.size(1));
  const int N = static_cast<int>(b_mn_major ? B.size(1) : B.size(0));
  RAB_CHECK(D.scalar_type() == torch::kFloat32 && D.size(0) == 128 && D.size(1) == N,
              "D must be fp32 [128, N]");
  const c10::cuda::CUDAGuard guard(A.device());
  check_launch(umma_selftest_launch(A.data_ptr(), B.data_ptr(), f32_ptr(D, "D"), N, K, tf32,
                                    a_in_tmem, b_mn_major, status_ptr(status), cur_stream()),
               "umma_selftest");
}

void simt_partial_attention(torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor acc,
                            c10::optional<torch::Tensor> m, c10::optional<torch::Tensor> l,
                            double scale, int64_t causal_offset, bool normalize) {
  for (auto* p : {&Q, &K, &V, &acc}) {
    check_cuda(*p, "tensor");
    RAB_CHECK(p->scalar_type() == torch::kFloat32, "simt attention is fp32 only");
  }
  RAB_CHECK(Q.dim() == 3 && K.dim() == 3 && V.dim() == 3, "Q/K/V must be [seq, heads, D]");
  const int D = static_cast<int>(Q.size(2));
  const c10::cuda::CUDAGuard guard(Q.device());
  check_launch(simt_partial_attention_launch(
                   f32_ptr(Q, "Q"), f32_ptr(K, "K"), f32_ptr(V, "V"),
                   static_cast<int>(Q.size(0)), static_cast<int>(K.size(0)),
                   static_cast<int>(Q.size(1)), static_cast<int>(K.size(1)), D,
                   static_cast<float>(scale), static_cast<int>(causal_offset),
                   f32_ptr(acc, "acc"), m ? f32_ptr(*m, "m") : nullptr,
                   l ? f32_ptr(*l, "l") : nullptr, normalize, cur_stream()),
               "simt_partial_attention");
}

void merge_lse(torch::Tensor m_run, torch::Tensor l_run, torch::Tensor acc_run, torch::Tensor m_new,
               torch::Tensor l_new, torch::Tensor acc_new) {
  for (auto* p : {&m_run, &l_run, &acc_run, &m_new, &l_new, &acc_new}) check_cuda(*p, "tensor");
  const int D = static_cast<int>(acc_run.size(-1));
  const int rows = static_cast<int>(m_run.numel());
  RAB_CHECK(acc_run.numel() == static_cast<int64_t>(rows) * D, "acc/m shape mismatch");
  const c10::cuda::CUDAGuard guard(m_run.device());
  check_launch(merge_lse_launch(f32_ptr(m_run, "m_run"), f32_ptr(l_run, "l_run"),
                                f32_ptr(acc_run, "acc_run"), f32_ptr(m_new, "m_new"),
                                f32_ptr(l_new, "l_new"), f32_ptr(acc_new, "acc_new"), rows, D,
                                cur_stream()),
               "merge_lse");
}

void normalize(torch::Tensor acc, torch::Tensor m, torch::Tensor l, torch::Tensor out,
               c10::optional<torch::Tensor> lse) {
  for (auto* p : {&acc, &m, &l, &out}) check_cuda(*p, "tensor");
  const int D = static_cast<int>(acc.size(-1));
  const int rows = static_cast<int>(m.numel());
  const bool bf16 = out.scalar_type() == torch::kBFloat16;
  RAB_CHECK(bf16 || out.scalar_type() == torch::kFloat32, "out must be fp32 or bf16");
  const c10::cuda::CUDAGuard guard(acc.device());
  check_launch(normalize_launch(f32_ptr(acc, "acc"), f32_ptr(m, "m"), f32_ptr(l, "l"),
                                out.data_ptr(), bf16, lse ? f32_ptr(*lse, "lse") : nullptr, rows,
                                D, cur_stream()),
               "normalize");
}

void cast(torch::Tensor in, torch::Tensor out) {
  check_cuda(in, "in");
  check_cuda(out, "out");
  RAB_CHECK(in.numel() == out.numel(), "cast: size mismatch");
  const c10::cuda::CUDAGuard guard(in.device());
  if (in.scalar_type() == torch::kFloat32 && out.scalar_type() == torch::kBFloat16) {
    check_launch(cast_f32_bf16_launch(f32_ptr(in, "in"), out.data_ptr(), in.numel(),
                                      cur_stream()),
                 "cast_f32_bf16");
  } else if (in.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kFloat32) {
    check_launch(cast_bf16_f32_launch(in.data_ptr(), f32_ptr(out, "out"), in.numel(),
                                      cur_stream()),
                 "cast_bf16_f32");
  } else {
    RAB_CHECK(false, "cast supports fp32<->bf16 only");
  }
}

void split_tf32(torch::Tensor in, torch::Tensor big, torch::Tensor small) {
  for (auto* p : {&in, &big, &small}) {
    check_cuda(*p, "tensor");
    RAB_CHECK(p->scalar_type() == torch::kFloat32, "split_tf32 is fp32 only");
  }
  RAB_CHECK(in.numel() == big.numel() && in.numel() == small.numel(), "split_tf32: size mismatch");
  const c10::cuda::CUDAGuard guard(in.device());
  check_launch(split_tf32_launch(f32_ptr(in, "in"), f32_ptr(big, "big"),
                                 f32_ptr(small, "small"), in.numel(), cur_stream()),
               "split_tf32");
}

void wait_selftest(torch::Tensor flag, int64_t target, double timeout_s, torch::Tensor status) {
  check_cuda(flag, "flag");
  RAB_CHECK(flag.scalar_type() == torch::kInt64 && flag.numel() >= 1, "flag must be int64");
  const c10::cuda::CUDAGuard guard(flag.device());
  check_launch(wait_selftest_launch(reinterpret_cast<const uint64_t*>(flag.data_ptr()),
                                    static_cast<uint64_t>(target),
                                    static_cast<uint64_t>(timeout_s * 1e9), status_ptr(status),
                                    cur_stream()),
               "wait_selftest");
}

}  // namespace
}  // namespace rab

void register_runtime(pybind11::module_& m);  // runtime_bindings.cpp
void register_flash(pybind11::module_& m);    // flash_bindings.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200-native ring attention: sm_100a kernels and the native ring runtime";
  m.def("umma_selftest", &rab::umma_selftest, "one-tile tcgen05 GEMM check", py::arg("A"),
        py::arg("B"), py::arg("D"), py::arg("a_in_tmem"), py::arg("b_mn_major"),
        py::arg("status") = c10::nullopt);
  m.def("simt_partial_attention", &rab::simt_partial_attention,
        "fp32 CUDA-core partial attention in the reference's arithmetic order", py::arg("Q"),
        py::arg("K"), py::arg("V"), py::arg("acc"), py::arg("m") = c10::nullopt,
        py::arg("l") = c10::nullopt, py::arg("scale") = 1.0, py::arg("causal_offset") = -1,
        py::arg("normalize") = false);
  m.def("merge_lse", &rab::merge_lse, "online-softmax merge (in place on the running state)");
  m.def("normalize", &rab::normalize, "out = acc / l, lse = m + log l", py::arg("acc"),
        py::arg("m"), py::arg("l"), py::arg("out"), py::arg("lse") = c10::nullopt);
  m.def("cast", &rab::cast, "fp32 <-> bf16 cast");
  m.def("split_tf32", &rab::split_tf32, "fp32 -> tf32 big/small planes");
  m.def("wait_selftest", &rab::wait_selftest,
        "bounded device wait on a flag word; records a timeout in the status word");
  register_flash(m);
  register_runtime(m);
}
