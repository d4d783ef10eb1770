// runtime_bindings.cpp - pybind11 surface of the native ring runtime:
// HostComm (shared-memory control plane), RingContext (device arena, IPC,
// NCCL), the comm / attention benchmark drivers and the FusedRing engine.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <memory>
#include <string>
#include <vector>

#include "drivers.h"
#include "bind_util.h"
#include "strfmt.h"
#include "host_comm.h"
#include "ring_context.h"

namespace py = pybind11;
using namespace rab;

namespace {

Prec prec_from(const std::string& s) {
  if (s == "bf16" || s == "bfloat16") return Prec::kBF16;
  if (s == "fp32" || s == "float32") return Prec::kF32x3;
  throw std::runtime_error("precision must be fp32 or bf16");
}

void check_cpu_contig(const torch::Tensor& t, const char* name) {
  RAB_CHECK(!t.is_cuda() && t.is_contiguous(), "%s must be a contiguous CPU tensor", name);
}

// Inputs and outputs of a FusedRing call must match the engine's shapes and
// precision exactly (the kernels index them with the engine's sizes) and sit
// on one GPU.  Null pointers are skipped.
void check_fused_io(const FusedRing& f, const torch::Tensor* q, const torch::Tensor* k,
                    const torch::Tensor* v, const torch::Tensor* out,
                    const c10::optional<torch::Tensor>& lse) {
  const FlashArgs& a = f.args();
  const auto in_type = a.prec == Prec::kBF16 ? torch::kBFloat16 : torch::kFloat32;
  const int64_t nq = static_cast<int64_t>(a.Sq) * a.Hq * a.D;
  const int64_t nkv = static_cast<int64_t>(a.Skv) * a.Hkv * a.D;
  const torch::Tensor* first = q ? q : k;
  auto check = [&](const torch::Tensor* t, const char* name, int64_t numel, bool out_tensor) {
    if (t == nullptr) return;
    RAB_CHECK(t->is_cuda() && t->is_contiguous(), "%s: a contiguous CUDA tensor is required", name);
    RAB_CHECK(t->device() == first->device(), "%s: all tensors must be on one GPU", name);
    RAB_CHECK(t->numel() == numel, "%s: expected %lld elements for the engine's shape, got %lld",
              name, static_cast<long long>(numel), static_cast<long long>(t->numel()));
    if (out_tensor) {
      RAB_CHECK(t->scalar_type() == torch::kFloat32 || t->scalar_type() == torch::kBFloat16,
                "%s: must be float32 or bfloat16", name);
    } else {
      RAB_CHECK(t->scalar_type() == in_type, "%s: dtype does not match the engine's precision", name);
    }
  };
  check(q, "q", nq, false);
  check(k, "k", nkv, false);
  check(v, "v", nkv, false);
  check(out, "out", nq, true);
  if (lse) {
    check(&*lse, "lse", static_cast<int64_t>(a.Sq) * a.Hq, true);
    RAB_CHECK(lse->scalar_type() == torch::kFloat32, "lse: must be float32");
  }
}

}  // namespace

namespace rab {
void install_crash_handler();
}

void register_runtime(py::module_& m) {
  rab::install_crash_handler();
  py::register_exception<RankFailure>(m, "RankFailure", PyExc_RuntimeError);

  py::class_<HostComm>(m, "HostComm")
      .def(py::init<const std::string&, int, int, bool, size_t, double>(), py::arg("name"),
           py::arg("rank"), py::arg("world"), py::arg("create"), py::arg("frag_bytes") = 1 << 20,
           py::arg("timeout_s") = 60.0)
      .def_property_readonly("rank", &HostComm::rank)
      .def_property_readonly("world", &HostComm::world)
      .def("set_timeout", &HostComm::set_timeout)
      .def("unlink", &HostComm::unlink)
      .def("barrier", &HostComm::barrier, py::call_guard<py::gil_scoped_release>())
      .def("reduce_max", &HostComm::reduce_max, py::call_guard<py::gil_scoped_release>())
      .def("ring_sendrecv",
           [](HostComm& h, torch::Tensor send, torch::Tensor recv) {
             check_cpu_contig(send, "send");
             check_cpu_contig(recv, "recv");
             const size_t n = send.numel() * send.element_size();
             RAB_CHECK(static_cast<size_t>(recv.numel() * recv.element_size()) == n,
                         "send/recv size mismatch");
             py::gil_scoped_release nogil;
             h.ring_sendrecv(send.data_ptr(), recv.data_ptr(), n);
           })
      .def("abort", &HostComm::abort)
      .def("aborted", &HostComm::aborted)
      .def("abort_message", &HostComm::abort_message)
      .def("user_store", [](HostComm& h, int r, int i, uint64_t v) { h.user_word(r, i).store(v); })
      .def("user_load", [](HostComm& h, int r, int i) { return h.user_word(r, i).load(); })
      .def(
          "wait_user",
          [](HostComm& h, int r, int i, uint64_t v) {
            py::gil_scoped_release nogil;
            h.wait_at_least(h.user_word(r, i), v, "user word", r);
          });

  py::class_<RingContext>(m, "RingContext")
      .def(py::init<int, int, int, const std::string&, bool, size_t, size_t, double>(),
           py::arg("rank"), py::arg("world"), py::arg("device"), py::arg("shm_name"),
           py::arg("create_shm"), py::arg("frag_bytes"), py::arg("arena_bytes"),
           py::arg("timeout_s"))
      .def_property_readonly("rank", &RingContext::rank)
      .def_property_readonly("world", &RingContext::world)
      .def_property_readonly("device", &RingContext::device)
      .def_property_readonly("arena_bytes", &RingContext::arena_bytes)
      .def("ipc_handle", [](RingContext& c) { return py::bytes(c.ipc_handle()); })
      .def("open_peers",
           [](RingContext& c, const std::vector<py::bytes>& hs) {
             std::vector<std::string> v;
             for (auto& h : hs) v.push_back(std::string(h));
             c.open_peers(v);
           })
      .def_static("nccl_unique_id", []() { return py::bytes(RingContext::nccl_unique_id()); })
      .def("init_nccl", [](RingContext& c, py::bytes uid) { c.init_nccl(std::string(uid)); },
           py::call_guard<py::gil_scoped_release>())
      .def("set_devices_unique", &RingContext::set_devices_unique)
      .def("unlink_shm", [](RingContext& c) { c.host().unlink(); })
      .def("barrier", [](RingContext& c) { c.host().barrier(); },
           py::call_guard<py::gil_scoped_release>())
      .def("reduce_max", [](RingContext& c, const std::vector<double>& v) {
        py::gil_scoped_release nogil;
        return c.host().reduce_max(v);
      })
      .def("abort", [](RingContext& c, const std::string& msg) { c.host().abort(msg); })
      .def("reset_flags", &RingContext::reset_flags, py::call_guard<py::gil_scoped_release>())
      .def("read_status", [](RingContext& c, bool clear) {
        const DeviceStatus s = c.read_status(clear);
        return std::vector<uint32_t>{s.code, s.where, s.block, s.detail, s.n_errors};
      }, py::arg("clear") = true);

  m.def(
      "run_comm_bench",
      [](RingContext& ctx, const std::string& backend, size_t bytes, int warmup, int iters,
         int slices, bool precheck, int p2p_mode) {
        CommOptions o;
        o.backend = backend;
        o.bytes = bytes;
        o.warmup = warmup;
        o.iters = iters;
        o.slices = slices;
        o.precheck = precheck;
        o.p2p_mode = p2p_mode;
        CommResult r;
        {
          py::gil_scoped_release nogil;
          r = run_comm_bench(ctx, o);
        }
        return r.avg_ms;
      },
      py::arg("ctx"), py::arg("backend"), py::arg("bytes"), py::arg("warmup") = 10,
      py::arg("iters") = 100, py::arg("slices") = 0, py::arg("precheck") = true,
      py::arg("p2p_mode") = 0);
  m.def("comm_arena_bytes", &comm_arena_bytes);

  py::class_<AttnBench>(m, "AttnBench")
      .def(py::init([](RingContext& ctx, const std::string& backend, const std::string& prec,
                       int seq, int heads, int heads_kv, int dim, double scale, bool kv_shared,
                       bool causal, bool zigzag, const std::string& kernel, bool ring_chain,
                       int warmup, int iters, double timeout_s) {
             AttnOptions o;
             o.backend = backend;
             o.prec = prec_from(prec);
             o.seq = seq;
             o.heads = heads;
             o.heads_kv = heads_kv;
             o.dim = dim;
             o.scale = static_cast<float>(scale);
             o.kv_shared = kv_shared;
             o.causal = causal;
             o.zigzag = zigzag;
             o.kernel = kernel;
             o.ring_chain = ring_chain;
             o.warmup = warmup;
             o.iters = iters;
             o.timeout_s = timeout_s;
             return std::make_unique<AttnBench>(ctx, o);
           }),
           py::arg("ctx"), py::arg("backend"), py::arg("prec"), py::arg("seq"),
           py::arg("heads") = 1, py::arg("heads_kv") = 1, py::arg("dim") = 64,
           py::arg("scale") = 1.0, py::arg("kv_shared") = false, py::arg("causal") = false,
           py::arg("zigzag") = false, py::arg("kernel") = "tcgen05", py::arg("ring_chain") = false,
           py::arg("warmup") = 10, py::arg("iters") = 50, py::arg("timeout_s") = 10.0,
           py::keep_alive<1, 2>())
      .def("set_inputs",
           [](AttnBench& b, torch::Tensor q, torch::Tensor k, torch::Tensor v) {
             check_cpu_contig(q, "q");
             check_cpu_contig(k, "k");
             check_cpu_contig(v, "v");
             b.set_inputs(q.data_ptr(), k.data_ptr(), v.data_ptr());
           })
      .def("run",
           [](AttnBench& b) {
             AttnResult r;
             {
               py::gil_scoped_release nogil;
               r = b.run();
             }
             py::dict d;
             for (auto& kv : r.avg_ms) d[py::str(kv.first)] = kv.second;
             d["step_ms"] = r.step_ms;
             return d;
           })
      .def("output",
           [](AttnBench& b, torch::Tensor dst) {
             check_cpu_contig(dst, "dst");
             RAB_CHECK(static_cast<size_t>(dst.numel() * dst.element_size()) == b.output_bytes(),
                         "output size mismatch");
             b.copy_output(dst.data_ptr());
           })
      .def_static("arena_bytes", [](const std::string& prec, int seq, int heads_kv, int dim,
                                    bool kv_shared, int world) {
        AttnOptions o;
        o.prec = prec_from(prec);
        o.seq = seq;
        o.heads_kv = heads_kv;
        o.dim = dim;
        o.kv_shared = kv_shared;
        return AttnBench::arena_bytes(o, world);
      });

  py::class_<FusedRing>(m, "FusedRing")
      .def(py::init([](RingContext& ctx, const std::string& prec, int seq, int heads, int heads_kv,
                       int dim, bool causal, bool zigzag, bool ring_chain, double timeout_s,
                       bool device_epochs) {
             return std::make_unique<FusedRing>(ctx, prec_from(prec), seq, heads, heads_kv, dim,
                                                causal, zigzag, ring_chain, timeout_s,
                                                device_epochs);
           }),
           py::arg("ctx"), py::arg("prec"), py::arg("seq"), py::arg("heads"),
           py::arg("heads_kv"), py::arg("dim"), py::arg("causal") = false,
           py::arg("zigzag") = false, py::arg("ring_chain") = false,
           py::arg("timeout_s") = 10.0, py::arg("device_epochs") = false, py::keep_alive<1, 2>())
      .def_static("arena_bytes", [](const std::string& prec, int seq, int heads_kv, int dim,
                                    int world) {
        return FusedRing::arena_bytes(prec_from(prec), seq, heads_kv, dim, world);
      })
      .def("forward",
           [](FusedRing& f, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
              c10::optional<torch::Tensor> lse, double scale) {
             check_fused_io(f, &q, &k, &v, &out, lse);
             const c10::cuda::CUDAGuard guard(q.device());
             f.forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                       out.scalar_type() == torch::kBFloat16,
                       lse ? f32_ptr(*lse, "lse") : nullptr, static_cast<float>(scale),
                       at::cuda::getCurrentCUDAStream().stream());
           },
           py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"), py::arg("lse") = c10::nullopt,
           py::arg("scale"))
      .def("prepare",
           [](FusedRing& f, torch::Tensor k, torch::Tensor v) {
             check_fused_io(f, nullptr, &k, &v, nullptr, c10::nullopt);
             const c10::cuda::CUDAGuard guard(k.device());
             f.prepare(k.data_ptr(), v.data_ptr(), at::cuda::getCurrentCUDAStream().stream());
           })
      .def("attend",
           [](FusedRing& f, torch::Tensor q, torch::Tensor out, c10::optional<torch::Tensor> lse,
              double scale) {
             check_fused_io(f, &q, nullptr, nullptr, &out, lse);
             const c10::cuda::CUDAGuard guard(q.device());
             f.attend(q.data_ptr(), out.data_ptr(), out.scalar_type() == torch::kBFloat16,
                      lse ? f32_ptr(*lse, "lse") : nullptr, static_cast<float>(scale),
                      at::cuda::getCurrentCUDAStream().stream());
           },
           py::arg("q"), py::arg("out"), py::arg("lse") = c10::nullopt, py::arg("scale"))
      .def("check", &FusedRing::check)
      .def("set_trace", &FusedRing::set_trace)
      .def("read_trace",
           [](const FusedRing& f) {
             torch::Tensor t = torch::empty({static_cast<int64_t>(f.grid()), kMaxSlots, 2},
                                            torch::dtype(torch::kInt64));
             f.read_trace(reinterpret_cast<uint64_t*>(t.data_ptr()));
             return t;
           })
      .def_property_readonly("grid", &FusedRing::grid)
      .def_property_readonly("nsplit", &FusedRing::nsplit)
      .def_property_readonly("merge_launches", &FusedRing::merge_launches)
      .def_property_readonly("launches", &FusedRing::launches)
      .def_property_readonly("device_epochs", &FusedRing::device_epochs)
      .def("slot0_ptrs", [](FusedRing& f) {
        return std::make_pair(reinterpret_cast<uintptr_t>(f.slot0_k()),
                              reinterpret_cast<uintptr_t>(f.slot0_v()));
      });
}
