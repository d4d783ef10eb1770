// flash_bindings.cpp - torch surface of the tcgen05 flash forward (single GPU:
// all K/V blocks already sit in local ring slots).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <pybind11/stl.h>

#include "flash.h"
#include "bind_util.h"
#include "strfmt.h"

namespace rab {
namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// A tensor the kernel writes: contiguous, on `dev`, at least `min_numel`
// elements.  A short buffer would be written past its end by the kernel (a
// device fault), so it is refused here as a RuntimeError instead.
void check_output(const torch::Tensor& t, const char* name, const c10::Device& dev,
                  int64_t min_numel) {
  RAB_CHECK(t.is_cuda() && t.device() == dev, "%s must be on the same GPU as q", name);
  RAB_CHECK(t.is_contiguous(), "%s must be contiguous", name);
  RAB_CHECK(t.numel() >= min_numel, "%s has %lld elements, needs at least %lld", name,
            static_cast<long long>(t.numel()), static_cast<long long>(min_numel));
}

Prec to_prec(int64_t p) {
  RAB_CHECK(p == 0 || p == 1, "prec must be 0 (bf16) or 1 (fp32 via 3xTF32)");
  return static_cast<Prec>(p);
}

void ring_format(int64_t prec, torch::Tensor k, torch::Tensor v, torch::Tensor slot) {
  const Prec pr = to_prec(prec);
  RAB_CHECK(k.is_cuda() && v.is_cuda() && slot.is_cuda(), "CUDA tensors required");
  RAB_CHECK(k.is_contiguous() && v.is_contiguous() && slot.is_contiguous(), "contiguous tensors");
  RAB_CHECK(k.dim() == 3 && v.sizes() == k.sizes(), "k/v must be [Skv, Hkv, D]");
  RAB_CHECK(k.scalar_type() == (pr == Prec::kBF16 ? torch::kBFloat16 : torch::kFloat32),
              "k/v dtype does not match prec");
  const int Skv = k.size(0), Hkv = k.size(1), D = k.size(2);
  const size_t need = ring_block_bytes(pr, Skv, Hkv, D);
  RAB_CHECK(static_cast<size_t>(slot.numel() * slot.element_size()) >= need, "slot too small");
  const c10::cuda::CUDAGuard guard(k.device());
  uint8_t* base = static_cast<uint8_t*>(slot.data_ptr());
  const int err = ring_format_launch(pr, k.data_ptr(), v.data_ptr(), base,
                                     base + ring_v_offset(pr, Skv, Hkv, D), Skv, Hkv, D,
                                     cur_stream());
  RAB_CHECK(err == 0, "ring_format failed: %s", cudaGetErrorString(static_cast<cudaError_t>(err)));
}

std::vector<int64_t> flash_fwd(int64_t prec, torch::Tensor q, torch::Tensor slots, int64_t nblk,
                               int64_t Skv, int64_t Hkv, c10::optional<torch::Tensor> out,
                               c10::optional<torch::Tensor> lse, double scale, bool causal,
                               bool zigzag, int64_t world, int64_t rank, int64_t nsplit,
                               c10::optional<torch::Tensor> acc, c10::optional<torch::Tensor> m,
                               c10::optional<torch::Tensor> l, torch::Tensor status,
                               double timeout_s, int64_t grid) {
  const Prec pr = to_prec(prec);
  RAB_CHECK(q.is_cuda() && q.is_contiguous() && q.dim() == 3, "q must be contiguous [Sq, Hq, D]");
  RAB_CHECK(q.scalar_type() == (pr == Prec::kBF16 ? torch::kBFloat16 : torch::kFloat32),
              "q dtype does not match prec");
  RAB_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32 && status.numel() >= 8,
              "status must be int32[8] on the GPU");
  RAB_CHECK(status.device() == q.device(), "status must be on the same GPU as q");
  RAB_CHECK(slots.is_cuda() && slots.device() == q.device() && slots.is_contiguous(),
            "slots must be contiguous on the same GPU as q");
  const int64_t rows = q.size(0) * q.size(1);  // Sq * Hq
  const c10::cuda::CUDAGuard guard(q.device());
  FlashArgs a;
  a.prec = pr;
  a.q = q.data_ptr();
  a.Sq = q.size(0);
  a.Hq = q.size(1);
  a.D = q.size(2);
  a.Hkv = static_cast<int>(Hkv);
  a.Skv = static_cast<int>(Skv);
  a.nblk = static_cast<int>(nblk);
  a.scale = static_cast<float>(scale);
  const size_t bb = ring_block_bytes(pr, a.Skv, a.Hkv, a.D);
  RAB_CHECK(static_cast<size_t>(slots.numel() * slots.element_size()) >= bb * nblk,
              "slots tensor too small for nblk blocks");
  uint8_t* base = static_cast<uint8_t*>(slots.data_ptr());
  a.k_base = base;
  a.v_base = base + ring_v_offset(pr, a.Skv, a.Hkv, a.D);
  a.slot_stride = bb;
  a.causal = causal;
  a.zigzag = zigzag;
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.nsplit = static_cast<int>(nsplit);
  a.grid = static_cast<int>(grid);
  a.status = reinterpret_cast<DeviceStatus*>(status.data_ptr());
  a.timeout_s = timeout_s;
  if (acc.has_value()) {
    a.partial = true;
    check_output(*acc, "acc", q.device(), rows * q.size(2));
    a.acc = f32_ptr(*acc, "acc");
    if (m) check_output(*m, "m", q.device(), rows);
    if (l) check_output(*l, "l", q.device(), rows);
    a.m = m ? f32_ptr(*m, "m") : nullptr;
    a.l = l ? f32_ptr(*l, "l") : nullptr;
  } else {
    RAB_CHECK(out.has_value(), "out (or partial acc/m/l) is required");
    check_output(*out, "out", q.device(), q.numel());
    RAB_CHECK(out->sizes() == q.sizes(), "out must have q's shape [Sq, Hq, D]");
    RAB_CHECK(out->scalar_type() == torch::kBFloat16 || out->scalar_type() == torch::kFloat32,
              "out must be bfloat16 or float32");
    a.out = out->data_ptr();
    a.out_bf16 = out->scalar_type() == torch::kBFloat16;
    if (lse) check_output(*lse, "lse", q.device(), rows);
    a.lse = lse ? f32_ptr(*lse, "lse") : nullptr;
  }
  const FlashPlan pl = flash_plan(a);
  torch::Tensor ws;
  if (pl.workspace_bytes > 0) {
    ws = torch::empty({static_cast<int64_t>(pl.workspace_bytes)},
                      torch::dtype(torch::kUInt8).device(q.device()));
    a.workspace = ws.data_ptr();
    a.workspace_bytes = pl.workspace_bytes;
  }
  const int err = flash_run(a, pl, cur_stream());
  RAB_CHECK(err == 0, "flash_fwd launch failed: %s",
            cudaGetErrorString(static_cast<cudaError_t>(err)));
  // nsplit -1 reports the balanced schedule
  return {pl.balanced ? -1 : pl.nsplit, pl.n_items, pl.grid};
}

// The fused ring kernel run as rank `rank` of an emulated `world`-rank ring on
// ONE GPU: `blocks` holds every rank's ring-format slot-0 block
// ([world][slot_bytes] uint8); the "peer" slots and flag words the copy warps
// read are regions of this GPU's memory, with each peer's slot0_ready word
// set to the launch's epoch before the kernel starts and no peer reads to wait
// for.  Everything else - the copy role's slices, the per-block arrival
// counters, the TMA thread's waits on them, the generic->async proxy fence
// before TMA reads the copied bytes, the cooperative launch - is the code
// path of a real multi-GPU launch.  Direct mode (block s from its origin's
// slot 0).
std::vector<int64_t> flash_fused_loopback(int64_t prec, torch::Tensor q, torch::Tensor blocks,
                                          int64_t world, int64_t rank, int64_t Skv, int64_t Hkv,
                                          torch::Tensor out, c10::optional<torch::Tensor> lse,
                                          double scale, bool causal, bool zigzag,
                                          torch::Tensor status, double timeout_s) {
  const Prec pr = to_prec(prec);
  RAB_CHECK(q.is_cuda() && q.is_contiguous() && q.dim() == 3, "q must be contiguous [Sq, Hq, D]");
  RAB_CHECK(q.scalar_type() == (pr == Prec::kBF16 ? torch::kBFloat16 : torch::kFloat32),
            "q dtype does not match prec");
  RAB_CHECK(world >= 2 && world <= kMaxRanks && rank >= 0 && rank < world,
            "need 2 <= world <= %d and 0 <= rank < world", kMaxRanks);
  RAB_CHECK(status.is_cuda() && status.device() == q.device() &&
                status.scalar_type() == torch::kInt32 && status.numel() >= 8,
            "status must be int32[8] on q's GPU");
  const int64_t rows = q.size(0) * q.size(1);
  check_output(out, "out", q.device(), q.numel());
  RAB_CHECK(out.sizes() == q.sizes() &&
                (out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32),
            "out must be bfloat16/float32 with q's shape");
  if (lse) check_output(*lse, "lse", q.device(), rows);
  const size_t bb = ring_block_bytes(pr, static_cast<int>(Skv), static_cast<int>(Hkv),
                                     static_cast<int>(q.size(2)));
  RAB_CHECK(blocks.is_cuda() && blocks.device() == q.device() && blocks.is_contiguous() &&
                static_cast<size_t>(blocks.numel() * blocks.element_size()) >= bb * world,
            "blocks must hold world ring-format blocks on q's GPU");
  const c10::cuda::CUDAGuard guard(q.device());
  const auto u8 = torch::dtype(torch::kUInt8).device(q.device());
  // this rank's ring slots; slot 0 = its own block
  torch::Tensor local = torch::empty({static_cast<int64_t>(bb * world)}, u8);
  uint8_t* src = static_cast<uint8_t*>(blocks.data_ptr());
  local.narrow(0, 0, bb).copy_(blocks.narrow(0, rank * bb, bb));
  // flag words: row 0 this rank's, row 1 + r emulated peer r's (slot0_ready = epoch 1)
  torch::Tensor flags = torch::zeros({world + 1, 128}, torch::dtype(torch::kInt64).device(q.device()));
  flags.narrow(0, 1, world).select(1, kFlagSlot0Ready).fill_(1);
  uint64_t* fl = reinterpret_cast<uint64_t*>(flags.data_ptr());

  FlashArgs a;
  a.prec = pr;
  a.q = q.data_ptr();
  a.Sq = q.size(0);
  a.Hq = q.size(1);
  a.D = q.size(2);
  a.Hkv = static_cast<int>(Hkv);
  a.Skv = static_cast<int>(Skv);
  a.nblk = static_cast<int>(world);
  a.scale = static_cast<float>(scale);
  uint8_t* base = static_cast<uint8_t*>(local.data_ptr());
  a.k_base = base;
  a.v_base = base + ring_v_offset(pr, a.Skv, a.Hkv, a.D);
  a.slot_stride = bb;
  a.causal = causal;
  a.zigzag = zigzag;
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.out = out.data_ptr();
  a.out_bf16 = out.scalar_type() == torch::kBFloat16;
  a.lse = lse ? f32_ptr(*lse, "lse") : nullptr;
  a.status = reinterpret_cast<DeviceStatus*>(status.data_ptr());
  a.timeout_s = timeout_s;
  a.fused = true;
  a.local_slots = base;
  a.slot_bytes = bb;
  a.flags_local = fl;
  for (int r = 0; r < world; ++r) {
    a.peer_slots[r] = r == rank ? base : src + static_cast<size_t>(r) * bb;
    a.flags_peer[r] = r == rank ? fl : fl + static_cast<size_t>(1 + r) * 128;
  }
  const FlashPlan pl = flash_plan(a);
  a.epoch = 1;
  a.arrive_target = static_cast<uint64_t>(pl.grid);  // one slice per CTA and block
  a.reads_target = 0;                                 // no peer reads this rank's slots
  torch::Tensor ws;
  if (pl.workspace_bytes > 0) {
    ws = torch::empty({static_cast<int64_t>(pl.workspace_bytes)}, u8);
    a.workspace = ws.data_ptr();
    a.workspace_bytes = pl.workspace_bytes;
  }
  const int err = flash_run(a, pl, cur_stream());
  RAB_CHECK(err == 0, "fused loopback launch failed: %s",
            cudaGetErrorString(static_cast<cudaError_t>(err)));
  // keep the buffers alive until the kernel is done with them
  c10::cuda::getCurrentCUDAStream().synchronize();
  return {pl.balanced ? -1 : pl.nsplit, pl.n_items, pl.grid, pl.rows_per_unit};
}

}  // namespace
}  // namespace rab

namespace rab {
namespace {

// Host-only view of the planner (no GPU needed when sms > 0).
FlashArgs plan_args(int64_t prec, int64_t Sq, int64_t Skv, int64_t nblk, int64_t Hq, int64_t Hkv,
                    int64_t D, bool causal, bool zigzag, int64_t world, int64_t rank,
                    int64_t blk_offset, int64_t nsplit, int64_t sms, bool fused) {
  FlashArgs a;
  a.prec = to_prec(prec);
  a.Sq = static_cast<int>(Sq);
  a.Skv = static_cast<int>(Skv);
  a.nblk = static_cast<int>(nblk);
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.D = static_cast<int>(D);
  a.causal = causal;
  a.zigzag = zigzag;
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.blk_offset = static_cast<int>(blk_offset);
  a.nsplit = static_cast<int>(nsplit);
  a.sms = static_cast<int>(sms);
  a.fused = fused;
  return a;
}

}  // namespace
}  // namespace rab

void register_flash(pybind11::module_& m) {
  m.def(
      "flash_plan_info",
      [](int64_t prec, int64_t Sq, int64_t Skv, int64_t nblk, int64_t Hq, int64_t Hkv, int64_t D,
         bool causal, bool zigzag, int64_t world, int64_t rank, int64_t blk_offset, int64_t nsplit,
         int64_t sms, bool fused) {
        const rab::FlashPlan pl = rab::flash_plan(rab::plan_args(
            prec, Sq, Skv, nblk, Hq, Hkv, D, causal, zigzag, world, rank, blk_offset, nsplit, sms,
            fused));
        pybind11::dict d;
        d["rows_per_unit"] = pl.rows_per_unit;
        d["nsplit"] = pl.nsplit;
        d["balanced"] = pl.balanced;
        d["full_waves"] = pl.full_waves;
        d["dynamic"] = pl.dynamic;
        d["n_units"] = pl.n_units;
        d["n_items"] = pl.n_items;
        d["grid"] = pl.grid;
        d["workspace_bytes"] = pl.workspace_bytes;
        d["merge_kernel"] = pl.merge_kernel;
        return d;
      },
      pybind11::arg("prec"), pybind11::arg("Sq"), pybind11::arg("Skv"), pybind11::arg("nblk"),
      pybind11::arg("Hq"), pybind11::arg("Hkv"), pybind11::arg("D"), pybind11::arg("causal") = false,
      pybind11::arg("zigzag") = false, pybind11::arg("world") = 1, pybind11::arg("rank") = 0,
      pybind11::arg("blk_offset") = 0, pybind11::arg("nsplit") = 0, pybind11::arg("sms") = 0,
      pybind11::arg("fused") = false);
  m.def(
      "flash_visible_ranges",
      [](int64_t prec, int64_t Sq, int64_t Skv, int64_t nblk, bool zigzag, int64_t world,
         int64_t rank, int64_t blk_offset, int64_t q0) {
        return rab::flash_visible_ranges(
            rab::plan_args(prec, Sq, Skv, nblk, 1, 1, 64, true, zigzag, world, rank, blk_offset, 0,
                           1, false),
            static_cast<int>(q0));
      },
      pybind11::arg("prec"), pybind11::arg("Sq"), pybind11::arg("Skv"), pybind11::arg("nblk"),
      pybind11::arg("zigzag"), pybind11::arg("world"), pybind11::arg("rank"),
      pybind11::arg("blk_offset") = 0, pybind11::arg("q0") = 0);
  m.def("ring_block_bytes", [](int64_t prec, int64_t Skv, int64_t Hkv, int64_t D) {
    return static_cast<int64_t>(rab::ring_block_bytes(static_cast<rab::Prec>(prec), Skv, Hkv, D));
  });
  m.def("ring_v_offset", [](int64_t prec, int64_t Skv, int64_t Hkv, int64_t D) {
    return static_cast<int64_t>(rab::ring_v_offset(static_cast<rab::Prec>(prec), Skv, Hkv, D));
  });
  m.def("ring_format", &rab::ring_format, "write one K/V block into a ring slot");
  m.def("flash_fwd", &rab::flash_fwd, "tcgen05 flash attention over local ring slots",
        py::arg("prec"), py::arg("q"), py::arg("slots"), py::arg("nblk"), py::arg("Skv"),
        py::arg("Hkv"), py::arg("out") = c10::nullopt, py::arg("lse") = c10::nullopt,
        py::arg("scale") = 1.0, py::arg("causal") = false, py::arg("zigzag") = false,
        py::arg("world") = 1, py::arg("rank") = 0, py::arg("nsplit") = 0,
        py::arg("acc") = c10::nullopt, py::arg("m") = c10::nullopt, py::arg("l") = c10::nullopt,
        py::arg("status"), py::arg("timeout_s") = 10.0, py::arg("grid") = 0);
  m.def("sm_count", &rab::flash_sm_count);
  m.def("flash_fused_loopback", &rab::flash_fused_loopback,
        "fused ring kernel as one rank of an emulated ring on one GPU (peers in local memory)",
        py::arg("prec"), py::arg("q"), py::arg("blocks"), py::arg("world"), py::arg("rank"),
        py::arg("Skv"), py::arg("Hkv"), py::arg("out"), py::arg("lse") = c10::nullopt,
        py::arg("scale") = 1.0, py::arg("causal") = false, py::arg("zigzag") = false,
        py::arg("status"), py::arg("timeout_s") = 10.0);
}
