// ring_context.cpp - see ring_context.h.
#include "ring_context.h"

#include <cstring>
#include "strfmt.h"
#include <stdexcept>

namespace rab {

void cuda_check(cudaError_t err, const char* what) {
  if (err != cudaSuccess) {
    throw std::runtime_error(strfmt("%s: %s", what, cudaGetErrorString(err)));
  }
}

void nccl_check(ncclResult_t res, const char* what) {
  if (res != ncclSuccess) {
    throw std::runtime_error(strfmt("%s: %s", what, ncclGetErrorString(res)));
  }
}

RingContext::RingContext(int rank, int world, int device, const std::string& shm_name,
                         bool create_shm, size_t frag_bytes, size_t arena_bytes, double timeout_s)
    : rank_(rank), world_(world), device_(device) {
  host_ = std::make_unique<HostComm>(shm_name, rank, world, create_shm, frag_bytes, timeout_s);
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  flag_bytes_ = kFlagWords * sizeof(uint64_t);
  arena_bytes_ = ((arena_bytes + flag_bytes_ + (2u << 20) - 1) / (2u << 20)) * (2u << 20);
  cuda_check(cudaMalloc(&arena_, arena_bytes_), "cudaMalloc(arena)");
  cuda_check(cudaMemset(arena_, 0, flag_bytes_), "cudaMemset(flags)");
  arena_used_ = flag_bytes_;
  peers_.assign(world_, nullptr);
  peers_[rank_] = arena_;
  cuda_check(cudaStreamCreateWithFlags(&compute_, cudaStreamNonBlocking), "stream");
  cuda_check(cudaStreamCreateWithFlags(&comm_, cudaStreamNonBlocking), "stream");
  cuda_check(cudaMalloc(&status_dev_, sizeof(DeviceStatus)), "cudaMalloc(status)");
  cuda_check(cudaMemset(status_dev_, 0, sizeof(DeviceStatus)), "cudaMemset(status)");
  cuda_check(cudaDeviceSynchronize(), "init sync");
}

RingContext::~RingContext() {
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  if (nccl_ != nullptr) ncclCommDestroy(nccl_);
  for (int r = 0; r < world_; ++r)
    if (r != rank_ && peers_[r] != nullptr) cudaIpcCloseMemHandle(peers_[r]);
  if (status_dev_) cudaFree(status_dev_);
  if (compute_) cudaStreamDestroy(compute_);
  if (comm_) cudaStreamDestroy(comm_);
  if (arena_) cudaFree(arena_);
}

size_t RingContext::arena_alloc(size_t bytes, size_t align) {
  size_t off = (arena_used_ + align - 1) / align * align;
  if (off + bytes > arena_bytes_) {
    throw std::runtime_error(strfmt("arena_alloc: out of arena space (need %zu of %zu bytes)",
                                    off + bytes, arena_bytes_));
  }
  arena_used_ = off + bytes;
  return off;
}

uint8_t* RingContext::peer(int r, size_t off) const {
  if (r == rank_) return arena_ + off;
  if (!peers_open_ || peers_[r] == nullptr)
    throw std::runtime_error("RingContext: peer buffers are not mapped (call open_peers)");
  return peers_[r] + off;
}

std::string RingContext::ipc_handle() const {
  cudaIpcMemHandle_t h;
  cuda_check(cudaIpcGetMemHandle(&h, arena_), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void RingContext::open_peers(const std::vector<std::string>& handles) {
  if (static_cast<int>(handles.size()) != world_)
    throw std::runtime_error("open_peers: need one handle per rank");
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  for (int r = 0; r < world_; ++r) {
    if (r == rank_) continue;
    if (handles[r].size() != sizeof(cudaIpcMemHandle_t))
      throw std::runtime_error("open_peers: malformed IPC handle");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    void* p = nullptr;
    cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
               "cudaIpcOpenMemHandle");
    peers_[r] = static_cast<uint8_t*>(p);
  }
  peers_open_ = true;
}

std::string RingContext::nccl_unique_id() {
  ncclUniqueId id;
  nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId");
  return std::string(reinterpret_cast<const char*>(&id), sizeof(id));
}

void RingContext::init_nccl(const std::string& uid) {
  if (uid.size() != sizeof(ncclUniqueId)) throw std::runtime_error("init_nccl: bad unique id");
  ncclUniqueId id;
  std::memcpy(&id, uid.data(), sizeof(id));
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  nccl_check(ncclCommInitRank(&nccl_, world_, id, rank_), "ncclCommInitRank");
}

void RingContext::reset_flags() {
  // every rank's kernels (which may write into peers' flags) finish first
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  cuda_check(cudaDeviceSynchronize(), "reset_flags sync");
  host_->barrier();
  cuda_check(cudaMemset(arena_, 0, flag_bytes_), "reset_flags memset");
  cuda_check(cudaDeviceSynchronize(), "reset_flags sync");
  host_->ready_words()[rank_].v.store(0);
  host_->delivered_words()[rank_].v.store(0);
  host_->barrier();
  epoch_ = 0;
  step_seq_ = 0;
  xfer_seq_ = 0;
}

DeviceStatus RingContext::read_status(bool clear) {
  DeviceStatus s;
  cuda_check(cudaMemcpy(&s, status_dev_, sizeof(s), cudaMemcpyDeviceToHost), "read status");
  if (clear) cuda_check(cudaMemset(status_dev_, 0, sizeof(DeviceStatus)), "clear status");
  return s;
}

}  // namespace rab
