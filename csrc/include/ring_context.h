// ring_context.h - per-rank device runtime for the ring: device selection,
// a symmetric device arena mapped into every peer (CUDA IPC), the NCCL
// communicator of the `nccl` baseline, streams and the device status word.
//
// Device selection mirrors the reference's select_local_cuda_device
// (src/common/device_utils.cuh:44-81): local rank -> device local_rank % ndev,
// refusing more ranks than devices unless oversubscription is allowed.  Unlike
// the reference, backends that spin on peer flags inside a kernel refuse to run
// when two ranks share a GPU: kernels that wait on one another must never run
// on the same device.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "host_comm.h"
#include "status.h"

namespace rab {

void cuda_check(cudaError_t err, const char* what);
void nccl_check(ncclResult_t res, const char* what);

class RingContext {
 public:
  RingContext(int rank, int world, int device, const std::string& shm_name, bool create_shm,
              size_t frag_bytes, size_t arena_bytes, double timeout_s);
  ~RingContext();
  RingContext(const RingContext&) = delete;
  RingContext& operator=(const RingContext&) = delete;

  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }
  int right() const { return (rank_ + 1) % world_; }
  int left() const { return (rank_ - 1 + world_) % world_; }
  HostComm& host() { return *host_; }

  // --- symmetric arena -------------------------------------------------
  // Every rank allocates the same arena size and makes the same sequence of
  // arena_alloc calls, so an offset names the same buffer on every rank.
  size_t arena_bytes() const { return arena_bytes_; }
  size_t arena_alloc(size_t bytes, size_t align = 256);
  void arena_reset() { arena_used_ = flag_bytes_; }
  uint8_t* local(size_t off = 0) const { return arena_ + off; }
  uint8_t* peer(int r, size_t off = 0) const;  // r == rank -> local
  std::string ipc_handle() const;                // 64 raw bytes
  void open_peers(const std::vector<std::string>& handles);
  bool peers_open() const { return peers_open_; }
  bool devices_unique() const { return devices_unique_; }
  void set_devices_unique(bool u) { devices_unique_ = u; }

  // Flag words live at the start of the arena (zeroed at construction).
  uint64_t* flags_local() const { return reinterpret_cast<uint64_t*>(arena_); }
  uint64_t* flags_peer(int r) const { return reinterpret_cast<uint64_t*>(peer(r)); }
  static constexpr size_t kFlagWords = 8192;  // 64 KiB of uint64 flag words

  // --- NCCL ---------------------------------------------------------------
  static std::string nccl_unique_id();
  void init_nccl(const std::string& uid);
  bool has_nccl() const { return nccl_ != nullptr; }
  ncclComm_t nccl() const { return nccl_; }

  // --- streams / status -----------------------------------------------------
  cudaStream_t compute_stream() const { return compute_; }
  cudaStream_t comm_stream() const { return comm_; }
  DeviceStatus* status_dev() const { return status_dev_; }
  DeviceStatus read_status(bool clear);

  // Monotonic counters shared by the fused kernels of all ranks; every rank
  // advances them identically (same launches in the same order).
  uint64_t next_epoch() { return ++epoch_; }
  uint64_t epoch() const { return epoch_; }
  // Collective: zero every rank's device flag words and host transport words
  // and restart all sequence counters (all ranks must call it together).
  void reset_flags();
  uint64_t next_xfer() { return ++xfer_seq_; }

  uint64_t take_steps(uint64_t n) {
    const uint64_t b = step_seq_;
    step_seq_ += n;
    return b;
  }

 private:
  int rank_, world_, device_;
  std::unique_ptr<HostComm> host_;
  uint8_t* arena_ = nullptr;
  size_t arena_bytes_ = 0;
  size_t flag_bytes_ = 0;
  size_t arena_used_ = 0;
  std::vector<uint8_t*> peers_;
  bool peers_open_ = false;
  bool devices_unique_ = true;
  ncclComm_t nccl_ = nullptr;
  cudaStream_t compute_ = nullptr, comm_ = nullptr;
  DeviceStatus* status_dev_ = nullptr;
  uint64_t epoch_ = 0;
  uint64_t step_seq_ = 0;
  uint64_t xfer_seq_ = 0;
};

}  // namespace rab
