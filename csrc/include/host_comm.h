// host_comm.h - node-local control plane over a POSIX shared-memory segment.
//
// Replaces what the reference asks of MPI on the host side
// (src/loop/ring_loop_staged.cu: MPI_Barrier at :173, MPI_Sendrecv of pinned
// host buffers at :187, MPI_Reduce(MPI_MAX) of the phase timers at :221) with
// native equivalents for ranks on one node:
//   * barrier(): generation counters, bounded wait, names the missing ranks
//   * reduce_max(): element-wise max of a few doubles over all ranks
//   * ring_sendrecv(): send a host buffer to the right neighbour and receive
//     one from the left neighbour through fixed-size fragment mailboxes
//     (copy-in / copy-out, the way an MPI shared-memory transport moves data)
//   * flag words for device-to-device transports (ready / delivered)
//   * an abort word: the first rank that fails publishes it and every other
//     rank's next wait raises instead of running into its timeout.
// Every wait is bounded by `timeout_s`; expiry throws RankFailure.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace rab {

constexpr int kMaxRanks = 16;
constexpr int kMailSlots = 4;
constexpr int kReduceWidth = 16;

class RankFailure : public std::runtime_error {
 public:
  explicit RankFailure(const std::string& what) : std::runtime_error(what) {}
};

struct alignas(64) PaddedU64 {
  std::atomic<uint64_t> v;
  char pad[64 - sizeof(std::atomic<uint64_t>)];
};

struct ShmLayout {
  uint64_t magic;
  int32_t world;
  int32_t frag_bytes;
  alignas(64) std::atomic<uint32_t> abort_flag;
  std::atomic<int32_t> abort_rank;
  char abort_msg[240];
  PaddedU64 arrive[kMaxRanks];        // barrier generation reached by each rank
  PaddedU64 heartbeat[kMaxRanks];     // monotonic ns of each rank's last wait
  alignas(64) double reduce_buf[2][kMaxRanks][kReduceWidth];
  // staged transport: mailbox of rank r is written by r's left neighbour
  PaddedU64 mail_written[kMaxRanks][kMailSlots];  // fragment sequence (+1) in the slot
  PaddedU64 mail_read[kMaxRanks][kMailSlots];     // fragment sequence (+1) consumed
  // device transports: per-rank monotonically increasing step counters
  PaddedU64 ready[kMaxRanks];      // rank's receive buffer is free for step n
  PaddedU64 delivered[kMaxRanks];  // data for rank's step n has landed in its buffer
  PaddedU64 user[kMaxRanks][4];    // spare words for tests / tools
};

class HostComm {
 public:
  // create=true: rank 0 creates (and sizes) the segment; others attach.
  HostComm(const std::string& name, int rank, int world, bool create, size_t frag_bytes,
           double timeout_s);
  ~HostComm();
  HostComm(const HostComm&) = delete;
  HostComm& operator=(const HostComm&) = delete;

  int rank() const { return rank_; }
  int world() const { return world_; }
  double timeout_s() const { return timeout_s_; }
  void set_timeout(double s) { timeout_s_ = s; }
  void unlink();  // remove the name; the mapping stays valid

  void barrier();
  std::vector<double> reduce_max(const std::vector<double>& vals);
  // Ring exchange: send `bytes` from `send` to (rank+1)%world, receive the
  // same amount from (rank-1+world)%world into `recv`.  Interleaves both
  // directions fragment by fragment, so it cannot deadlock.
  void ring_sendrecv(const void* send, void* recv, size_t bytes);

  // device-transport flag words (monotonic counters)
  void publish(std::atomic<uint64_t>& word, uint64_t value);
  void wait_at_least(const std::atomic<uint64_t>& word, uint64_t value, const char* what,
                     int peer);
  PaddedU64* ready_words() { return seg_->ready; }
  PaddedU64* delivered_words() { return seg_->delivered; }
  std::atomic<uint64_t>& user_word(int r, int i) { return seg_->user[r][i].v; }

  void abort(const std::string& msg);
  bool aborted() const;
  std::string abort_message() const;
  void check_abort() const;

 private:
  void heartbeat();
  [[noreturn]] void fail_timeout(const std::string& what);

  std::string name_;
  int rank_ = 0, world_ = 1;
  size_t frag_bytes_ = 0;
  double timeout_s_ = 60.0;
  size_t map_bytes_ = 0;
  ShmLayout* seg_ = nullptr;
  uint8_t* mail_data_ = nullptr;  // [world][kMailSlots][frag_bytes]
  uint64_t generation_ = 0;
  uint64_t reduce_round_ = 0;
  uint64_t frags_sent_ = 0;      // fragments sent to the right neighbour
  uint64_t frags_received_ = 0;  // fragments received from the left neighbour
  bool owner_ = false;
  bool unlinked_ = false;
};

}  // namespace rab
