// host_comm.cpp - see host_comm.h.
#include "host_comm.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include "strfmt.h"
#include <thread>

namespace rab {

namespace {

constexpr uint64_t kMagic = 0x52414232303042ull;  // "RAB200B"

uint64_t now_ns() {
  return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                   std::chrono::steady_clock::now().time_since_epoch())
                                   .count());
}

inline void cpu_relax(uint64_t spins) {
  if (spins < 2048) {
#if defined(__x86_64__)
    __builtin_ia32_pause();
#endif
  } else {
    std::this_thread::yield();
  }
}

}  // namespace

HostComm::HostComm(const std::string& name, int rank, int world, bool create, size_t frag_bytes,
                   double timeout_s)
    : name_(name), rank_(rank), world_(world), frag_bytes_(frag_bytes), timeout_s_(timeout_s) {
  if (world < 1 || world > kMaxRanks)
    throw std::runtime_error("HostComm: world size must be 1.." + std::to_string(kMaxRanks));
  if (rank < 0 || rank >= world) throw std::runtime_error("HostComm: bad rank");
  if (frag_bytes == 0 || frag_bytes % 64 != 0)
    throw std::runtime_error("HostComm: frag_bytes must be a positive multiple of 64");
  const size_t header = (sizeof(ShmLayout) + 4095) & ~size_t(4095);
  map_bytes_ = header + static_cast<size_t>(world) * kMailSlots * frag_bytes;
  int fd = -1;
  if (create) {
    shm_unlink(name.c_str());  // stale segment of a crashed run with the same name
    fd = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
    if (fd < 0) throw std::runtime_error("HostComm: shm_open(create) failed for " + name);
    if (ftruncate(fd, static_cast<off_t>(map_bytes_)) != 0) {
      close(fd);
      shm_unlink(name.c_str());
      throw std::runtime_error("HostComm: ftruncate failed (is /dev/shm large enough?)");
    }
    owner_ = true;
  } else {
    fd = shm_open(name.c_str(), O_RDWR, 0600);
    if (fd < 0) throw std::runtime_error("HostComm: shm_open(attach) failed for " + name);
    struct stat sb;
    if (fstat(fd, &sb) != 0 || static_cast<size_t>(sb.st_size) != map_bytes_) {
      close(fd);
      throw std::runtime_error("HostComm: segment size mismatch for " + name +
                               " (different world/frag_bytes on another rank?)");
    }
  }
  void* p = mmap(nullptr, map_bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) throw std::runtime_error("HostComm: mmap failed");
  seg_ = static_cast<ShmLayout*>(p);
  mail_data_ = static_cast<uint8_t*>(p) + header;
  if (create) {
    // ftruncate zero-fills, so every counter starts at 0.
    seg_->world = world;
    seg_->frag_bytes = static_cast<int32_t>(frag_bytes);
    seg_->abort_rank.store(-1);
    std::atomic_thread_fence(std::memory_order_seq_cst);
    reinterpret_cast<std::atomic<uint64_t>*>(&seg_->magic)->store(kMagic, std::memory_order_release);
  } else {
    const uint64_t t0 = now_ns();
    while (reinterpret_cast<std::atomic<uint64_t>*>(&seg_->magic)->load(std::memory_order_acquire) !=
           kMagic) {
      if ((now_ns() - t0) * 1e-9 > timeout_s_)
        throw RankFailure("HostComm: segment " + name + " never initialised");
      std::this_thread::yield();
    }
    if (seg_->world != world || seg_->frag_bytes != static_cast<int32_t>(frag_bytes))
      throw std::runtime_error("HostComm: world/frag_bytes mismatch across ranks");
  }
}

HostComm::~HostComm() {
  if (seg_ != nullptr) munmap(seg_, map_bytes_);
  if (owner_ && !unlinked_) shm_unlink(name_.c_str());
}

void HostComm::unlink() {
  if (owner_ && !unlinked_) {
    shm_unlink(name_.c_str());
    unlinked_ = true;
  }
}

void HostComm::heartbeat() { seg_->heartbeat[rank_].v.store(now_ns(), std::memory_order_relaxed); }

bool HostComm::aborted() const { return seg_->abort_flag.load(std::memory_order_acquire) != 0; }

std::string HostComm::abort_message() const {
  return std::string(seg_->abort_msg, strnlen(seg_->abort_msg, sizeof(seg_->abort_msg)));
}

void HostComm::check_abort() const {
  if (aborted()) {
    throw RankFailure(strfmt("rank %d: job aborted by rank %d: %s", rank_,
                             seg_->abort_rank.load(), abort_message().c_str()));
  }
}

void HostComm::abort(const std::string& msg) {
  uint32_t expected = 0;
  if (seg_->abort_flag.compare_exchange_strong(expected, 1u)) {
    seg_->abort_rank.store(rank_);
    std::strncpy(seg_->abort_msg, msg.c_str(), sizeof(seg_->abort_msg) - 1);
  }
}

void HostComm::fail_timeout(const std::string& what) {
  const std::string msg = strfmt("rank %d: timed out after %.1f s %s", rank_, timeout_s_,
                                 what.c_str());
  abort(msg);
  throw RankFailure(msg);
}

void HostComm::barrier() {
  const uint64_t gen = ++generation_;
  seg_->arrive[rank_].v.store(gen, std::memory_order_release);
  const uint64_t t0 = now_ns();
  uint64_t spins = 0;
  while (true) {
    bool all = true;
    for (int r = 0; r < world_; ++r)
      if (seg_->arrive[r].v.load(std::memory_order_acquire) < gen) {
        all = false;
        break;
      }
    if (all) return;
    check_abort();
    if ((++spins & 255) == 0) {
      heartbeat();
      if ((now_ns() - t0) * 1e-9 > timeout_s_) {
        std::string what = strfmt("in barrier %llu; missing ranks:", (unsigned long long)gen);
        for (int r = 0; r < world_; ++r)
          if (seg_->arrive[r].v.load() < gen) what += strfmt(" %d", r);
        fail_timeout(what);
      }
    }
    cpu_relax(spins);
  }
}

std::vector<double> HostComm::reduce_max(const std::vector<double>& vals) {
  if (vals.size() > static_cast<size_t>(kReduceWidth))
    throw std::runtime_error("reduce_max: at most 16 values");
  const int buf = static_cast<int>(reduce_round_++ & 1);
  for (size_t i = 0; i < vals.size(); ++i) seg_->reduce_buf[buf][rank_][i] = vals[i];
  barrier();
  std::vector<double> out(vals);
  for (int r = 0; r < world_; ++r)
    for (size_t i = 0; i < vals.size(); ++i)
      out[i] = std::max(out[i], seg_->reduce_buf[buf][r][i]);
  // The other buffer is used next round, so a second barrier is not needed
  // before it is rewritten: a rank can only get two rounds ahead after every
  // rank has passed this round's barrier.
  return out;
}

void HostComm::publish(std::atomic<uint64_t>& word, uint64_t value) {
  word.store(value, std::memory_order_release);
}

void HostComm::wait_at_least(const std::atomic<uint64_t>& word, uint64_t value, const char* what,
                             int peer) {
  if (word.load(std::memory_order_acquire) >= value) return;
  const uint64_t t0 = now_ns();
  uint64_t spins = 0;
  while (word.load(std::memory_order_acquire) < value) {
    check_abort();
    if ((++spins & 255) == 0) {
      heartbeat();
      if ((now_ns() - t0) * 1e-9 > timeout_s_) {
        fail_timeout(strfmt("waiting for %s of rank %d to reach %llu", what, peer,
                            (unsigned long long)value));
      }
    }
    cpu_relax(spins);
  }
}

void HostComm::ring_sendrecv(const void* send, void* recv, size_t bytes) {
  if (world_ == 1) {
    if (send != recv) std::memcpy(recv, send, bytes);
    return;
  }
  const int right = (rank_ + 1) % world_;
  const int left = (rank_ - 1 + world_) % world_;
  const size_t nfrag = (bytes + frag_bytes_ - 1) / frag_bytes_;
  const uint8_t* src = static_cast<const uint8_t*>(send);
  uint8_t* dst = static_cast<uint8_t*>(recv);
  size_t sent = 0, got = 0;
  const uint64_t send_base = frags_sent_, recv_base = frags_received_;
  uint64_t t_last = now_ns();
  uint64_t spins = 0;
  while (sent < nfrag || got < nfrag) {
    bool progressed = false;
    if (sent < nfrag) {
      const uint64_t g = send_base + sent;  // global fragment number toward right
      const int slot = static_cast<int>(g % kMailSlots);
      // the slot is free once the right neighbour consumed fragment g - kMailSlots
      if (g < kMailSlots ||
          seg_->mail_read[right][slot].v.load(std::memory_order_acquire) >= g - kMailSlots + 1) {
        const size_t off = sent * frag_bytes_;
        const size_t n = std::min(frag_bytes_, bytes - off);
        std::memcpy(mail_data_ + (static_cast<size_t>(right) * kMailSlots + slot) * frag_bytes_,
                    src + off, n);
        seg_->mail_written[right][slot].v.store(g + 1, std::memory_order_release);
        ++sent;
        progressed = true;
      }
    }
    if (got < nfrag) {
      const uint64_t g = recv_base + got;
      const int slot = static_cast<int>(g % kMailSlots);
      if (seg_->mail_written[rank_][slot].v.load(std::memory_order_acquire) == g + 1) {
        const size_t off = got * frag_bytes_;
        const size_t n = std::min(frag_bytes_, bytes - off);
        std::memcpy(dst + off,
                    mail_data_ + (static_cast<size_t>(rank_) * kMailSlots + slot) * frag_bytes_, n);
        seg_->mail_read[rank_][slot].v.store(g + 1, std::memory_order_release);
        ++got;
        progressed = true;
      }
    }
    if (progressed) {
      t_last = now_ns();
      spins = 0;
      continue;
    }
    check_abort();
    if ((++spins & 255) == 0) {
      heartbeat();
      if ((now_ns() - t_last) * 1e-9 > timeout_s_) {
        fail_timeout(strfmt("in ring_sendrecv (sent %zu/%zu fragments to rank %d, received "
                            "%zu/%zu from rank %d)", sent, nfrag, right, got, nfrag, left));
      }
    }
    cpu_relax(spins);
  }
  frags_sent_ += nfrag;
  frags_received_ += nfrag;
}

}  // namespace rab
