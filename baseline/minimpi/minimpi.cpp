// minimpi.cpp - a one-node implementation of the MPI subset declared in mpi.h,
// so the reference benchmark's MPI programs build and run unmodified where no
// MPI is installed.  It is launch plumbing for the reference arm, not part of
// the framework's own data path.
//
// Ranks: every process of a job reads its rank and size from the launcher's
// environment (OMPI_COMM_WORLD_RANK/SIZE, PMI_RANK/SIZE or RANK/WORLD_SIZE)
// and a job name from MINIMPI_JOB.  Rank 0 creates a POSIX shared-memory
// header /mmpi_<job> (barrier counter, reduce and broadcast areas, abort
// word); the others attach to it.
//
// Point-to-point: one shared-memory channel per ordered (source, destination)
// pair, created on first use: a ring of 4 slots of 512 KiB with a head
// (written by the sender) and a tail (by the receiver).  Messages on a channel
// are matched in the order they were posted (MPI's non-overtaking rule; the
// receive's tag must match the message's, MPI_ANY_TAG matches any).
//  * host buffers: eager, copied through the slots in fragments;
//  * device buffers (cudaMalloc memory): one slot carries a CUDA IPC handle of
//    the sender's allocation and the offset; the receiver maps it once
//    (cached), copies GPU to GPU with cuMemcpyAsync on a non-blocking stream of
//    its own (so it never waits for, or blocks, the application's streams),
//    and acknowledges when the copy's event completes; the send completes on
//    that acknowledgement.  This is the rendezvous protocol of an intra-node
//    CUDA-aware MPI.
// Progress happens inside every MPI call that waits or tests.
//
// The CUDA driver API is loaded with dlopen at first use, so the library
// needs no CUDA runtime of its own and shares the application's current
// context (the device the application selected).  Without a driver every
// buffer is treated as host memory.
//
// Every wait is bounded (MINIMPI_TIMEOUT_S, default 600 s) and watches the
// abort word: MPI_Abort in any rank ends every rank with that code.
#include "mpi.h"

#include <cuda.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <sched.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <array>
#include <atomic>
#include <cerrno>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <string>
#include <utility>
#include <vector>

namespace {

constexpr uint64_t kMagic = 0x314950494d494e4dULL;
constexpr int kMaxRanks = 64;
constexpr int kReduceBytes = 4096;      // per rank per reduce round
constexpr size_t kBcastBytes = 64 << 10;  // per broadcast round
constexpr int kSlots = 4;
constexpr size_t kFrag = 512 << 10;

struct Header {
  std::atomic<uint64_t> magic;
  std::atomic<uint32_t> world;
  std::atomic<uint32_t> attached;
  alignas(64) std::atomic<uint64_t> barrier_arrivals;
  alignas(64) std::atomic<int32_t> abort_code;  // errorcode + 1; 0: no abort
  std::atomic<int32_t> abort_rank;
  alignas(64) unsigned char reduce_buf[kMaxRanks][kReduceBytes];
  alignas(64) unsigned char bcast_buf[kBcastBytes];
};

enum : uint32_t { kKindHost = 1, kKindIpc = 2, kKindSelfDevice = 3 };

struct SlotHdr {
  int32_t tag;
  uint32_t kind;
  uint64_t msg_bytes;
  uint64_t frag_off;
  uint64_t frag_bytes;
  uint64_t offset;               // IPC: byte offset inside the exported allocation
  unsigned char handle[64];      // IPC: CUipcMemHandle of the allocation
};

struct Chan {
  alignas(64) std::atomic<uint64_t> head;      // fragments posted by the sender
  alignas(64) std::atomic<uint64_t> tail;      // fragments taken by the receiver
  alignas(64) std::atomic<uint64_t> ipc_done;  // device messages the receiver finished copying
  SlotHdr hdr[kSlots];
  alignas(4096) unsigned char data[kSlots][kFrag];
};

// ------------------------------------------------------------------ driver API
struct Cu {
  bool ok = false;
  CUresult (*ctxGetCurrent)(CUcontext*) = nullptr;
  CUresult (*pointerGetAttribute)(void*, CUpointer_attribute, CUdeviceptr) = nullptr;
  CUresult (*memGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr) = nullptr;
  CUresult (*ipcGetMemHandle)(CUipcMemHandle*, CUdeviceptr) = nullptr;
  CUresult (*ipcOpenMemHandle)(CUdeviceptr*, CUipcMemHandle, unsigned int) = nullptr;
  CUresult (*ipcCloseMemHandle)(CUdeviceptr) = nullptr;
  CUresult (*streamCreate)(CUstream*, unsigned int) = nullptr;
  CUresult (*streamDestroy)(CUstream) = nullptr;
  CUresult (*memcpyAsync)(CUdeviceptr, CUdeviceptr, size_t, CUstream) = nullptr;
  CUresult (*memcpy)(CUdeviceptr, CUdeviceptr, size_t) = nullptr;
  CUresult (*eventCreate)(CUevent*, unsigned int) = nullptr;
  CUresult (*eventDestroy)(CUevent) = nullptr;
  CUresult (*eventRecord)(CUevent, CUstream) = nullptr;
  CUresult (*eventQuery)(CUevent) = nullptr;
};

template <class F>
bool sym(void* lib, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(lib, name));
  return f != nullptr;
}

Cu& cu() {
  static Cu c;
  static bool tried = false;
  if (tried) return c;
  tried = true;
  void* lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
  if (lib == nullptr) return c;
  c.ok = sym(lib, "cuCtxGetCurrent", c.ctxGetCurrent) &&
         sym(lib, "cuPointerGetAttribute", c.pointerGetAttribute) &&
         sym(lib, "cuMemGetAddressRange_v2", c.memGetAddressRange) &&
         sym(lib, "cuIpcGetMemHandle", c.ipcGetMemHandle) &&
         sym(lib, "cuIpcOpenMemHandle_v2", c.ipcOpenMemHandle) &&
         sym(lib, "cuIpcCloseMemHandle", c.ipcCloseMemHandle) &&
         sym(lib, "cuStreamCreate", c.streamCreate) &&
         sym(lib, "cuStreamDestroy_v2", c.streamDestroy) &&
         sym(lib, "cuMemcpyAsync", c.memcpyAsync) && sym(lib, "cuMemcpy", c.memcpy) &&
         sym(lib, "cuEventCreate", c.eventCreate) &&
         sym(lib, "cuEventDestroy_v2", c.eventDestroy) &&
         sym(lib, "cuEventRecord", c.eventRecord) && sym(lib, "cuEventQuery", c.eventQuery);
  return c;
}

bool is_device_ptr(const void* p) {
  Cu& c = cu();
  if (!c.ok || p == nullptr) return false;
  CUcontext ctx = nullptr;
  if (c.ctxGetCurrent(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  unsigned int type = 0;
  if (c.pointerGetAttribute(&type, CU_POINTER_ATTRIBUTE_MEMORY_TYPE,
                            reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
    return false;
  return type == CU_MEMORYTYPE_DEVICE;
}

// --------------------------------------------------------------------- state

struct State {
  bool initialized = false;
  bool finalized = false;
  int rank = 0;
  int world = 1;
  std::string job;
  Header* hdr = nullptr;
  uint64_t barrier_gen = 0;
  double timeout_s = 600.0;
  Chan* chans_out[kMaxRanks] = {};  // this rank -> r
  Chan* chans_in[kMaxRanks] = {};   // r -> this rank
  std::vector<std::string> chan_names;
  uint64_t ipc_posted[kMaxRanks] = {};
  std::deque<MPI_Request> sendq[kMaxRanks];
  std::deque<MPI_Request> recvq[kMaxRanks];
  CUstream stream = nullptr;
  std::map<CUdeviceptr, std::pair<size_t, CUipcMemHandle>> exported;  // base -> (size, handle)
  std::map<std::pair<int, std::array<unsigned char, 64>>, CUdeviceptr> imported;
  int next_comm = 3;
};

State& S() {
  static State s;
  return s;
}

// Remove this job's shared-memory names this rank knows of (an ending job
// leaves nothing behind in /dev/shm; existing mappings stay valid).
void unlink_names() {
  State& s = S();
  for (const auto& n : s.chan_names) shm_unlink(n.c_str());
  if (!s.job.empty()) shm_unlink(("/mmpi_" + s.job).c_str());
}

[[noreturn]] void die(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  fprintf(stderr, "[minimpi] rank %d: ", S().rank);
  vfprintf(stderr, fmt, ap);
  fprintf(stderr, "\n");
  va_end(ap);
  fflush(stderr);
  fflush(stdout);
  if (S().hdr != nullptr) {
    int32_t expected = 0;
    if (S().hdr->abort_code.compare_exchange_strong(expected, code + 1))
      S().hdr->abort_rank.store(S().rank);
  }
  unlink_names();
  _exit(code);
}

double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return static_cast<double>(ts.tv_sec) + 1e-9 * static_cast<double>(ts.tv_nsec);
}

void check_abort() {
  Header* h = S().hdr;
  if (h == nullptr) return;
  const int32_t c = h->abort_code.load(std::memory_order_acquire);
  if (c != 0) {
    fprintf(stderr, "[minimpi] rank %d: rank %d called MPI_Abort(%d); exiting\n", S().rank,
            h->abort_rank.load(), c - 1);
    fflush(stderr);
    fflush(stdout);
    unlink_names();
    _exit(c - 1);
  }
}

// Spin-then-yield wait helper with the global time limit and abort check.
struct Waiter {
  double t0 = now_s();
  uint64_t n = 0;
  const char* what;
  explicit Waiter(const char* w) : what(w) {}
  void pause() {
    ++n;
    if (n < 2000) {
#if defined(__x86_64__)
      __builtin_ia32_pause();
#endif
      return;
    }
    sched_yield();
    if ((n & 1023) == 0) {
      check_abort();
      if (now_s() - t0 > S().timeout_s)
        die(MPI_ERR_OTHER, "timed out after %.0f s waiting for %s", S().timeout_s, what);
    }
  }
};

void* map_shm(const std::string& name, size_t bytes, bool create_fresh) {
  int fd;
  if (create_fresh) {
    shm_unlink(name.c_str());
    fd = shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  } else {
    fd = shm_open(name.c_str(), O_CREAT | O_RDWR, 0600);
  }
  if (fd < 0) die(MPI_ERR_OTHER, "shm_open(%s) failed: %s", name.c_str(), strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || static_cast<size_t>(st.st_size) < bytes) {
    if (ftruncate(fd, static_cast<off_t>(bytes)) != 0)
      die(MPI_ERR_OTHER, "ftruncate(%s, %zu) failed: %s", name.c_str(), bytes, strerror(errno));
  }
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) die(MPI_ERR_OTHER, "mmap(%s) failed: %s", name.c_str(), strerror(errno));
  return p;
}

// The channel src -> dst, mapped on first use by either side (a message to
// oneself uses chans_out[rank] for both ends).
Chan* channel(int src, int dst) {
  State& s = S();
  Chan*& slot = src == s.rank ? s.chans_out[dst] : s.chans_in[src];
  if (slot == nullptr) {
    const std::string name = "/mmpi_" + s.job + "_" + std::to_string(src) + "_" +
                             std::to_string(dst);
    slot = static_cast<Chan*>(map_shm(name, sizeof(Chan), false));
    s.chan_names.push_back(name);
  }
  return slot;
}

size_t type_size(MPI_Datatype t) {
  switch (t) {
    case MPI_CHAR:
    case MPI_BYTE: return 1;
    case MPI_INT:
    case MPI_FLOAT:
    case MPI_UNSIGNED: return 4;
    case MPI_DOUBLE:
    case MPI_LONG_LONG:
    case MPI_UNSIGNED_LONG_LONG: return 8;
    default: die(MPI_ERR_OTHER, "unsupported MPI_Datatype %d", t);
  }
}

int comm_rank(MPI_Comm c) { return c == MPI_COMM_SELF ? 0 : S().rank; }
int comm_size(MPI_Comm c) { return c == MPI_COMM_SELF ? 1 : S().world; }
void check_comm(MPI_Comm c) {
  if (c == MPI_COMM_NULL || c < 0 || c >= S().next_comm)
    die(MPI_ERR_OTHER, "invalid communicator %d", c);
}

// Copy between any two buffers (host or device, unified addressing).
void copy_any(void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return;
  if (is_device_ptr(dst) || is_device_ptr(src)) {
    if (cu().memcpy(reinterpret_cast<CUdeviceptr>(dst), reinterpret_cast<CUdeviceptr>(src),
                    bytes) != CUDA_SUCCESS)
      die(MPI_ERR_OTHER, "cuMemcpy of %zu bytes failed", bytes);
    return;
  }
  memcpy(dst, src, bytes);
}

CUstream copy_stream() {
  State& s = S();
  if (s.stream == nullptr && cu().streamCreate(&s.stream, CU_STREAM_NON_BLOCKING) != CUDA_SUCCESS)
    die(MPI_ERR_OTHER, "cuStreamCreate failed");
  return s.stream;
}

void barrier_world() {
  State& s = S();
  if (s.world == 1) return;
  ++s.barrier_gen;
  s.hdr->barrier_arrivals.fetch_add(1, std::memory_order_acq_rel);
  const uint64_t target = s.barrier_gen * static_cast<uint64_t>(s.world);
  Waiter w("a barrier");
  while (s.hdr->barrier_arrivals.load(std::memory_order_acquire) < target) w.pause();
}

}  // namespace

// ---------------------------------------------------------------- requests
struct minimpi_request {
  bool send = false;
  int peer = 0;
  int tag = 0;
  const unsigned char* sbuf = nullptr;
  unsigned char* rbuf = nullptr;
  size_t bytes = 0;       // send: message size; recv: capacity
  size_t moved = 0;       // bytes posted (send) or taken (recv)
  bool device = false;    // the local buffer is device memory
  int state = 0;          // 0: moving data; 1: device copy / acknowledgement pending; 2: done
  bool posted_any = false;
  uint64_t ipc_seq = 0;
  CUevent ev = nullptr;
  size_t msg_bytes = 0;   // recv: size of the matched message
  int msg_tag = 0;
  int error = MPI_SUCCESS;
};

namespace {

void advance_send(MPI_Request r) {
  State& s = S();
  Chan* ch = channel(s.rank, r->peer);
  if (r->state == 1) {
    if (ch->ipc_done.load(std::memory_order_acquire) >= r->ipc_seq) r->state = 2;
    return;
  }
  while (r->state == 0) {
    const uint64_t head = ch->head.load(std::memory_order_relaxed);
    if (head - ch->tail.load(std::memory_order_acquire) >= kSlots) return;  // channel full
    SlotHdr& h = ch->hdr[head % kSlots];
    h.tag = r->tag;
    h.msg_bytes = r->bytes;
    if (r->device) {
      const CUdeviceptr p = reinterpret_cast<CUdeviceptr>(r->sbuf);
      if (r->peer == s.rank) {
        h.kind = kKindSelfDevice;
        h.offset = static_cast<uint64_t>(p);
      } else {
        CUdeviceptr base = 0;
        size_t size = 0;
        if (cu().memGetAddressRange(&base, &size, p) != CUDA_SUCCESS)
          die(MPI_ERR_OTHER, "cuMemGetAddressRange failed for a device send buffer");
        auto it = s.exported.find(base);
        if (it == s.exported.end() || it->second.first != size) {
          CUipcMemHandle hd;
          if (cu().ipcGetMemHandle(&hd, base) != CUDA_SUCCESS)
            die(MPI_ERR_OTHER, "cuIpcGetMemHandle failed (device buffers must come from "
                               "cudaMalloc)");
          it = s.exported.insert_or_assign(base, std::make_pair(size, hd)).first;
        }
        h.kind = kKindIpc;
        h.offset = static_cast<uint64_t>(p - base);
        static_assert(sizeof(CUipcMemHandle) == 64, "IPC handle size");
        memcpy(h.handle, &it->second.second, 64);
      }
      h.frag_off = 0;
      h.frag_bytes = r->bytes;
      r->ipc_seq = ++s.ipc_posted[r->peer];
      ch->head.store(head + 1, std::memory_order_release);
      r->state = 1;
      if (ch->ipc_done.load(std::memory_order_acquire) >= r->ipc_seq) r->state = 2;
      return;
    }
    const size_t n = r->bytes - r->moved < kFrag ? r->bytes - r->moved : kFrag;
    h.kind = kKindHost;
    h.frag_off = r->moved;
    h.frag_bytes = n;
    if (n > 0) memcpy(ch->data[head % kSlots], r->sbuf + r->moved, n);
    ch->head.store(head + 1, std::memory_order_release);
    r->moved += n;
    r->posted_any = true;
    if (r->moved == r->bytes) r->state = 2;  // eager: the data sits in the channel
  }
}

void advance_recv(MPI_Request r) {
  State& s = S();
  Chan* ch = channel(r->peer, s.rank);
  if (r->state == 1) {
    const CUresult q = cu().eventQuery(r->ev);
    if (q == CUDA_ERROR_NOT_READY) return;
    if (q != CUDA_SUCCESS) die(MPI_ERR_OTHER, "device copy of a received message failed");
    ch->ipc_done.fetch_add(1, std::memory_order_acq_rel);
    r->state = 2;
    return;
  }
  while (r->state == 0) {
    const uint64_t tail = ch->tail.load(std::memory_order_relaxed);
    if (tail >= ch->head.load(std::memory_order_acquire)) return;  // nothing yet
    const SlotHdr& h = ch->hdr[tail % kSlots];
    if (r->tag != MPI_ANY_TAG && h.tag != r->tag)
      die(MPI_ERR_OTHER,
          "message from rank %d has tag %d but the oldest posted receive expects tag %d "
          "(messages between two ranks are matched in order)",
          r->peer, h.tag, r->tag);
    if (h.msg_bytes > r->bytes)
      die(MPI_ERR_TRUNCATE, "message of %llu bytes from rank %d exceeds the %zu-byte receive",
          static_cast<unsigned long long>(h.msg_bytes), r->peer, r->bytes);
    r->msg_bytes = h.msg_bytes;
    r->msg_tag = h.tag;
    if (h.kind == kKindIpc || h.kind == kKindSelfDevice) {
      CUdeviceptr src;
      if (h.kind == kKindSelfDevice) {
        src = static_cast<CUdeviceptr>(h.offset);
      } else {
        std::array<unsigned char, 64> key;
        memcpy(key.data(), h.handle, 64);
        auto it = s.imported.find({r->peer, key});
        if (it == s.imported.end()) {
          CUipcMemHandle hd;
          memcpy(&hd, h.handle, 64);
          CUdeviceptr base = 0;
          if (cu().ipcOpenMemHandle(&base, hd, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS) !=
              CUDA_SUCCESS)
            die(MPI_ERR_OTHER, "cuIpcOpenMemHandle of rank %d's buffer failed", r->peer);
          it = s.imported.emplace(std::make_pair(r->peer, key), base).first;
        }
        src = it->second + h.offset;
      }
      if (r->ev == nullptr && cu().eventCreate(&r->ev, CU_EVENT_DISABLE_TIMING) != CUDA_SUCCESS)
        die(MPI_ERR_OTHER, "cuEventCreate failed");
      if (h.msg_bytes > 0 &&
          cu().memcpyAsync(reinterpret_cast<CUdeviceptr>(r->rbuf), src, h.msg_bytes,
                           copy_stream()) != CUDA_SUCCESS)
        die(MPI_ERR_OTHER, "cuMemcpyAsync of %llu bytes from rank %d failed",
            static_cast<unsigned long long>(h.msg_bytes), r->peer);
      if (cu().eventRecord(r->ev, copy_stream()) != CUDA_SUCCESS)
        die(MPI_ERR_OTHER, "cuEventRecord failed");
      ch->tail.store(tail + 1, std::memory_order_release);  // the slot held only the handle
      r->moved = h.msg_bytes;
      r->state = 1;
      advance_recv(r);
      return;
    }
    copy_any(r->rbuf + h.frag_off, ch->data[tail % kSlots], h.frag_bytes);
    const bool last = h.frag_off + h.frag_bytes == h.msg_bytes;
    ch->tail.store(tail + 1, std::memory_order_release);
    r->moved += h.frag_bytes;
    if (last) r->state = 2;
  }
}

// Advance every pending request in posting order per channel; completed
// requests leave their queue (their handles stay valid until waited on).
void progress() {
  State& s = S();
  for (int p = 0; p < s.world; ++p) {
    while (!s.sendq[p].empty()) {
      MPI_Request r = s.sendq[p].front();
      advance_send(r);
      if (r->state != 2) break;
      s.sendq[p].pop_front();
    }
    while (!s.recvq[p].empty()) {
      MPI_Request r = s.recvq[p].front();
      advance_recv(r);
      if (r->state != 2) break;
      s.recvq[p].pop_front();
    }
  }
}

void fill_status(MPI_Request r, MPI_Status* st) {
  if (st == MPI_STATUS_IGNORE) return;
  st->MPI_SOURCE = r->peer;
  st->MPI_TAG = r->send ? r->tag : r->msg_tag;
  st->MPI_ERROR = r->error;
  st->minimpi_count_bytes = static_cast<int>(r->send ? r->bytes : r->msg_bytes);
}

void release(MPI_Request* req) {
  if ((*req)->ev != nullptr) cu().eventDestroy((*req)->ev);
  delete *req;
  *req = MPI_REQUEST_NULL;
}

void require_init(const char* fn) {
  if (!S().initialized || S().finalized) die(MPI_ERR_OTHER, "%s called outside MPI_Init/Finalize", fn);
}

int env_int(const char* const* names, int dflt) {
  for (int i = 0; names[i] != nullptr; ++i) {
    const char* v = getenv(names[i]);
    if (v != nullptr && v[0] != '\0') return atoi(v);
  }
  return dflt;
}

template <class T>
void reduce_into(T* acc, const T* x, size_t n, MPI_Op op) {
  for (size_t i = 0; i < n; ++i) {
    if (op == MPI_MAX)
      acc[i] = x[i] > acc[i] ? x[i] : acc[i];
    else if (op == MPI_MIN)
      acc[i] = x[i] < acc[i] ? x[i] : acc[i];
    else
      acc[i] += x[i];
  }
}

void reduce_chunk(unsigned char* acc, const unsigned char* x, size_t n, MPI_Datatype t, MPI_Op op) {
  switch (t) {
    case MPI_INT: reduce_into(reinterpret_cast<int32_t*>(acc), reinterpret_cast<const int32_t*>(x), n, op); break;
    case MPI_UNSIGNED: reduce_into(reinterpret_cast<uint32_t*>(acc), reinterpret_cast<const uint32_t*>(x), n, op); break;
    case MPI_FLOAT: reduce_into(reinterpret_cast<float*>(acc), reinterpret_cast<const float*>(x), n, op); break;
    case MPI_DOUBLE: reduce_into(reinterpret_cast<double*>(acc), reinterpret_cast<const double*>(x), n, op); break;
    case MPI_LONG_LONG: reduce_into(reinterpret_cast<int64_t*>(acc), reinterpret_cast<const int64_t*>(x), n, op); break;
    case MPI_UNSIGNED_LONG_LONG: reduce_into(reinterpret_cast<uint64_t*>(acc), reinterpret_cast<const uint64_t*>(x), n, op); break;
    default: die(MPI_ERR_OTHER, "reduction on MPI_Datatype %d is not supported", t);
  }
}

int reduce_impl(const void* sendbuf, void* recvbuf, int count, MPI_Datatype t, MPI_Op op,
                int root, MPI_Comm comm, bool all) {
  require_init(all ? "MPI_Allreduce" : "MPI_Reduce");
  check_comm(comm);
  if (op != MPI_MAX && op != MPI_MIN && op != MPI_SUM) die(MPI_ERR_OTHER, "unsupported MPI_Op %d", op);
  State& s = S();
  const size_t es = type_size(t);
  const size_t total = static_cast<size_t>(count) * es;
  const bool in_place = sendbuf == MPI_IN_PLACE;
  const unsigned char* src = static_cast<const unsigned char*>(in_place ? recvbuf : sendbuf);
  unsigned char* dst = static_cast<unsigned char*>(recvbuf);
  if (comm_size(comm) == 1) {
    if (!in_place) copy_any(dst, src, total);
    return MPI_SUCCESS;
  }
  const size_t chunk = (kReduceBytes / es) * es;
  std::vector<unsigned char> acc(chunk);
  for (size_t off = 0; off < total || (total == 0 && off == 0); off += chunk) {
    const size_t n = total - off < chunk ? total - off : chunk;
    copy_any(s.hdr->reduce_buf[s.rank], src + off, n);
    barrier_world();
    if (all || s.rank == root) {
      memcpy(acc.data(), s.hdr->reduce_buf[0], n);
      for (int r = 1; r < s.world; ++r) reduce_chunk(acc.data(), s.hdr->reduce_buf[r], n / es, t, op);
      copy_any(dst + off, acc.data(), n);
    }
    barrier_world();
    if (total == 0) break;
  }
  return MPI_SUCCESS;
}

}  // namespace

extern "C" {

int MPI_Init_thread(int*, char***, int required, int* provided) {
  State& s = S();
  if (s.initialized) die(MPI_ERR_OTHER, "MPI_Init called twice");
  static const char* rank_vars[] = {"OMPI_COMM_WORLD_RANK", "PMI_RANK", "RANK", nullptr};
  static const char* size_vars[] = {"OMPI_COMM_WORLD_SIZE", "PMI_SIZE", "WORLD_SIZE", nullptr};
  s.rank = env_int(rank_vars, 0);
  s.world = env_int(size_vars, 1);
  if (s.world < 1 || s.world > kMaxRanks || s.rank < 0 || s.rank >= s.world)
    die(MPI_ERR_OTHER, "bad rank %d / size %d from the environment (at most %d ranks)", s.rank,
        s.world, kMaxRanks);
  if (const char* t = getenv("MINIMPI_TIMEOUT_S")) s.timeout_s = atof(t);
  if (s.world > 1) {
    const char* job = getenv("MINIMPI_JOB");
    if (job == nullptr || job[0] == '\0')
      die(MPI_ERR_OTHER, "MINIMPI_JOB must name the job (the same string on every rank)");
    s.job = job;
    const std::string name = "/mmpi_" + s.job;
    if (s.rank == 0) {
      s.hdr = static_cast<Header*>(map_shm(name, sizeof(Header), true));
      s.hdr->world.store(static_cast<uint32_t>(s.world));
      s.hdr->magic.store(kMagic, std::memory_order_release);
    } else {
      Waiter w("rank 0 to create the job's shared memory");
      int fd;
      while ((fd = shm_open(name.c_str(), O_RDWR, 0600)) < 0) w.pause();
      struct stat st;
      while (fstat(fd, &st) == 0 && static_cast<size_t>(st.st_size) < sizeof(Header)) w.pause();
      void* p = mmap(nullptr, sizeof(Header), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
      close(fd);
      if (p == MAP_FAILED) die(MPI_ERR_OTHER, "mmap(%s) failed: %s", name.c_str(), strerror(errno));
      s.hdr = static_cast<Header*>(p);
      while (s.hdr->magic.load(std::memory_order_acquire) != kMagic) w.pause();
      if (s.hdr->world.load() != static_cast<uint32_t>(s.world))
        die(MPI_ERR_OTHER, "job %s was started with %u ranks, this rank expects %d", job,
            s.hdr->world.load(), s.world);
    }
    s.hdr->attached.fetch_add(1);
  }
  s.initialized = true;
  barrier_world();
  if (provided != nullptr) *provided = required < MPI_THREAD_SERIALIZED ? required : MPI_THREAD_SERIALIZED;
  return MPI_SUCCESS;
}

int MPI_Init(int* argc, char*** argv) {
  int provided;
  return MPI_Init_thread(argc, argv, MPI_THREAD_SINGLE, &provided);
}

int MPI_Initialized(int* flag) {
  *flag = S().initialized ? 1 : 0;
  return MPI_SUCCESS;
}

int MPI_Finalized(int* flag) {
  *flag = S().finalized ? 1 : 0;
  return MPI_SUCCESS;
}

int MPI_Finalize(void) {
  require_init("MPI_Finalize");
  State& s = S();
  {
    Waiter w("pending requests at MPI_Finalize");
    bool pending = true;
    while (pending) {
      progress();
      pending = false;
      for (int p = 0; p < s.world; ++p) pending |= !s.sendq[p].empty() || !s.recvq[p].empty();
      if (pending) w.pause();
    }
  }
  barrier_world();
  for (auto& kv : s.imported) cu().ipcCloseMemHandle(kv.second);
  s.imported.clear();
  if (s.stream != nullptr) cu().streamDestroy(s.stream);
  s.stream = nullptr;
  for (int r = 0; r < kMaxRanks; ++r) {
    if (s.chans_out[r] != nullptr) munmap(s.chans_out[r], sizeof(Chan));
    if (s.chans_in[r] != nullptr) munmap(s.chans_in[r], sizeof(Chan));
    s.chans_out[r] = s.chans_in[r] = nullptr;
  }
  for (const auto& n : s.chan_names) shm_unlink(n.c_str());
  barrier_world();  // nobody touches the header after this
  if (s.hdr != nullptr) {
    munmap(s.hdr, sizeof(Header));
    s.hdr = nullptr;
    if (s.rank == 0) shm_unlink(("/mmpi_" + s.job).c_str());
  }
  s.finalized = true;
  return MPI_SUCCESS;
}

int MPI_Abort(MPI_Comm, int errorcode) {
  State& s = S();
  fprintf(stderr, "[minimpi] rank %d: MPI_Abort(%d)\n", s.rank, errorcode);
  fflush(stderr);
  fflush(stdout);
  if (s.hdr != nullptr) {
    int32_t expected = 0;
    if (s.hdr->abort_code.compare_exchange_strong(expected, errorcode + 1))
      s.hdr->abort_rank.store(s.rank);
  }
  unlink_names();
  _exit(errorcode);
}

int MPI_Comm_rank(MPI_Comm comm, int* rank) {
  require_init("MPI_Comm_rank");
  check_comm(comm);
  *rank = comm_rank(comm);
  return MPI_SUCCESS;
}

int MPI_Comm_size(MPI_Comm comm, int* size) {
  require_init("MPI_Comm_size");
  check_comm(comm);
  *size = comm_size(comm);
  return MPI_SUCCESS;
}

int MPI_Comm_split_type(MPI_Comm comm, int split_type, int, MPI_Info, MPI_Comm* newcomm) {
  require_init("MPI_Comm_split_type");
  check_comm(comm);
  if (split_type != MPI_COMM_TYPE_SHARED) {
    *newcomm = MPI_COMM_NULL;
    return MPI_SUCCESS;
  }
  // one node: the shared-memory communicator has the same members and order
  *newcomm = comm == MPI_COMM_SELF ? MPI_COMM_SELF : S().next_comm++;
  return MPI_SUCCESS;
}

int MPI_Comm_free(MPI_Comm* comm) {
  *comm = MPI_COMM_NULL;
  return MPI_SUCCESS;
}

int MPI_Get_processor_name(char* name, int* resultlen) {
  if (gethostname(name, MPI_MAX_PROCESSOR_NAME) != 0) snprintf(name, MPI_MAX_PROCESSOR_NAME, "localhost");
  name[MPI_MAX_PROCESSOR_NAME - 1] = '\0';
  *resultlen = static_cast<int>(strlen(name));
  return MPI_SUCCESS;
}

int MPI_Barrier(MPI_Comm comm) {
  require_init("MPI_Barrier");
  check_comm(comm);
  if (comm_size(comm) > 1) barrier_world();
  return MPI_SUCCESS;
}

int MPI_Bcast(void* buffer, int count, MPI_Datatype t, int root, MPI_Comm comm) {
  require_init("MPI_Bcast");
  check_comm(comm);
  State& s = S();
  if (comm_size(comm) == 1) return MPI_SUCCESS;
  const size_t total = static_cast<size_t>(count) * type_size(t);
  unsigned char* b = static_cast<unsigned char*>(buffer);
  for (size_t off = 0; off < total; off += kBcastBytes) {
    const size_t n = total - off < kBcastBytes ? total - off : kBcastBytes;
    if (s.rank == root) copy_any(s.hdr->bcast_buf, b + off, n);
    barrier_world();
    if (s.rank != root) copy_any(b + off, s.hdr->bcast_buf, n);
    barrier_world();
  }
  return MPI_SUCCESS;
}

int MPI_Reduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype t, MPI_Op op, int root,
               MPI_Comm comm) {
  return reduce_impl(sendbuf, recvbuf, count, t, op, root, comm, false);
}

int MPI_Allreduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype t, MPI_Op op,
                  MPI_Comm comm) {
  return reduce_impl(sendbuf, recvbuf, count, t, op, 0, comm, true);
}

int MPI_Isend(const void* buf, int count, MPI_Datatype t, int dest, int tag, MPI_Comm comm,
              MPI_Request* request) {
  require_init("MPI_Isend");
  check_comm(comm);
  State& s = S();
  if (dest == MPI_PROC_NULL) {
    *request = new minimpi_request();
    (*request)->state = 2;
    return MPI_SUCCESS;
  }
  if (comm == MPI_COMM_SELF) dest = s.rank;
  if (dest < 0 || dest >= s.world) die(MPI_ERR_OTHER, "MPI_Isend to invalid rank %d", dest);
  MPI_Request r = new minimpi_request();
  r->send = true;
  r->peer = dest;
  r->tag = tag;
  r->sbuf = static_cast<const unsigned char*>(buf);
  r->bytes = static_cast<size_t>(count) * type_size(t);
  r->device = is_device_ptr(buf);
  s.sendq[dest].push_back(r);
  *request = r;
  progress();
  return MPI_SUCCESS;
}

int MPI_Irecv(void* buf, int count, MPI_Datatype t, int source, int tag, MPI_Comm comm,
              MPI_Request* request) {
  require_init("MPI_Irecv");
  check_comm(comm);
  State& s = S();
  if (source == MPI_PROC_NULL) {
    *request = new minimpi_request();
    (*request)->state = 2;
    return MPI_SUCCESS;
  }
  if (comm == MPI_COMM_SELF) source = s.rank;
  if (source == MPI_ANY_SOURCE) die(MPI_ERR_OTHER, "MPI_ANY_SOURCE is not supported");
  if (source < 0 || source >= s.world) die(MPI_ERR_OTHER, "MPI_Irecv from invalid rank %d", source);
  MPI_Request r = new minimpi_request();
  r->peer = source;
  r->tag = tag;
  r->rbuf = static_cast<unsigned char*>(buf);
  r->bytes = static_cast<size_t>(count) * type_size(t);
  r->device = is_device_ptr(buf);
  s.recvq[source].push_back(r);
  *request = r;
  progress();
  return MPI_SUCCESS;
}

int MPI_Test(MPI_Request* request, int* flag, MPI_Status* status) {
  require_init("MPI_Test");
  if (*request == MPI_REQUEST_NULL) {
    *flag = 1;
    return MPI_SUCCESS;
  }
  progress();
  *flag = (*request)->state == 2 ? 1 : 0;
  if (*flag) {
    fill_status(*request, status);
    release(request);
  }
  return MPI_SUCCESS;
}

int MPI_Testall(int count, MPI_Request requests[], int* flag, MPI_Status statuses[]) {
  require_init("MPI_Testall");
  progress();
  bool all = true;
  for (int i = 0; i < count; ++i)
    if (requests[i] != MPI_REQUEST_NULL && requests[i]->state != 2) all = false;
  *flag = all ? 1 : 0;
  if (all) {
    for (int i = 0; i < count; ++i) {
      if (requests[i] == MPI_REQUEST_NULL) continue;
      fill_status(requests[i], statuses == MPI_STATUSES_IGNORE ? MPI_STATUS_IGNORE : &statuses[i]);
      release(&requests[i]);
    }
  }
  return MPI_SUCCESS;
}

int MPI_Wait(MPI_Request* request, MPI_Status* status) {
  require_init("MPI_Wait");
  if (*request == MPI_REQUEST_NULL) return MPI_SUCCESS;
  Waiter w("a point-to-point message");
  while (true) {
    progress();
    if ((*request)->state == 2) break;
    w.pause();
  }
  fill_status(*request, status);
  release(request);
  return MPI_SUCCESS;
}

int MPI_Waitall(int count, MPI_Request requests[], MPI_Status statuses[]) {
  require_init("MPI_Waitall");
  Waiter w("point-to-point messages");
  while (true) {
    progress();
    bool all = true;
    for (int i = 0; i < count; ++i)
      if (requests[i] != MPI_REQUEST_NULL && requests[i]->state != 2) all = false;
    if (all) break;
    w.pause();
  }
  for (int i = 0; i < count; ++i) {
    if (requests[i] == MPI_REQUEST_NULL) continue;
    fill_status(requests[i], statuses == MPI_STATUSES_IGNORE ? MPI_STATUS_IGNORE : &statuses[i]);
    release(&requests[i]);
  }
  return MPI_SUCCESS;
}

int MPI_Send(const void* buf, int count, MPI_Datatype t, int dest, int tag, MPI_Comm comm) {
  MPI_Request r;
  MPI_Isend(buf, count, t, dest, tag, comm, &r);
  return MPI_Wait(&r, MPI_STATUS_IGNORE);
}

int MPI_Recv(void* buf, int count, MPI_Datatype t, int source, int tag, MPI_Comm comm,
             MPI_Status* status) {
  MPI_Request r;
  MPI_Irecv(buf, count, t, source, tag, comm, &r);
  return MPI_Wait(&r, status);
}

int MPI_Sendrecv(const void* sendbuf, int sendcount, MPI_Datatype sendtype, int dest, int sendtag,
                 void* recvbuf, int recvcount, MPI_Datatype recvtype, int source, int recvtag,
                 MPI_Comm comm, MPI_Status* status) {
  // both directions progress together, so a ring of Sendrecv cannot deadlock
  MPI_Request r[2];
  MPI_Irecv(recvbuf, recvcount, recvtype, source, recvtag, comm, &r[0]);
  MPI_Isend(sendbuf, sendcount, sendtype, dest, sendtag, comm, &r[1]);
  MPI_Status st[2];
  MPI_Waitall(2, r, st);
  if (status != MPI_STATUS_IGNORE) *status = st[0];
  return MPI_SUCCESS;
}

int MPI_Get_count(const MPI_Status* status, MPI_Datatype t, int* count) {
  *count = static_cast<int>(static_cast<size_t>(status->minimpi_count_bytes) / type_size(t));
  return MPI_SUCCESS;
}

double MPI_Wtime(void) { return now_s(); }

}  // extern "C"
