#pragma once

// POSIX shared-memory transport between the ranks of one host.
//
// Each rank creates one segment holding a header (doorbell futex word, abort
// word, heartbeat, pid) and one single-producer/single-consumer byte ring per
// peer: ring[p] of rank r carries the records that rank p sends to rank r
// (p == r is the loopback ring for self-sends). Every peer maps every other
// rank's segment, so a producer writes straight into the consumer's ring and
// the consumer's progress thread drains its own rings.
//
// This replaces the UCX `sm`/`tcp` host transports of the reference
// (reference: src/process_group_ucx.cpp:393-472 bootstraps UCX endpoints; here
// the c10d::Store carries segment names instead of UCX worker addresses).

#include <sys/types.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>

namespace commux {
namespace shm {

constexpr std::uint64_t kSegMagic = 0x31584d4d4f434d53ull;  // "SMCOMMX1"
constexpr std::uint32_t kSegVersion = 4;

// Record header; `len` covers header + payload and is a multiple of 8.
struct WireHdr {
  std::uint32_t len;
  std::uint16_t type;
  std::uint16_t flags;
};
static_assert(sizeof(WireHdr) == 8, "wire header is 8 bytes");
constexpr std::uint16_t kRecPad = 0;  // skip to the end of the ring

struct alignas(64) RingCtl {
  std::atomic<std::uint64_t> tail;  // bytes published by the producer
  char pad0[56];
  std::atomic<std::uint64_t> head;  // bytes released by the consumer
  char pad1[56];
};
static_assert(sizeof(RingCtl) == 128, "ring control is two cache lines");

struct alignas(64) SegHeader {
  std::uint64_t magic;
  std::uint32_t version;
  std::uint32_t nranks;
  std::uint32_t rank;
  std::int32_t pid;
  std::uint64_t ring_bytes;
  std::uint64_t instance;  // process-group instance id (shared by all ranks)
  char hostname[64];
  alignas(64) std::atomic<std::uint32_t> doorbell;  // futex word
  alignas(64) std::atomic<std::uint32_t> sleeping;  // consumer parked
  alignas(64) std::atomic<std::uint32_t> abort_code;  // nonzero: abort group
  std::atomic<std::int32_t> abort_rank;
  alignas(64) std::atomic<std::uint64_t> heartbeat;  // bumped by progress
  alignas(64) std::atomic<std::uint32_t> closed;     // rank shut down cleanly
  // CUDA device this rank drives p2p from (published on first CUDA use), so
  // a sender knows whether its peer shares its GPU.
  alignas(64) std::atomic<std::uint32_t> cuda_uuid_valid;
  unsigned char cuda_uuid[16];
};

inline std::uint64_t align8(std::uint64_t n) { return (n + 7) & ~7ull; }

// futex on a shared (non-private) mapping; timeout in microseconds (<0: none)
int futex_wait(std::atomic<std::uint32_t>* addr, std::uint32_t expected,
               long timeout_us);
void futex_wake(std::atomic<std::uint32_t>* addr, int count);

class Segment {
 public:
  Segment() = default;
  ~Segment();
  Segment(const Segment&) = delete;
  Segment& operator=(const Segment&) = delete;

  static std::size_t bytes_for(int nranks, std::uint64_t ring_bytes);
  // Create and initialise this rank's segment.
  void create(const std::string& name, int nranks, int rank,
              std::uint64_t ring_bytes, std::uint64_t instance);
  // Map a peer's segment (validates magic/version/size).
  void open(const std::string& name);
  void unlink();  // remove the name (mapping stays valid)
  void unmap();

  SegHeader* header() const { return hdr_; }
  RingCtl* ring_ctl(int producer) const;
  char* ring_data(int producer) const;
  std::uint64_t ring_bytes() const { return hdr_->ring_bytes; }
  const std::string& name() const { return name_; }
  bool mapped() const { return base_ != nullptr; }

 private:
  std::string name_;
  void* base_ = nullptr;
  std::size_t size_ = 0;
  SegHeader* hdr_ = nullptr;
  bool owner_ = false;
  bool unlinked_ = false;
};

// Producer side of one ring (lives in the consumer's segment). Not
// thread-safe: callers serialise with a per-ring lock.
class RingWriter {
 public:
  void attach(RingCtl* ctl, char* data, std::uint64_t cap) {
    ctl_ = ctl;
    data_ = data;
    cap_ = cap;
    tail_ = ctl->tail.load(std::memory_order_relaxed);
    head_cache_ = ctl->head.load(std::memory_order_acquire);
  }
  // Largest record that always fits (so one record can never wedge a ring).
  std::uint64_t max_record() const { return cap_ / 2; }
  // Reserve `n` contiguous bytes (n multiple of 8, n <= max_record()).
  // Returns nullptr if the ring lacks space right now.
  char* reserve(std::uint64_t n);
  // Publish everything reserved since the last publish.
  void publish() { ctl_->tail.store(tail_, std::memory_order_release); }
  std::uint64_t free_bytes();

 private:
  RingCtl* ctl_ = nullptr;
  char* data_ = nullptr;
  std::uint64_t cap_ = 0;
  std::uint64_t tail_ = 0;
  std::uint64_t head_cache_ = 0;
};

// Consumer side of one ring. Used only by the progress thread.
class RingReader {
 public:
  void attach(RingCtl* ctl, char* data, std::uint64_t cap) {
    ctl_ = ctl;
    data_ = data;
    cap_ = cap;
    head_ = ctl->head.load(std::memory_order_relaxed);
    tail_cache_ = head_;
  }
  // Next record, or nullptr if the ring is empty. Skips pad records.
  const WireHdr* peek();
  // Consume the record returned by peek().
  void pop(const WireHdr* h) {
    head_ += h->len;
    ++pending_release_;
    if (pending_release_ >= 8) release();
  }
  void release() {
    ctl_->head.store(head_, std::memory_order_release);
    pending_release_ = 0;
  }
  bool empty_hint() const { return head_ == tail_cache_; }

 private:
  RingCtl* ctl_ = nullptr;
  char* data_ = nullptr;
  std::uint64_t cap_ = 0;
  std::uint64_t head_ = 0;
  std::uint64_t tail_cache_ = 0;
  int pending_release_ = 0;
};

}  // namespace shm
}  // namespace commux
