#include "shm.hpp"

#include <fcntl.h>
#include <linux/futex.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <time.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>

namespace commux {
namespace shm {

int futex_wait(std::atomic<std::uint32_t>* addr, std::uint32_t expected,
               long timeout_us) {
  struct timespec ts;
  struct timespec* tsp = nullptr;
  if (timeout_us >= 0) {
    ts.tv_sec = timeout_us / 1000000;
    ts.tv_nsec = (timeout_us % 1000000) * 1000;
    tsp = &ts;
  }
  // Not FUTEX_PRIVATE: the word lives in a mapping shared between processes.
  return static_cast<int>(syscall(SYS_futex, reinterpret_cast<std::uint32_t*>(addr),
                                  FUTEX_WAIT, expected, tsp, nullptr, 0));
}

void futex_wake(std::atomic<std::uint32_t>* addr, int count) {
  syscall(SYS_futex, reinterpret_cast<std::uint32_t*>(addr), FUTEX_WAKE, count,
          nullptr, nullptr, 0);
}

namespace {
constexpr std::size_t kHeaderBytes = 4096;
std::size_t ring_stride(std::uint64_t ring_bytes) {
  return sizeof(RingCtl) + static_cast<std::size_t>(ring_bytes);
}
}  // namespace

std::size_t Segment::bytes_for(int nranks, std::uint64_t ring_bytes) {
  return kHeaderBytes + static_cast<std::size_t>(nranks) * ring_stride(ring_bytes);
}

Segment::~Segment() {
  unlink();
  unmap();
}

void Segment::create(const std::string& name, int nranks, int rank,
                     std::uint64_t ring_bytes, std::uint64_t instance) {
  static_assert(sizeof(SegHeader) <= kHeaderBytes, "header fits its page");
  if (ring_bytes % 64 != 0 || ring_bytes < 4096)
    throw std::invalid_argument("commux shm: ring size must be >=4096 and a multiple of 64");
  name_ = name;
  size_ = bytes_for(nranks, ring_bytes);
  int fd = ::shm_open(name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (fd < 0)
    throw std::runtime_error("commux shm: shm_open(" + name + ") failed: " +
                             std::strerror(errno));
  if (::ftruncate(fd, static_cast<off_t>(size_)) != 0) {
    int e = errno;
    ::close(fd);
    ::shm_unlink(name.c_str());
    throw std::runtime_error("commux shm: ftruncate(" + std::to_string(size_) +
                             ") failed: " + std::strerror(e) +
                             " (is /dev/shm large enough? set COMMUX_SHM_RING_BYTES)");
  }
  base_ = ::mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  ::close(fd);
  if (base_ == MAP_FAILED) {
    base_ = nullptr;
    ::shm_unlink(name.c_str());
    throw std::runtime_error("commux shm: mmap failed: " + std::string(std::strerror(errno)));
  }
  owner_ = true;
  // Touch the pages now (ftruncate gives a sparse object; a later SIGBUS on a
  // full /dev/shm is far harder to diagnose than a failure here).
  std::memset(base_, 0, size_);
  hdr_ = static_cast<SegHeader*>(base_);
  new (hdr_) SegHeader();
  hdr_->version = kSegVersion;
  hdr_->nranks = static_cast<std::uint32_t>(nranks);
  hdr_->rank = static_cast<std::uint32_t>(rank);
  hdr_->pid = static_cast<std::int32_t>(::getpid());
  hdr_->ring_bytes = ring_bytes;
  hdr_->instance = instance;
  ::gethostname(hdr_->hostname, sizeof(hdr_->hostname) - 1);
  hdr_->doorbell.store(0);
  hdr_->sleeping.store(0);
  hdr_->abort_code.store(0);
  hdr_->abort_rank.store(-1);
  hdr_->heartbeat.store(0);
  hdr_->closed.store(0);
  hdr_->cuda_uuid_valid.store(0);
  for (int p = 0; p < nranks; ++p) {
    RingCtl* c = ring_ctl(p);
    new (c) RingCtl();
    c->tail.store(0);
    c->head.store(0);
  }
  std::atomic_thread_fence(std::memory_order_seq_cst);
  reinterpret_cast<std::atomic<std::uint64_t>*>(&hdr_->magic)
      ->store(kSegMagic, std::memory_order_release);
}

void Segment::open(const std::string& name) {
  name_ = name;
  int fd = ::shm_open(name.c_str(), O_RDWR, 0600);
  if (fd < 0)
    throw std::runtime_error("commux shm: cannot open peer segment " + name +
                             ": " + std::strerror(errno) +
                             " (peers must share a host and /dev/shm)");
  struct stat st;
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    throw std::runtime_error("commux shm: fstat failed");
  }
  size_ = static_cast<std::size_t>(st.st_size);
  base_ = ::mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  ::close(fd);
  if (base_ == MAP_FAILED) {
    base_ = nullptr;
    throw std::runtime_error("commux shm: mmap of peer segment failed");
  }
  owner_ = false;
  hdr_ = static_cast<SegHeader*>(base_);
  auto magic = reinterpret_cast<std::atomic<std::uint64_t>*>(&hdr_->magic)
                   ->load(std::memory_order_acquire);
  if (magic != kSegMagic || hdr_->version != kSegVersion ||
      size_ < bytes_for(static_cast<int>(hdr_->nranks), hdr_->ring_bytes))
    throw std::runtime_error("commux shm: peer segment " + name +
                             " is not a compatible commux segment");
}

void Segment::unlink() {
  if (owner_ && !unlinked_ && !name_.empty()) {
    ::shm_unlink(name_.c_str());
    unlinked_ = true;
  }
}

void Segment::unmap() {
  if (base_ != nullptr) {
    ::munmap(base_, size_);
    base_ = nullptr;
    hdr_ = nullptr;
  }
}

RingCtl* Segment::ring_ctl(int producer) const {
  char* p = static_cast<char*>(base_) + kHeaderBytes +
            static_cast<std::size_t>(producer) * ring_stride(hdr_->ring_bytes);
  return reinterpret_cast<RingCtl*>(p);
}

char* Segment::ring_data(int producer) const {
  return reinterpret_cast<char*>(ring_ctl(producer)) + sizeof(RingCtl);
}

// ---------------------------------------------------------------------------

std::uint64_t RingWriter::free_bytes() {
  head_cache_ = ctl_->head.load(std::memory_order_acquire);
  return cap_ - (tail_ - head_cache_);
}

char* RingWriter::reserve(std::uint64_t n) {
  std::uint64_t pos = tail_ % cap_;
  std::uint64_t contiguous = cap_ - pos;
  std::uint64_t need = n <= contiguous ? n : contiguous + n;
  if (cap_ - (tail_ - head_cache_) < need) {
    head_cache_ = ctl_->head.load(std::memory_order_acquire);
    if (cap_ - (tail_ - head_cache_) < need) return nullptr;
  }
  if (n > contiguous) {
    // Pad to the end of the ring; the record starts at offset 0.
    auto* pad = reinterpret_cast<WireHdr*>(data_ + pos);
    pad->len = static_cast<std::uint32_t>(contiguous);
    pad->type = kRecPad;
    pad->flags = 0;
    tail_ += contiguous;
    pos = 0;
  }
  char* p = data_ + pos;
  tail_ += n;
  return p;
}

const WireHdr* RingReader::peek() {
  for (;;) {
    if (head_ == tail_cache_) {
      tail_cache_ = ctl_->tail.load(std::memory_order_acquire);
      if (head_ == tail_cache_) {
        if (pending_release_) release();
        return nullptr;
      }
    }
    auto* h = reinterpret_cast<const WireHdr*>(data_ + head_ % cap_);
    if (h->type == kRecPad) {
      head_ += h->len;
      continue;
    }
    return h;
  }
}

}  // namespace shm
}  // namespace commux
