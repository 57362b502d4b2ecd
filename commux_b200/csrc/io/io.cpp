// IOContext: collective file primitives over a private commux group
// (behaviour of reference: src/io.cpp:43-192). Error agreement is one
// allreduce-MAX of the local errno, so every rank raises, all with the same
// errno (the largest of those that failed). Sizes travel in collectives
// (broadcast, allgather); gathered payloads are sends with tag kDataTag on
// the context's private group (send_bytes/recv_bytes callers should keep
// that tag free while a gather runs).

#include "commux/io.hpp"

#include <ATen/ATen.h>
#include <fcntl.h>
#include <sys/types.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <stdexcept>
#include <string>
#include <torch/csrc/distributed/c10d/TCPStore.hpp>

#include "commux/process_group_ucx.hpp"

namespace commux {

namespace {

constexpr int kDataTag = 0x11;

at::Tensor bytes_view(void* data, std::size_t n) {
  return at::from_blob(data, {static_cast<std::int64_t>(n)}, at::TensorOptions().dtype(at::kByte));
}

}  // namespace

IOContext::IOContext(c10::intrusive_ptr<c10d::Store> store, int rank, int size)
    : rank_(rank),
      size_(size),
      pg_(c10::make_intrusive<ProcessGroupUCX>(std::move(store), rank, size)) {}

IOContext::~IOContext() = default;

void IOContext::barrier() { pg_->barrier()->wait(); }

void IOContext::send_bytes(const void* data, std::size_t nbytes, int dst, int tag) {
  // copy: the caller's buffer may be reused as soon as this returns
  at::Tensor t = at::empty({static_cast<std::int64_t>(nbytes)}, at::TensorOptions().dtype(at::kByte));
  if (nbytes) std::memcpy(t.data_ptr(), data, nbytes);
  std::vector<at::Tensor> v{t};
  pg_->send(v, dst, tag)->wait();
}

void IOContext::recv_bytes(void* data, std::size_t nbytes, int src, int tag) {
  std::vector<at::Tensor> v{bytes_view(data, nbytes)};
  pg_->recv(v, src, tag)->wait();
}

void IOContext::agree(int local_errno, const char* what) {
  at::Tensor st = at::full({1}, static_cast<std::int64_t>(local_errno), at::TensorOptions().dtype(at::kLong));
  std::vector<at::Tensor> v{st};
  c10d::AllreduceOptions o;
  o.reduceOp = c10d::ReduceOp::MAX;
  pg_->allreduce(v, o)->wait();
  std::int64_t e = st.item<std::int64_t>();
  if (e != 0)
    throw std::runtime_error(std::string("commux::IOContext ") + what + " failed on some rank: " +
                             std::strerror(static_cast<int>(e)));
}

int IOContext::open_file(const std::string& path, int flags, int mode) {
  int fd = ::open(path.c_str(), flags, static_cast<mode_t>(mode));
  int err = fd >= 0 ? 0 : errno;
  try {
    agree(err, "open_file");
  } catch (...) {
    if (fd >= 0) ::close(fd);
    throw;
  }
  return fd;
}

void IOContext::close_file(int fd) {
  int err = ::close(fd) == 0 ? 0 : errno;
  agree(err, "close_file");
}

// Positional write of the whole buffer, local to this rank. Linux moves at
// most 0x7ffff000 bytes per write call, so the buffer goes out in pieces of
// at most kWritePiece bytes; a piece that was cut short resumes where the
// kernel stopped. A failure reports how far the write got, so a caller can
// tell a full disk (partial progress) from a bad descriptor (none).
void IOContext::write_at(int fd, const void* data, std::size_t nbytes, std::int64_t offset) {
  constexpr std::size_t kWritePiece = std::size_t(1) << 30;
  if (offset < 0)
    throw std::invalid_argument("commux::IOContext::write_at: offset " + std::to_string(offset) +
                                " is negative");
  const auto* base = static_cast<const unsigned char*>(data);
  std::size_t written = 0;
  int stalls = 0;  // consecutive zero-byte writes
  while (written < nbytes) {
    const std::size_t piece = std::min(nbytes - written, kWritePiece);
    const off_t at = static_cast<off_t>(offset) + static_cast<off_t>(written);
    const ssize_t got = ::pwrite(fd, base + written, piece, at);
    if (got > 0) {
      written += static_cast<std::size_t>(got);
      stalls = 0;
      continue;
    }
    const int err = got < 0 ? errno : 0;
    if (err == EINTR || err == EAGAIN) continue;
    if (got == 0 && ++stalls < 3) continue;
    throw std::runtime_error("commux::IOContext::write_at(fd " + std::to_string(fd) + ", offset " +
                             std::to_string(offset) + "): " + std::to_string(written) + " of " +
                             std::to_string(nbytes) + " bytes written; " +
                             (err != 0 ? std::strerror(err) : "the file accepts no more bytes"));
  }
}

void IOContext::sync_file(int fd) {
  int err = ::fsync(fd) == 0 ? 0 : errno;
  agree(err, "sync_file");
}

void IOContext::broadcast_bytes(std::vector<std::uint8_t>& bytes, int root) {
  if (root < 0 || root >= size_) throw std::invalid_argument("commux::IOContext broadcast: root out of range");
  std::int64_t n = static_cast<std::int64_t>(bytes.size());
  at::Tensor sz = at::full({1}, n, at::TensorOptions().dtype(at::kLong));
  c10d::BroadcastOptions o;
  o.rootRank = root;
  std::vector<at::Tensor> v{sz};
  pg_->broadcast(v, o)->wait();
  n = sz.item<std::int64_t>();
  if (n < 0) throw std::runtime_error("commux::IOContext broadcast: negative size");
  if (rank_ != root) bytes.resize(static_cast<std::size_t>(n));
  if (n > 0) {
    std::vector<at::Tensor> d{bytes_view(bytes.data(), bytes.size())};
    pg_->broadcast(d, o)->wait();
  }
}

// Every rank learns every payload size from one allgather; the root then
// sizes the result once and receives each peer's payload straight into its
// place (offset = sum of the sizes of the lower ranks), all receives in
// flight together. No size messages, no per-peer temporaries, no padding.
std::vector<std::uint8_t> IOContext::gather_bytes(const std::vector<std::uint8_t>& bytes, int root) {
  if (root < 0 || root >= size_) throw std::invalid_argument("commux::IOContext gather: root out of range");
  at::Tensor mine = at::full({1}, static_cast<std::int64_t>(bytes.size()), at::TensorOptions().dtype(at::kLong));
  at::Tensor all = at::empty({size_}, at::TensorOptions().dtype(at::kLong));
  pg_->_allgather_base(all, mine)->wait();
  const std::int64_t* sizes = all.data_ptr<std::int64_t>();
  std::vector<std::size_t> offset(static_cast<std::size_t>(size_) + 1, 0);
  for (int r = 0; r < size_; ++r) {
    if (sizes[r] < 0) throw std::runtime_error("commux::IOContext gather: rank " + std::to_string(r) +
                                               " reported a negative size");
    offset[r + 1] = offset[r] + static_cast<std::size_t>(sizes[r]);
  }
  std::vector<std::uint8_t> out;
  if (rank_ == root) {
    out.resize(offset[size_]);
    if (!bytes.empty()) std::memcpy(out.data() + offset[root], bytes.data(), bytes.size());
    std::vector<c10::intrusive_ptr<c10d::Work>> pending;
    for (int r = 0; r < size_; ++r) {
      if (r == root || sizes[r] == 0) continue;
      std::vector<at::Tensor> v{bytes_view(out.data() + offset[r], static_cast<std::size_t>(sizes[r]))};
      pending.push_back(pg_->recv(v, r, kDataTag));
    }
    for (auto& w : pending) w->wait();
  } else if (!bytes.empty()) {
    // the send completes once the root holds the bytes, so `bytes` is
    // borrowed in place, not copied
    std::vector<at::Tensor> v{bytes_view(const_cast<std::uint8_t*>(bytes.data()), bytes.size())};
    pg_->send(v, root, kDataTag)->wait();
  }
  return out;
}

std::shared_ptr<IOContext> make_tcp_io_context(const std::string& host, int port, int rank, int size) {
  c10d::TCPStoreOptions opts;
  opts.port = static_cast<std::uint16_t>(port);
  opts.isServer = rank == 0;
  opts.numWorkers = size;
  opts.waitWorkers = true;
  auto store = c10::make_intrusive<c10d::TCPStore>(host, opts);
  return std::make_shared<IOContext>(store, rank, size);
}

}  // namespace commux
