// IOContext: collective file primitives over a private commux group
// (behaviour of reference: src/io.cpp:43-192). Error agreement is one
// allreduce-MAX of the local errno, so every rank raises, all with the same
// errno (the largest of those that failed); sizes and payloads travel on the collective tag namespace.

#include "commux/io.hpp"

#include <ATen/ATen.h>
#include <fcntl.h>
#include <sys/types.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>
#include <string>
#include <torch/csrc/distributed/c10d/TCPStore.hpp>

#include "commux/process_group_ucx.hpp"

namespace commux {

namespace {

constexpr int kSizeTag = 0x10;
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

void IOContext::write_at(int fd, const void* data, std::size_t nbytes, std::int64_t offset) {
  if (offset < 0) throw std::invalid_argument("commux::IOContext write_at: negative offset");
  const char* p = static_cast<const char*>(data);
  std::size_t done = 0;
  while (done < nbytes) {
    ssize_t n = ::pwrite(fd, p + done, nbytes - done, static_cast<off_t>(offset + static_cast<std::int64_t>(done)));
    if (n < 0) {
      if (errno == EINTR) continue;
      throw std::runtime_error(std::string("commux::IOContext write_at failed: ") + std::strerror(errno));
    }
    if (n == 0) throw std::runtime_error("commux::IOContext write_at made no progress");
    done += static_cast<std::size_t>(n);
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

std::vector<std::uint8_t> IOContext::gather_bytes(const std::vector<std::uint8_t>& bytes, int root) {
  if (root < 0 || root >= size_) throw std::invalid_argument("commux::IOContext gather: root out of range");
  std::vector<std::uint8_t> out;
  if (rank_ == root) {
    std::vector<std::vector<std::uint8_t>> parts(size_);
    parts[root] = bytes;
    for (int r = 0; r < size_; ++r) {
      if (r == root) continue;
      std::int64_t n = 0;
      recv_bytes(&n, sizeof(n), r, kSizeTag);
      if (n < 0) throw std::runtime_error("commux::IOContext gather: negative size");
      parts[r].resize(static_cast<std::size_t>(n));
      recv_bytes(parts[r].data(), parts[r].size(), r, kDataTag);
    }
    std::size_t total = 0;
    for (auto& p : parts) total += p.size();
    out.reserve(total);
    for (auto& p : parts) out.insert(out.end(), p.begin(), p.end());
  } else {
    std::int64_t n = static_cast<std::int64_t>(bytes.size());
    send_bytes(&n, sizeof(n), root, kSizeTag);
    send_bytes(bytes.data(), bytes.size(), root, kDataTag);
  }
  barrier();
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
