#pragma once

// Rank-collective POSIX file I/O helper over a private commux process group
// (API of reference: include/commux/io.hpp:15-41). A consumer builds
// checkpoints from it: every rank opens/syncs/closes together and an error on
// any rank raises on all of them; payload metadata travels with
// broadcast_bytes / gather_bytes.

#include <c10/util/intrusive_ptr.h>

#include <cstdint>
#include <memory>
#include <string>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <vector>

namespace commux {

class ProcessGroupUCX;

class IOContext {
 public:
  IOContext(c10::intrusive_ptr<c10d::Store> store, int rank, int size);
  ~IOContext();

  int rank() const { return rank_; }
  int size() const { return size_; }

  void barrier();
  // Root's bytes replace every other rank's `bytes`.
  void broadcast_bytes(std::vector<std::uint8_t>& bytes, int root);
  // Root gets every rank's bytes concatenated in rank order; others get {}.
  std::vector<std::uint8_t> gather_bytes(const std::vector<std::uint8_t>& bytes,
                                         int root);
  void send_bytes(const void* data, std::size_t nbytes, int dst, int tag);
  void recv_bytes(void* data, std::size_t nbytes, int src, int tag);
  // Collective: throws on every rank if any rank failed.
  int open_file(const std::string& path, int flags, int mode);
  void close_file(int fd);
  // Local positional write (loops until all bytes are written).
  void write_at(int fd, const void* data, std::size_t nbytes,
                std::int64_t offset);
  void sync_file(int fd);

  ProcessGroupUCX& process_group() { return *pg_; }

 private:
  void agree(int local_errno, const char* what);

  int rank_;
  int size_;
  c10::intrusive_ptr<ProcessGroupUCX> pg_;
};

// IOContext over a fresh TCPStore (rank 0 hosts it).
std::shared_ptr<IOContext> make_tcp_io_context(const std::string& host,
                                               int port, int rank, int size);

}  // namespace commux
