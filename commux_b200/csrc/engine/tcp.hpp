#pragma once

// TCP links to peers on other hosts (or to every peer with
// COMMUX_TRANSPORT=tcp).
//
// The engine speaks to every peer through byte rings of self-describing
// records (shm.hpp). For a peer reached over TCP, the rings are proxied: the
// engine writes its records into a private out-ring that a pump thread drains
// into the socket, and the pump parses the bytes arriving from the socket
// back into whole records that it publishes into this rank's own in-ring for
// that peer (the ring a same-host peer would write directly). Matching,
// rendezvous and completion logic is therefore identical for both transports;
// only the bytes travel differently. This stands in for UCX's tcp transport
// of the reference (reference: src/process_group_ucx.cpp:393-472, where UCX
// picks tcp/ib for off-node endpoints).
//
// Wake-ups: the engine signals new out-ring data through an eventfd; the pump
// rings this rank's doorbell after publishing into an in-ring. A closed or
// failed socket reports the peer dead through a callback.

#include <c10/util/intrusive_ptr.h>
#include <torch/csrc/distributed/c10d/Store.hpp>

#include <atomic>
#include <chrono>
#include <functional>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "shm.hpp"

namespace commux {
namespace tcp {

class Links {
 public:
  // `remote[p]`: peer p is reached over TCP. `own` is this rank's segment
  // (its ring[p] is the in-ring of peer p).
  Links(int rank, int size, std::uint64_t ring_bytes, std::vector<bool> remote, shm::Segment* own);
  ~Links();
  Links(const Links&) = delete;
  Links& operator=(const Links&) = delete;

  // Collective over the group: listen, publish the address under
  // `pfx` + "tcp/<rank>", connect to lower ranks, accept higher ranks.
  void connect(c10d::Store& store, const std::string& pfx, std::chrono::milliseconds timeout);

  // Out-ring of peer p (the engine attaches its RingWriter here).
  shm::RingCtl* out_ctl(int p) const;
  char* out_data(int p) const;

  // Start the pump thread. `wake` rings this rank's doorbell; `dead(p, why)`
  // reports a lost peer; `sent(id)` reports that the last indirect record of
  // request `id` has left (its payload memory is no longer read).
  void start(std::function<void()> wake, std::function<void(int, const std::string&)> dead,
             std::function<void(std::uint64_t)> sent);
  void notify();  // new bytes in some out-ring
  void stop();

  bool remote(int p) const { return remote_[p]; }
  std::int64_t bytes_sent() const { return sent_.load(); }
  std::int64_t bytes_received() const { return received_.load(); }

 private:
  struct Peer;
  void pump();
  bool pump_peer(Peer& p, bool* want_out, bool* blocked_in);

  int rank_, size_;
  std::uint64_t ring_bytes_;
  std::vector<bool> remote_;
  shm::Segment* own_;
  std::vector<std::unique_ptr<Peer>> peers_;
  int listen_fd_ = -1;
  int event_fd_ = -1;
  std::thread thread_;
  std::atomic<bool> stop_{false};
  std::function<void()> wake_;
  std::function<void(int, const std::string&)> dead_;
  std::function<void(std::uint64_t)> sent_cb_;
  std::atomic<std::int64_t> sent_{0}, received_{0};
};

// Transport choice for peer p from COMMUX_TRANSPORT (auto|shm|tcp): auto uses
// shared memory on this host and TCP across hosts.
bool use_tcp(const std::string& my_host, const std::string& peer_host);

}  // namespace tcp
}  // namespace commux
