#include "tcp.hpp"

#include "protocol.hpp"

#include <arpa/inet.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/eventfd.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

namespace commux {
namespace tcp {

namespace {

constexpr std::uint32_t kHelloMagic = 0x434d5854u;  // "TXMC"

struct Hello {
  std::uint32_t magic;
  std::uint32_t rank;
};

std::string env_str(const char* name) {
  const char* v = std::getenv(name);
  return v ? std::string(v) : std::string();
}

[[noreturn]] void sys_fail(const std::string& what) {
  throw std::runtime_error("commux tcp: " + what + ": " + std::strerror(errno));
}

void set_nonblocking(int fd) {
  int fl = ::fcntl(fd, F_GETFL, 0);
  ::fcntl(fd, F_SETFL, fl | O_NONBLOCK);
}

void tune(int fd) {
  int one = 1;
  ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  int buf = 4 << 20;
  ::setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &buf, sizeof(buf));
  ::setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &buf, sizeof(buf));
}

// Blocking I/O of exactly n bytes with a deadline (handshake only).
bool io_all(int fd, void* buf, std::size_t n, bool send, std::chrono::steady_clock::time_point deadline) {
  char* p = static_cast<char*>(buf);
  while (n > 0) {
    auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - std::chrono::steady_clock::now());
    if (left.count() <= 0) return false;
    pollfd pf{fd, static_cast<short>(send ? POLLOUT : POLLIN), 0};
    int r = ::poll(&pf, 1, static_cast<int>(std::min<long long>(left.count(), 1000)));
    if (r < 0 && errno != EINTR) return false;
    if (r <= 0) continue;
    ssize_t k = send ? ::send(fd, p, n, MSG_NOSIGNAL) : ::recv(fd, p, n, 0);
    if (k == 0) return false;
    if (k < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      return false;
    }
    p += k;
    n -= static_cast<std::size_t>(k);
  }
  return true;
}

bool resolve_v4(const std::string& host, sockaddr_in* out) {
  addrinfo hints{};
  hints.ai_family = AF_INET;
  hints.ai_socktype = SOCK_STREAM;
  addrinfo* res = nullptr;
  if (::getaddrinfo(host.c_str(), nullptr, &hints, &res) != 0 || res == nullptr) return false;
  *out = *reinterpret_cast<sockaddr_in*>(res->ai_addr);
  ::freeaddrinfo(res);
  return true;
}

// The address peers should dial: COMMUX_TCP_ADDR, else the local address of
// the route to MASTER_ADDR (a UDP connect sends nothing), else the first
// address of this host's name, else loopback.
std::string local_addr(bool loopback_ok) {
  std::string forced = env_str("COMMUX_TCP_ADDR");
  if (!forced.empty()) return forced;
  if (loopback_ok) return "127.0.0.1";
  std::string master = env_str("MASTER_ADDR");
  sockaddr_in dst{};
  if (!master.empty() && resolve_v4(master, &dst)) {
    dst.sin_port = htons(9);
    int s = ::socket(AF_INET, SOCK_DGRAM, 0);
    if (s >= 0) {
      sockaddr_in me{};
      socklen_t len = sizeof(me);
      if (::connect(s, reinterpret_cast<sockaddr*>(&dst), sizeof(dst)) == 0 &&
          ::getsockname(s, reinterpret_cast<sockaddr*>(&me), &len) == 0 && me.sin_addr.s_addr != 0) {
        ::close(s);
        char buf[INET_ADDRSTRLEN];
        return ::inet_ntop(AF_INET, &me.sin_addr, buf, sizeof(buf)) ? std::string(buf) : "127.0.0.1";
      }
      ::close(s);
    }
  }
  char host[256] = {0};
  ::gethostname(host, sizeof(host) - 1);
  sockaddr_in a{};
  if (resolve_v4(host, &a)) {
    char buf[INET_ADDRSTRLEN];
    if (::inet_ntop(AF_INET, &a.sin_addr, buf, sizeof(buf))) return buf;
  }
  return "127.0.0.1";
}

struct AlignedFree {
  void operator()(char* p) const { std::free(p); }
};

}  // namespace

bool use_tcp(const std::string& my_host, const std::string& peer_host) {
  static const std::string mode = env_str("COMMUX_TRANSPORT");
  if (mode == "tcp") return true;
  if (my_host == peer_host) return false;
  if (mode == "shm")
    throw std::runtime_error("commux: COMMUX_TRANSPORT=shm but a peer runs on host '" + peer_host +
                             "' and this rank on '" + my_host + "'");
  return true;
}

struct Links::Peer {
  int p = -1;
  int fd = -1;
  bool dead = false;
  bool eof = false;  // the peer closed; reported once its last records were consumed
  std::unique_ptr<char, AlignedFree> mem;  // RingCtl + data of the out-ring
  shm::RingCtl* ctl = nullptr;
  char* data = nullptr;
  shm::RingReader out;
  shm::RingWriter in;
  const shm::WireHdr* cur = nullptr;  // record being sent
  const char* sptr = nullptr;
  std::uint64_t sleft = 0;
  const proto::IndirectRec* ind = nullptr;  // cur, when it is an indirect record
  std::uint64_t ioff = 0;                   // wire bytes of it already sent
  std::vector<char> rbuf;  // bytes received, not yet published
  std::size_t rlen = 0;
  // a large record received straight into its reserved in-ring slot
  char* direct = nullptr;
  std::uint64_t dlen = 0, dgot = 0;
};

namespace {
// Records at least this long that arrive in pieces are received straight
// into the in-ring rather than through rbuf (one copy fewer per byte).
constexpr std::uint64_t kDirectRecvBytes = 64 << 10;
}  // namespace

Links::Links(int rank, int size, std::uint64_t ring_bytes, std::vector<bool> remote, shm::Segment* own)
    : rank_(rank), size_(size), ring_bytes_(ring_bytes), remote_(std::move(remote)), own_(own) {
  peers_.resize(static_cast<std::size_t>(size));
  for (int p = 0; p < size; ++p) {
    if (!remote_[p]) continue;
    auto pe = std::make_unique<Peer>();
    pe->p = p;
    char* m = static_cast<char*>(std::aligned_alloc(64, sizeof(shm::RingCtl) + ring_bytes));
    if (m == nullptr) throw std::bad_alloc();
    pe->mem.reset(m);
    pe->ctl = new (m) shm::RingCtl();
    pe->ctl->head.store(0);
    pe->ctl->tail.store(0);
    pe->data = m + sizeof(shm::RingCtl);
    pe->out.attach(pe->ctl, pe->data, ring_bytes);
    pe->in.attach(own_->ring_ctl(p), own_->ring_data(p), ring_bytes);
    pe->rbuf.resize(ring_bytes);
    peers_[p] = std::move(pe);
  }
  event_fd_ = ::eventfd(0, EFD_NONBLOCK | EFD_CLOEXEC);
  if (event_fd_ < 0) sys_fail("eventfd");
}

Links::~Links() {
  stop();
  for (auto& pe : peers_)
    if (pe && pe->fd >= 0) ::close(pe->fd);
  if (listen_fd_ >= 0) ::close(listen_fd_);
  if (event_fd_ >= 0) ::close(event_fd_);
}

shm::RingCtl* Links::out_ctl(int p) const { return peers_[p]->ctl; }
char* Links::out_data(int p) const { return peers_[p]->data; }

void Links::connect(c10d::Store& store, const std::string& pfx, std::chrono::milliseconds timeout) {
  const auto deadline = std::chrono::steady_clock::now() + timeout;
  // every peer on this host as well (COMMUX_TRANSPORT=tcp on one machine):
  // loopback is enough
  bool loopback_ok = env_str("COMMUX_TRANSPORT") == "tcp" && env_str("COMMUX_TCP_ADDR").empty() &&
                     env_str("COMMUX_TCP_CROSS_HOST").empty();
  listen_fd_ = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (listen_fd_ < 0) sys_fail("socket");
  int one = 1;
  ::setsockopt(listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_addr.s_addr = htonl(loopback_ok ? INADDR_LOOPBACK : INADDR_ANY);
  a.sin_port = 0;
  if (::bind(listen_fd_, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0) sys_fail("bind");
  if (::listen(listen_fd_, size_) != 0) sys_fail("listen");
  socklen_t len = sizeof(a);
  ::getsockname(listen_fd_, reinterpret_cast<sockaddr*>(&a), &len);
  const std::string me = local_addr(loopback_ok) + ":" + std::to_string(ntohs(a.sin_port));
  store.set(pfx + "tcp/" + std::to_string(rank_), std::vector<std::uint8_t>(me.begin(), me.end()));

  // dial every lower remote rank
  for (int p = 0; p < rank_; ++p) {
    if (!remote_[p]) continue;
    const std::string k = pfx + "tcp/" + std::to_string(p);
    store.wait({k}, timeout);
    auto v = store.get(k);
    std::string addr(v.begin(), v.end());
    auto colon = addr.rfind(':');
    sockaddr_in dst{};
    if (colon == std::string::npos || !resolve_v4(addr.substr(0, colon), &dst))
      throw std::runtime_error("commux tcp: bad address '" + addr + "' for rank " + std::to_string(p));
    dst.sin_port = htons(static_cast<std::uint16_t>(std::stoi(addr.substr(colon + 1))));
    int fd = -1;
    for (;;) {
      fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
      if (fd < 0) sys_fail("socket");
      if (::connect(fd, reinterpret_cast<sockaddr*>(&dst), sizeof(dst)) == 0) break;
      ::close(fd);
      if (std::chrono::steady_clock::now() > deadline)
        throw std::runtime_error("commux tcp: cannot connect to rank " + std::to_string(p) + " at " + addr);
      std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    Hello h{kHelloMagic, static_cast<std::uint32_t>(rank_)};
    if (!io_all(fd, &h, sizeof(h), true, deadline))
      throw std::runtime_error("commux tcp: handshake with rank " + std::to_string(p) + " failed");
    tune(fd);
    set_nonblocking(fd);
    peers_[p]->fd = fd;
  }
  // accept every higher remote rank
  int expect = 0;
  for (int p = rank_ + 1; p < size_; ++p) expect += remote_[p] ? 1 : 0;
  while (expect > 0) {
    pollfd pf{listen_fd_, POLLIN, 0};
    auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - std::chrono::steady_clock::now());
    if (left.count() <= 0) throw std::runtime_error("commux tcp: peers did not connect in time");
    if (::poll(&pf, 1, static_cast<int>(std::min<long long>(left.count(), 1000))) <= 0) continue;
    int fd = ::accept4(listen_fd_, nullptr, nullptr, SOCK_CLOEXEC);
    if (fd < 0) continue;
    Hello h{};
    if (!io_all(fd, &h, sizeof(h), false, deadline) || h.magic != kHelloMagic ||
        h.rank >= static_cast<std::uint32_t>(size_) || static_cast<int>(h.rank) <= rank_ || !remote_[h.rank] ||
        peers_[h.rank]->fd >= 0) {
      ::close(fd);
      continue;
    }
    tune(fd);
    set_nonblocking(fd);
    peers_[h.rank]->fd = fd;
    --expect;
  }
  ::close(listen_fd_);
  listen_fd_ = -1;
}

void Links::start(std::function<void()> wake, std::function<void(int, const std::string&)> dead,
                  std::function<void(std::uint64_t)> sent) {
  wake_ = std::move(wake);
  dead_ = std::move(dead);
  sent_cb_ = std::move(sent);
  thread_ = std::thread([this] { pump(); });
}

void Links::notify() {
  std::uint64_t one = 1;
  ssize_t r = ::write(event_fd_, &one, sizeof(one));
  (void)r;
}

void Links::stop() {
  if (stop_.exchange(true)) return;
  notify();
  if (thread_.joinable()) thread_.join();
}

bool Links::pump_peer(Peer& P, bool* want_out, bool* blocked_in) {
  bool work = false;
  auto fail = [&](const std::string& why) {
    P.dead = true;
    if (dead_)
      dead_(P.p, "commux: peer rank " + std::to_string(P.p) + " failed: its TCP connection was lost (" + why + ")");
  };
  // outbound: whole records from the out-ring, in order
  static const char kZeros[8] = {};
  for (;;) {
    if (P.cur == nullptr) {
      const shm::WireHdr* h = P.out.peek();
      if (h == nullptr) break;
      P.cur = h;
      if (h->type == proto::kIndirect) {
        // header carried in the record, payload from the sender's memory,
        // zero padding up to wire_len
        P.ind = reinterpret_cast<const proto::IndirectRec*>(h);
        P.ioff = 0;
        P.sleft = P.ind->wire_len;
      } else {
        P.ind = nullptr;
        P.sptr = reinterpret_cast<const char*>(h);
        P.sleft = h->len;
      }
    }
    ssize_t n;
    if (P.ind != nullptr) {
      const proto::IndirectRec& ir = *P.ind;
      const std::uint64_t hb = ir.head_bytes, pb = ir.payload_bytes;
      iovec iov[3];
      int k = 0;
      std::uint64_t off = P.ioff;
      if (off < hb) {
        char* head = const_cast<char*>(reinterpret_cast<const char*>(ir.head));
        iov[k++] = {head + off, static_cast<std::size_t>(hb - off)};
        off = hb;
      }
      if (off < hb + pb) {
        iov[k++] = {reinterpret_cast<char*>(ir.payload) + (off - hb), static_cast<std::size_t>(hb + pb - off)};
        off = hb + pb;
      }
      if (off < ir.wire_len) iov[k++] = {const_cast<char*>(kZeros), static_cast<std::size_t>(ir.wire_len - off)};
      msghdr m{};
      m.msg_iov = iov;
      m.msg_iovlen = static_cast<std::size_t>(k);
      n = ::sendmsg(P.fd, &m, MSG_NOSIGNAL | MSG_DONTWAIT);
      if (n > 0) P.ioff += static_cast<std::uint64_t>(n);
    } else {
      n = ::send(P.fd, P.sptr, P.sleft, MSG_NOSIGNAL | MSG_DONTWAIT);
      if (n > 0) P.sptr += n;
    }
    if (n > 0) {
      P.sleft -= static_cast<std::uint64_t>(n);
      sent_ += n;
      work = true;
      if (P.sleft == 0) {
        const bool report = P.ind != nullptr && (P.ind->h.flags & proto::kIndirectComplete) != 0;
        const std::uint64_t id = report ? P.ind->done_id : 0;
        P.out.pop(P.cur);
        P.cur = nullptr;
        P.ind = nullptr;
        if (report && sent_cb_) sent_cb_(id);
      }
      continue;
    }
    if (n < 0 && errno == EINTR) continue;
    if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
      *want_out = true;
      break;
    }
    P.out.release();
    fail(std::string("send: ") + std::strerror(errno));
    return work;
  }
  P.out.release();
  // inbound: bytes -> whole records -> this rank's in-ring for the peer
  const std::uint64_t max_rec = ring_bytes_ / 2;
  for (;;) {
    if (P.direct != nullptr) {
      // the rest of a large record, straight into its reserved slot; the
      // slot is published only once the record is complete
      while (P.dgot < P.dlen) {
        ssize_t n = ::recv(P.fd, P.direct + P.dgot, P.dlen - P.dgot, MSG_DONTWAIT);
        if (n > 0) {
          P.dgot += static_cast<std::uint64_t>(n);
          received_ += n;
          work = true;
          continue;
        }
        if (n == 0) {
          P.eof = true;  // closed inside a record: the partial record is dropped
          return work;
        }
        if (errno == EINTR) continue;
        if (errno == EAGAIN || errno == EWOULDBLOCK) return work;
        fail(std::string("recv: ") + std::strerror(errno));
        return work;
      }
      P.direct = nullptr;
      P.in.publish();
      if (wake_) wake_();
      work = true;
    }
    std::size_t off = 0;
    bool published = false;
    while (P.rlen - off >= sizeof(shm::WireHdr)) {
      const auto* h = reinterpret_cast<const shm::WireHdr*>(P.rbuf.data() + off);
      if (h->len < sizeof(shm::WireHdr) || (h->len & 7u) != 0 || h->len > max_rec) {
        fail("corrupt record stream");
        return work;
      }
      if (P.rlen - off < h->len) {
        if (h->len < kDirectRecvBytes) break;
        // a large record in pieces: publish the complete records first
        // (publish() covers every reservation), then reserve its slot
        if (published) {
          P.in.publish();
          if (wake_) wake_();
          published = false;
          work = true;
        }
        char* dst = P.in.reserve(h->len);
        if (dst == nullptr) {
          *blocked_in = true;
          break;
        }
        const std::uint64_t have = P.rlen - off;
        std::memcpy(dst, h, have);
        P.direct = dst;
        P.dlen = h->len;
        P.dgot = have;
        off = P.rlen;
        break;
      }
      char* dst = P.in.reserve(h->len);
      if (dst == nullptr) {
        *blocked_in = true;
        break;
      }
      std::memcpy(dst, h, h->len);
      off += h->len;
      published = true;
    }
    if (published) {
      P.in.publish();
      if (wake_) wake_();
      work = true;
    }
    if (off > 0) {
      std::memmove(P.rbuf.data(), P.rbuf.data() + off, P.rlen - off);
      P.rlen -= off;
    }
    if (P.direct != nullptr) continue;  // receive the rest of the large record
    if (*blocked_in || P.rlen == P.rbuf.size()) break;
    ssize_t n = ::recv(P.fd, P.rbuf.data() + P.rlen, P.rbuf.size() - P.rlen, MSG_DONTWAIT);
    if (n > 0) {
      P.rlen += static_cast<std::size_t>(n);
      received_ += n;
      work = true;
      continue;
    }
    if (n == 0) {
      // Orderly close. Records that arrived before it may still sit in the
      // in-ring (or be waiting for room there): the peer is reported only
      // once the engine has consumed them, so a message sent just before
      // the peer left is still delivered.
      P.eof = true;
      return work;
    }
    if (errno == EINTR) continue;
    if (errno == EAGAIN || errno == EWOULDBLOCK) break;
    fail(std::string("recv: ") + std::strerror(errno));
    return work;
  }
  return work;
}

void Links::pump() {
  std::vector<pollfd> fds;
  std::chrono::steady_clock::time_point drain_until{};
  for (;;) {
    const bool stopping = stop_.load(std::memory_order_acquire);
    const auto now = std::chrono::steady_clock::now();
    if (stopping && drain_until == std::chrono::steady_clock::time_point{})
      drain_until = now + std::chrono::seconds(10);
    bool work = false, blocked = false, out_left = false;
    fds.clear();
    fds.push_back({event_fd_, POLLIN, 0});
    for (auto& pe : peers_) {
      if (!pe || pe->dead || pe->fd < 0) continue;
      bool want_out = false, blocked_in = false;
      work |= pump_peer(*pe, &want_out, &blocked_in);
      if (pe->dead) continue;
      out_left |= pe->sleft > 0 || pe->out.peek() != nullptr;
      if (pe->eof) {
        const shm::RingCtl* c = own_->ring_ctl(pe->p);
        const bool consumed = c->head.load(std::memory_order_acquire) == c->tail.load(std::memory_order_acquire);
        if (pe->rlen == 0 && consumed) {
          pe->dead = true;
          if (dead_)
            dead_(pe->p, "commux: peer rank " + std::to_string(pe->p) + " failed: it closed its TCP connection");
          continue;
        }
        blocked = true;  // re-check soon
        if (want_out) fds.push_back({pe->fd, POLLOUT, 0});
        continue;
      }
      blocked |= blocked_in;
      short ev = static_cast<short>((blocked_in ? 0 : POLLIN) | (want_out ? POLLOUT : 0));
      fds.push_back({pe->fd, ev, 0});
    }
    // on stop, what the engine already wrote is still sent (bounded)
    if (stopping && (!out_left || now > drain_until)) break;
    if (work) continue;
    // a full in-ring, or a closed peer with records still queued, is
    // re-checked every millisecond (the consumer drains it)
    ::poll(fds.data(), fds.size(), blocked || stopping ? 1 : 100);
    if (fds[0].revents & POLLIN) {
      std::uint64_t v;
      ssize_t r = ::read(event_fd_, &v, sizeof(v));
      (void)r;
    }
  }
}

}  // namespace tcp
}  // namespace commux
