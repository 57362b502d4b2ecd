#include "engine.hpp"

#include <sys/uio.h>
#include "log.hpp"

#include <c10/util/Exception.h>
#include <dlfcn.h>
#include <signal.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <sstream>

#if defined(__x86_64__)
#include <immintrin.h>
#define COMMUX_PAUSE() _mm_pause()
#else
#define COMMUX_PAUSE() std::this_thread::yield()
#endif

namespace commux {

std::int64_t env_int(const char* name, std::int64_t dflt) {
  const char* e = std::getenv(name);
  if (e == nullptr || *e == '\0') return dflt;
  char* end = nullptr;
  long long v = std::strtoll(e, &end, 0);
  if (end == e) return dflt;
  return static_cast<std::int64_t>(v);
}

bool env_flag(const char* name) {
  const char* e = std::getenv(name);
  if (e == nullptr) return false;
  std::string s(e);
  return s == "1" || s == "on" || s == "ON" || s == "true" || s == "yes";
}

namespace {

constexpr tag_t kKeyMask = 0x0000FFFFFFFFFFFFull;

std::uint64_t default_ring_bytes(int size) {
  std::int64_t v = env_int("COMMUX_SHM_RING_BYTES", 0);
  if (v <= 0) {
    // 4 MiB per ordered pair up to 32 ranks, shrinking beyond so one host's
    // segments stay bounded (size^2 rings in total).
    std::int64_t budget = 128ll << 20;
    v = std::min<std::int64_t>(4ll << 20, std::max<std::int64_t>(256ll << 10, budget / size));
  }
  v = (v + 4095) & ~4095ll;
  return static_cast<std::uint64_t>(v);
}

std::string hexid(std::uint64_t v) {
  char buf[32];
  std::snprintf(buf, sizeof(buf), "%016llx", static_cast<unsigned long long>(v));
  return buf;
}

std::vector<std::uint8_t> to_bytes(const std::string& s) {
  return std::vector<std::uint8_t>(s.begin(), s.end());
}
std::string from_bytes(const std::vector<std::uint8_t>& v) {
  return std::string(v.begin(), v.end());
}

[[noreturn]] void throw_backend(const std::string& msg) {
  C10_THROW_ERROR(DistBackendError, msg);
}

// A process that exited but was not reaped yet (a zombie) still answers
// kill(pid, 0); its /proc state says Z (or X) though.
bool pid_alive(pid_t pid) {
  if (::kill(pid, 0) != 0 && errno == ESRCH) return false;
  char path[64];
  std::snprintf(path, sizeof(path), "/proc/%d/stat", static_cast<int>(pid));
  FILE* f = std::fopen(path, "r");
  if (f == nullptr) return true;  // no procfs view: trust kill()
  char buf[512];
  std::size_t n = std::fread(buf, 1, sizeof(buf) - 1, f);
  std::fclose(f);
  buf[n] = '\0';
  const char* rp = std::strrchr(buf, ')');  // "pid (comm) S ..."
  if (rp == nullptr || rp[1] == '\0' || rp[2] == '\0') return true;
  char state = rp[2];
  return state != 'Z' && state != 'X';
}

}  // namespace

FaultSpec FaultSpec::from_env() {
  FaultSpec f;
  const char* e = std::getenv("COMMUX_FAULT");
  if (e == nullptr) return f;
  std::stringstream ss(e);
  std::string item;
  while (std::getline(ss, item, ',')) {
    std::vector<std::string> parts;
    std::stringstream is(item);
    std::string p;
    while (std::getline(is, p, ':')) parts.push_back(p);
    if (parts.empty()) continue;
    if (parts[0] == "drop" && parts.size() == 3) {
      f.drop_rank = std::atoi(parts[1].c_str());
      f.drop_tag = std::atoll(parts[2].c_str());
    } else if (parts[0] == "kill" && parts.size() == 3) {
      f.kill_rank = std::atoi(parts[1].c_str());
      f.kill_after = std::atoll(parts[2].c_str());
    } else if (parts[0] == "delay" && parts.size() == 2) {
      f.delay_ms = std::atoi(parts[1].c_str());
    } else {
      std::fprintf(stderr, "commux: ignoring malformed COMMUX_FAULT item '%s'\n",
                   item.c_str());
    }
  }
  return f;
}

// ---------------------------------------------------------------------------
// construction / bootstrap
// ---------------------------------------------------------------------------

namespace {
// every live engine (for the exit-time release)
std::mutex g_registry_mu;
std::vector<Engine*>& registry() {
  static std::vector<Engine*> r;
  return r;
}
}  // namespace

Engine::Engine(c10::intrusive_ptr<c10d::Store> store, int rank, int size,
               std::chrono::milliseconds timeout)
    : store_(std::move(store)),
      rank_(rank),
      size_(size),
      timeout_(timeout.count() > 0 ? timeout : std::chrono::milliseconds(30 * 60 * 1000)),
      dead_(static_cast<std::size_t>(size)) {
  TORCH_CHECK(size >= 1 && size <= 0xFFFF, "commux: world size must be in [1, 65535]");
  TORCH_CHECK(rank >= 0 && rank < size, "commux: rank ", rank, " out of range");
  for (auto& d : dead_) d.store(false);
  eager_limit_ = static_cast<std::uint64_t>(env_int("COMMUX_EAGER_BYTES", 64 << 10));
  spin_us_ = static_cast<int>(env_int("COMMUX_PROGRESS_SPIN_US", 200));
  spin_wait_us_ = static_cast<int>(std::max<std::int64_t>(0, env_int("COMMUX_WAIT_SPIN_US", 100)));
  wait_poll_ms_ = static_cast<int>(env_int("COMMUX_WAIT_POLL_MS", 1));
  if (wait_poll_ms_ <= 0) wait_poll_ms_ = 1;
  fault_ = FaultSpec::from_env();
  cma_enabled_ = env_int("COMMUX_CMA", 1) != 0;
  copy_threads_ = static_cast<int>(std::max<std::int64_t>(0, env_int("COMMUX_COPY_THREADS", 2)));
  cma_off_.reset(new std::atomic<bool>[static_cast<std::size_t>(size)]);
  for (int p = 0; p < size; ++p) cma_off_[p].store(false);
  bootstrap();
  last_liveness_ = std::chrono::steady_clock::now();
  progress_ = std::thread([this] { progress_loop(); });
  std::lock_guard<std::mutex> lk(g_registry_mu);
  registry().push_back(this);
}

void Engine::release_all() {
  std::vector<Engine*> all;
  {
    std::lock_guard<std::mutex> lk(g_registry_mu);
    all = registry();
  }
  for (auto* e : all) e->release_for_exit();
}

void Engine::release_for_exit() {
  if (released_.exchange(true)) return;
  if (my_header() != nullptr) my_header()->closed.store(1);
  stop_.store(true);
  wake_progress();
  if (progress_.joinable()) progress_.join();
  if (links_) links_->stop();
  {
    std::lock_guard<std::mutex> lk(dev_mu_);
    if (dev_) {
      try {
        dev_->shutdown();
      } catch (...) {
      }
      dev_.reset();
    }
  }
  std::lock_guard<SpinMutex> lk(mu_);
  posted_.clear();
  unexpected_.clear();
  sends_waiting_.clear();
  for (auto& m : inflight_) m.clear();
}

Engine::~Engine() {
  {
    std::lock_guard<std::mutex> lk(g_registry_mu);
    auto& r = registry();
    r.erase(std::remove(r.begin(), r.end(), this), r.end());
  }
  if (my_header() != nullptr) my_header()->closed.store(1);
  stop_.store(true);
  wake_progress();
  if (progress_.joinable()) progress_.join();
  if (links_) links_->stop();
  if (dev_) {
    try {
      dev_->shutdown();
    } catch (...) {
    }
    dev_.reset();
  }
  // dev_lib_ stays loaded: kernels/modules registered by it must outlive any
  // CUDA state torch still holds at process exit.
  for (auto& s : segs_)
    if (s) s->unmap();
}

void Engine::store_barrier(const std::string& key) {
  auto v = store_->add(key, 1);
  if (v == size_) store_->set(key + "/done", to_bytes("1"));
  store_->wait({key + "/done"}, timeout_);
}

void Engine::bootstrap() {
  // Generation of this group on the store: every rank adds 1, so the k-th
  // group built on one store sees values in [k*size+1, (k+1)*size]. The
  // barrier at the end keeps generations from interleaving.
  auto v = store_->add("commux/join", 1);
  std::int64_t gen = (v - 1) / size_;
  std::string pfx = "commux/" + std::to_string(gen) + "/";
  prefix_ = pfx;

  std::uint64_t instance = 0;
  if (rank_ == 0) {
    std::random_device rd;
    instance = (static_cast<std::uint64_t>(rd()) << 32) ^ rd() ^
               (static_cast<std::uint64_t>(::getpid()) << 16) ^
               static_cast<std::uint64_t>(
                   std::chrono::steady_clock::now().time_since_epoch().count());
    store_->set(pfx + "instance", to_bytes(hexid(instance)));
  } else {
    store_->wait({pfx + "instance"}, timeout_);
    instance = std::stoull(from_bytes(store_->get(pfx + "instance")), nullptr, 16);
  }

  std::uint64_t ring = default_ring_bytes(size_);
  frag_bytes_ = std::min<std::uint64_t>(ring / 4, 1ull << 20) - 64;
  frag_bytes_ &= ~63ull;

  segs_.resize(size_);
  std::string myname = "/cmx." + hexid(instance).substr(4) + "." + std::to_string(rank_);
  segs_[rank_] = std::make_unique<shm::Segment>();
  segs_[rank_]->create(myname, size_, rank_, ring, instance);
  char host[64] = {0};
  ::gethostname(host, sizeof(host) - 1);
  store_->set(pfx + "seg/" + std::to_string(rank_),
              to_bytes(myname + "\n" + host + "\n" + std::to_string(::getpid())));
  // Same-host peers map each other's segments; peers on other hosts (or every
  // peer under COMMUX_TRANSPORT=tcp) are reached through TCP links.
  remote_.assign(static_cast<std::size_t>(size_), false);
  for (int p = 0; p < size_; ++p) {
    if (p == rank_) continue;
    std::string k = pfx + "seg/" + std::to_string(p);
    store_->wait({k}, timeout_);
    std::string val = from_bytes(store_->get(k));
    std::stringstream ss(val);
    std::string name, phost;
    std::getline(ss, name);
    std::getline(ss, phost);
    if (tcp::use_tcp(host, phost)) {
      remote_[p] = true;
      any_remote_ = true;
      continue;
    }
    segs_[p] = std::make_unique<shm::Segment>();
    segs_[p]->open(name);
    if (segs_[p]->header()->instance != instance)
      throw std::runtime_error("commux: segment " + name + " belongs to another group");
  }
  if (any_remote_) links_ = std::make_unique<tcp::Links>(rank_, size_, ring, remote_, segs_[rank_].get());
  in_.resize(size_);
  out_.resize(size_);
  inflight_.resize(size_);
  for (int p = 0; p < size_; ++p) {
    in_[p].attach(segs_[rank_]->ring_ctl(p), segs_[rank_]->ring_data(p), ring);
    out_[p] = std::make_unique<PeerOut>();
    if (remote_[p])
      out_[p]->ring.attach(links_->out_ctl(p), links_->out_data(p), ring);
    else
      out_[p]->ring.attach(segs_[p]->ring_ctl(rank_), segs_[p]->ring_data(rank_), ring);
  }
  if (links_) {
    links_->connect(*store_, pfx, timeout_);
    links_->start([this] { wake_progress(); },
                  [this](int p, const std::string& why) { fail_peer(p, why); },
                  [this](std::uint64_t id) { on_pump_sent(id); });
  }
  // Everyone has mapped everyone: drop the names so a crash leaks nothing.
  store_barrier(pfx + "mapped");
  segs_[rank_]->unlink();
  int ntcp = 0;
  for (int p = 0; p < size_; ++p) ntcp += remote_[p] ? 1 : 0;
  logf(LogLevel::Info, rank_, "transports: %d peer(s) over shared memory, %d over TCP", size_ - 1 - ntcp, ntcp);
  logf(LogLevel::Info, rank_,
       "engine up: %d ranks on host %s, shm rings of %llu bytes per peer, eager <= %lld bytes, "
       "COMMUX_COALESCE=%d COMMUX_GROUP=%d, timeout %lld ms",
       size_, host, static_cast<unsigned long long>(ring), static_cast<long long>(eager_limit_),
       env_int("COMMUX_COALESCE", 0) != 0 ? 1 : 0, env_int("COMMUX_GROUP", 0) != 0 ? 1 : 0,
       static_cast<long long>(timeout_.count()));
}

// ---------------------------------------------------------------------------
// posting
// ---------------------------------------------------------------------------

void Engine::count_op() {
  auto n = op_count_.fetch_add(1) + 1;
  if (fault_.kill_rank == rank_ && fault_.kill_after >= 0 && n >= fault_.kill_after) {
    std::fprintf(stderr, "commux: fault injection: rank %d exits at operation %lld\n",
                 rank_, static_cast<long long>(n));
    std::fflush(stderr);
    ::_exit(77);
  }
}

ReqPtr Engine::post_send(std::vector<at::Tensor> tensors, int dst, tag_t tag) {
  count_op();
  if (released_.load()) throw_backend("commux: the process is shutting down");
  if (aborted_.load()) throw_backend("commux: group aborted: " + failure_reason());
  if (dead_[dst].load())
    throw_backend("commux send: peer rank " + std::to_string(dst) + " has failed");
  auto r = std::make_shared<Request>();
  r->kind = ReqKind::Send;
  r->peer = dst;
  r->key = tag & kKeyMask;
  r->id = next_id_.fetch_add(1);
  r->posted_at = std::chrono::steady_clock::now();
  r->device = !tensors.empty() && tensors[0].is_cuda();
  TORCH_CHECK(!r->device || !remote(dst),
              "commux send: CUDA tensors to a rank on another host must be staged through host memory");
  for (auto& t : tensors) {
    TORCH_CHECK(t.is_cuda() == r->device,
                "commux send: a coalesced message mixes CPU and CUDA tensors");
    r->total += static_cast<std::uint64_t>(t.numel()) * t.element_size();
  }
  r->tensors = std::move(tensors);
  stats_.sends++;
  stats_.bytes_sent += static_cast<std::int64_t>(r->total);

  const bool drop = fault_.drop_rank == rank_ &&
                    static_cast<std::int64_t>(tag & 0xFFFFFFFFull) == fault_.drop_tag;
  if (drop) {
    stats_.faults_injected++;
    complete(r);
    return r;
  }

  if (r->device) {
    stats_.device_msgs++;
    DeviceTransport* d = device();
    std::vector<char> blob;
    bool gate = false, complete_on_post = false;
    if (dst == rank_) {
      // Self-send: matched here, in the posting thread, so the copy can be
      // launched on the caller's stream (no ring, no progress thread).
      d->prepare_send(r, dst, blob, &gate, &complete_on_post);
      ReqPtr rr;
      {
        std::lock_guard<SpinMutex> lk(mu_);
        rr = match_posted(rank_, r->key);
        if (rr) {
          rr->source = rank_;
        } else {
          auto u = std::make_shared<Unexpected>();
          u->src = rank_;
          u->key = r->key;
          u->type = proto::kDrts;
          u->total = r->total;
          u->msg_id = r->id;
          u->data = std::move(blob);
          unexpected_[r->key].push_back(u);
          ++unexpected_count_;
          stats_.unexpected_msgs++;
          return r;
        }
      }
      if (!rr->device) {
        fail(rr, "commux recv: a CUDA tensor was sent to a CPU receive buffer; "
                 "send and receive tensors must live on the same kind of device");
        fail(r, "commux send: the matching receive buffer is a CPU tensor");
        return r;
      }
      d->on_match(rr, rank_, r->id, blob.data(), blob.size());
      return r;
    }
    {
      std::lock_guard<SpinMutex> lk(mu_);
      sends_waiting_[r->id] = r;
    }
    d->prepare_send(r, dst, blob, &gate, &complete_on_post);
    auto job = std::make_unique<OutJob>();
    job->complete_req_when_done = complete_on_post;
    job->type = proto::kDrts;
    job->head.resize(sizeof(proto::DrtsRec) + blob.size());
    auto* rec = reinterpret_cast<proto::DrtsRec*>(job->head.data());
    rec->key = r->key;
    rec->total = r->total;
    rec->send_id = r->id;
    rec->blob_bytes = static_cast<std::uint32_t>(blob.size());
    rec->pad = 0;
    std::memcpy(job->head.data() + sizeof(proto::DrtsRec), blob.data(), blob.size());
    job->req = r;
    if (gate) {
      enqueue(dst, std::move(job));
      wake_progress();  // the progress thread sends it once the data is ready
    } else {
      post_job(dst, std::move(job));
    }
    return r;
  }

  for (auto& t : r->tensors) {
    TORCH_CHECK(t.is_contiguous(), "commux send: internal error, non-contiguous host tensor");
    r->host.push_back({static_cast<char*>(t.data_ptr()),
                       static_cast<std::uint64_t>(t.numel()) * t.element_size()});
  }
  auto job = std::make_unique<OutJob>();
  if (r->total <= eager_limit_) {
    stats_.eager_msgs++;
    job->type = proto::kEager;
    job->req = r;
    job->msg_id = r->id;
    job->total = r->total;
    job->complete_req_when_done = true;
  } else {
    stats_.rndv_msgs++;
    {
      std::lock_guard<SpinMutex> lk(mu_);
      sends_waiting_[r->id] = r;
    }
    job->type = proto::kRts;
    // a same-host receiver may copy straight out of these segments
    const bool cma = cma_enabled_ && !remote(dst) && r->host.size() <= proto::kCmaSegs;
    const std::uint32_t nseg = cma ? static_cast<std::uint32_t>(r->host.size()) : 0u;
    job->head.assign(sizeof(proto::RtsRec) + nseg * sizeof(proto::CmaSeg), 0);
    auto* rec = reinterpret_cast<proto::RtsRec*>(job->head.data());
    rec->key = r->key;
    rec->total = r->total;
    rec->send_id = r->id;
    rec->pid = static_cast<std::int32_t>(::getpid());
    rec->nseg = nseg;
    auto* segs = reinterpret_cast<proto::CmaSeg*>(rec + 1);
    for (std::uint32_t i = 0; i < nseg; ++i)
      segs[i] = {reinterpret_cast<std::uint64_t>(r->host[i].ptr), r->host[i].bytes};
  }
  post_job(dst, std::move(job));
  return r;
}

ReqPtr Engine::post_recv(std::vector<at::Tensor> tensors, int src, tag_t tag) {
  count_op();
  if (released_.load()) throw_backend("commux: the process is shutting down");
  if (aborted_.load()) throw_backend("commux: group aborted: " + failure_reason());
  if (src >= 0 && dead_[src].load())
    throw_backend("commux recv: peer rank " + std::to_string(src) + " has failed");
  auto r = std::make_shared<Request>();
  r->kind = ReqKind::Recv;
  r->peer = src;
  r->key = tag & kKeyMask;
  r->id = next_id_.fetch_add(1);
  r->posted_at = std::chrono::steady_clock::now();
  r->device = !tensors.empty() && tensors[0].is_cuda();
  TORCH_CHECK(!r->device || (src >= 0 ? !remote(src) : !any_remote_),
              "commux recv: CUDA tensors from a rank on another host must be staged through host memory");
  for (auto& t : tensors) {
    TORCH_CHECK(t.is_cuda() == r->device,
                "commux recv: a coalesced message mixes CPU and CUDA tensors");
    r->total += static_cast<std::uint64_t>(t.numel()) * t.element_size();
  }
  r->tensors = std::move(tensors);
  stats_.recvs++;
  if (r->device) {
    device()->prepare_recv(r);
  } else {
    for (auto& t : r->tensors) {
      TORCH_CHECK(t.is_contiguous(), "commux recv: destination tensor must be contiguous");
      r->host.push_back({static_cast<char*>(t.data_ptr()),
                         static_cast<std::uint64_t>(t.numel()) * t.element_size()});
    }
  }

  UnexpPtr u;
  bool flush_to = false;
  bool cma = false;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    u = match_unexpected(src, r->key);
    if (!u) {
      posted_[r->key].push_back(r);
      return r;
    }
    r->source = u->src;
    if (u->type == proto::kEager) {
      if (!u->complete) {
        u->bound = r;  // the progress thread delivers when the bytes land
        return r;
      }
    } else if (u->type == proto::kRts) {
      if (r->device) {
        // fall through: reject below
      } else if (u->total > r->total) {
        // reject: tell the sender (recv id 0)
      } else if (!u->data.empty() && !cma_off_[u->src].load()) {
        cma = true;  // single-copy read, outside the lock
      } else {
        start_rndv_recv(r, u->src, u->msg_id, u->total);
        flush_to = true;
      }
    }
  }
  if (cma) {
    const auto* segs = reinterpret_cast<const proto::CmaSeg*>(u->data.data());
    const auto nseg = static_cast<std::uint32_t>(u->data.size() / sizeof(proto::CmaSeg));
    if (cma_read(u->src, r, u->pid, segs, nseg, u->total)) {
      send_fin(u->src, u->msg_id, 0);
      complete(r);
      return r;
    }
    {
      std::lock_guard<SpinMutex> lk(mu_);
      start_rndv_recv(r, u->src, u->msg_id, u->total);
    }
    flush_out(u->src, false);
    return r;
  }
  if (flush_to) {
    flush_out(u->src, false);
    return r;
  }
  if (u->type == proto::kEager) {
    deliver_unexpected(r, u);
  } else if (u->type == proto::kRts) {
    auto job = std::make_unique<OutJob>();
    job->type = proto::kCts;
    job->head.resize(sizeof(proto::CtsRec));
    auto* rec = reinterpret_cast<proto::CtsRec*>(job->head.data());
    rec->send_id = u->msg_id;
    rec->recv_id = 0;
    enqueue(u->src, std::move(job));
    flush_out(u->src, false);
    if (r->device)
      fail(r, "commux recv: a CPU tensor was sent to a CUDA receive buffer; "
              "send and receive tensors must live on the same kind of device");
    else
      fail(r, "commux recv: message of " + std::to_string(u->total) +
                  " bytes does not fit the " + std::to_string(r->total) + "-byte buffer");
  } else if (u->type == proto::kDrts) {
    if (!r->device) {
      send_fin(u->src, u->msg_id, -2);
      fail(r, "commux recv: a CUDA tensor was sent to a CPU receive buffer; "
              "send and receive tensors must live on the same kind of device");
    } else {
      device()->on_match(r, u->src, u->msg_id, u->data.data(), u->data.size());
    }
  }
  return r;
}

// ---------------------------------------------------------------------------
// matching (mu_ held)
// ---------------------------------------------------------------------------

ReqPtr Engine::match_posted(int src, tag_t key) {
  auto it = posted_.find(key);
  if (it == posted_.end()) return nullptr;
  auto& dq = it->second;
  for (auto q = dq.begin(); q != dq.end(); ++q) {
    if ((*q)->peer == src || (*q)->peer < 0) {
      ReqPtr r = *q;
      dq.erase(q);
      if (dq.empty()) posted_.erase(it);
      return r;
    }
  }
  return nullptr;
}

UnexpPtr Engine::match_unexpected(int src, tag_t key) {
  auto it = unexpected_.find(key);
  if (it == unexpected_.end()) return nullptr;
  auto& dq = it->second;
  for (auto q = dq.begin(); q != dq.end(); ++q) {
    if (src < 0 || (*q)->src == src) {
      UnexpPtr u = *q;
      dq.erase(q);
      if (dq.empty()) unexpected_.erase(it);
      --unexpected_count_;
      return u;
    }
  }
  return nullptr;
}

void Engine::start_rndv_recv(const ReqPtr& r, int src, std::uint64_t send_id,
                             std::uint64_t total) {
  Inflight inf;
  inf.recv = r;
  inf.total = total;
  inflight_[src][r->id | proto::kDataBit] = inf;
  auto job = std::make_unique<OutJob>();
  job->type = proto::kCts;
  job->head.resize(sizeof(proto::CtsRec));
  auto* rec = reinterpret_cast<proto::CtsRec*>(job->head.data());
  rec->send_id = send_id;
  rec->recv_id = r->id;
  enqueue(src, std::move(job));
}

void Engine::scatter(const ReqPtr& r, std::uint64_t off, const char* data,
                     std::uint64_t n) {
  if (n == 0) return;
  stats_.host_copies++;
  for (auto& s : r->host) {
    if (off >= s.bytes) {
      off -= s.bytes;
      continue;
    }
    std::uint64_t k = std::min(n, s.bytes - off);
    std::memcpy(s.ptr + off, data, k);
    data += k;
    n -= k;
    off = 0;
    if (n == 0) break;
  }
}

void Engine::deliver_unexpected(const ReqPtr& r, const UnexpPtr& u) {
  if (u->total > r->total) {
    fail(r, "commux recv: message of " + std::to_string(u->total) +
                " bytes does not fit the " + std::to_string(r->total) + "-byte buffer");
    return;
  }
  if (r->device) {
    fail(r, "commux recv: a CPU tensor was sent to a CUDA receive buffer; "
            "send and receive tensors must live on the same kind of device");
    return;
  }
  scatter(r, 0, u->data.data(), u->total);
  r->landed = u->total;
  stats_.bytes_recv += static_cast<std::int64_t>(u->total);
  complete(r);
}

// ---------------------------------------------------------------------------
// completion and waiting
// ---------------------------------------------------------------------------

void Engine::complete(const ReqPtr& r) {
  int expected = kPending;
  if (!r->state.compare_exchange_strong(expected, kDone, std::memory_order_seq_cst)) return;
  if (waiters_.load(std::memory_order_seq_cst) > 0) {
    std::lock_guard<std::mutex> lk(done_mu_);
    done_cv_.notify_all();
  }
}

void Engine::fail(const ReqPtr& r, const std::string& why) {
  if (r->state.load() != kPending) return;
  r->error = why;
  int expected = kPending;
  if (!r->state.compare_exchange_strong(expected, kFailed, std::memory_order_acq_rel)) return;
  std::lock_guard<std::mutex> lk(done_mu_);
  done_cv_.notify_all();
}

void Engine::wait(const ReqPtr& r, std::chrono::milliseconds timeout) {
  auto limit = timeout.count() > 0 ? timeout : timeout_;
  auto t0 = std::chrono::steady_clock::now();
  auto deadline = t0 + limit;
  // brief spin: most waits in a latency-bound exchange end within
  // microseconds. Bounded by time, not by a count: the latency of one pause
  // differs by an order of magnitude between CPU generations.
  if (r->state.load(std::memory_order_acquire) == kPending) {
    const auto spin_end = t0 + std::chrono::microseconds(spin_wait_us_);
    for (int i = 0; r->state.load(std::memory_order_acquire) == kPending; ++i) {
      COMMUX_PAUSE();
      if ((i & 63) == 63 && std::chrono::steady_clock::now() >= spin_end) break;
    }
  }
  if (r->state.load(std::memory_order_acquire) == kPending) {
    waiters_.fetch_add(1);
    std::unique_lock<std::mutex> lk(done_mu_);
    while (r->state.load(std::memory_order_acquire) == kPending) {
      // Bounded sleep (COMMUX_WAIT_POLL_MS): a parked waiter re-checks even if
      // its wakeup was consumed by another thread (reference rationale:
      // src/process_group_ucx.cpp:47-62).
      done_cv_.wait_for(lk, std::chrono::milliseconds(wait_poll_ms_));
      if (r->state.load(std::memory_order_acquire) != kPending) break;
      if (aborted_.load()) {
        lk.unlock();
        fail(r, "commux: group aborted: " + failure_reason());
        lk.lock();
        break;
      }
      const int srcr = r->source.load();
      int pr = r->kind == ReqKind::Send ? r->peer : (srcr >= 0 ? srcr : r->peer);
      if (pr >= 0 && dead_[pr].load()) {
        lk.unlock();
        fail(r, "commux: peer rank " + std::to_string(pr) + " failed");
        lk.lock();
        break;
      }
      if (std::chrono::steady_clock::now() >= deadline) {
        waiters_.fetch_sub(1);
        lk.unlock();
        std::ostringstream os;
        os << "commux: " << (r->kind == ReqKind::Send ? "send to" : "recv from")
           << " rank " << r->peer << " (tag " << (r->key & 0xFFFFFFFFull)
           << (((r->key >> 32) & 1) ? ", collective" : "") << ", " << r->total
           << " bytes) timed out after " << limit.count() << " ms";
        throw_backend(os.str());
      }
    }
    waiters_.fetch_sub(1);
  }
  if (r->state.load(std::memory_order_acquire) == kFailed) throw_backend(r->error);
}

std::string Engine::failure_reason() const {
  std::lock_guard<SpinMutex> lk(mu_);
  return abort_reason_;
}

void Engine::wake_progress() {
  auto* h = my_header();
  if (h == nullptr) return;
  h->doorbell.fetch_add(1);
  shm::futex_wake(&h->doorbell, 1);
}

// ---------------------------------------------------------------------------
// outbound
// ---------------------------------------------------------------------------

void Engine::enqueue(int dst, std::unique_ptr<OutJob> job) {
  auto& po = *out_[dst];
  std::lock_guard<SpinMutex> lk(po.mu);
  const bool control = job->type == proto::kFin || job->type == proto::kCts ||
                       job->type == proto::kAbort;
  (control ? po.ctrl : po.jobs).push_back(std::move(job));
  po.pending.fetch_add(1);
}

void Engine::post_job(int dst, std::unique_ptr<OutJob> job) {
  auto& po = *out_[dst];
  // released on every exit (a failed write throws): a count left behind
  // would keep the progress thread off this peer's queue for good
  struct Poster {
    std::atomic<int>& n;
    explicit Poster(std::atomic<int>& c) : n(c) { n.fetch_add(1, std::memory_order_acq_rel); }
    ~Poster() { n.fetch_sub(1, std::memory_order_acq_rel); }
  } poster(po.posters);
  enqueue(dst, std::move(job));
  flush_out(dst, false);
}

std::vector<std::pair<std::string, std::int64_t>> Engine::gauges() {
  std::int64_t posted = 0, unexpected = 0, partial = 0, waiting = 0, pump = 0;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    for (auto& kv : posted_) posted += static_cast<std::int64_t>(kv.second.size());
    for (auto& kv : unexpected_) unexpected += static_cast<std::int64_t>(kv.second.size());
    for (auto& m : inflight_) partial += static_cast<std::int64_t>(m.size());
    waiting = static_cast<std::int64_t>(sends_waiting_.size());
  }
  {
    std::lock_guard<std::mutex> lk(pump_mu_);
    pump = static_cast<std::int64_t>(pump_waiting_.size());
  }
  return {{"posted_now", posted},
          {"unexpected_now", unexpected},
          {"partial_now", partial},
          {"sends_waiting_now", waiting},
          {"pump_waiting_now", pump}};
}

CopyPool* Engine::copy_pool() {
  if (copy_threads_ <= 0) return nullptr;
  std::call_once(copy_pool_once_, [&] {
    try {
      copy_pool_ = std::make_unique<CopyPool>(copy_threads_);
    } catch (const std::exception& e) {  // no threads to spare: work alone
      logf(LogLevel::Info, rank_, "copy helper threads unavailable (%s)", e.what());
    }
  });
  return copy_pool_.get();
}

void Engine::parallel_ranges(std::int64_t n, std::int64_t grain,
                             const std::function<void(std::int64_t, std::int64_t)>& fn) {
  std::int64_t parts = 1;
  if (n >= 2 * grain && copy_threads_ > 0)
    parts = std::min<std::int64_t>(copy_threads_ + 1, n / std::max<std::int64_t>(1, grain));
  CopyPool* pool = parts > 1 ? copy_pool() : nullptr;
  if (pool == nullptr) {
    if (n > 0) fn(0, n);
    return;
  }
  std::vector<std::function<void()>> tasks;
  const std::int64_t step = (n + parts - 1) / parts;
  for (std::int64_t lo = 0; lo < n; lo += step)
    tasks.push_back([&fn, lo, hi = std::min(n, lo + step)] { fn(lo, hi); });
  pool->run_all(tasks);
}

void Engine::on_pump_sent(std::uint64_t id) {
  ReqPtr r;
  {
    std::lock_guard<std::mutex> lk(pump_mu_);
    auto it = pump_waiting_.find(id);
    if (it == pump_waiting_.end()) return;
    r = std::move(it->second);
    pump_waiting_.erase(it);
  }
  complete(r);
}

void Engine::send_fin(int dst, std::uint64_t send_id, std::int64_t status) {
  auto job = std::make_unique<OutJob>();
  job->type = proto::kFin;
  job->head.resize(sizeof(proto::FinRec));
  auto* rec = reinterpret_cast<proto::FinRec*>(job->head.data());
  rec->send_id = send_id;
  rec->status = status;
  enqueue(dst, std::move(job));
  flush_out(dst, false);
}

bool Engine::write_job(int dst, PeerOut& po, OutJob& job) {
  auto& ring = po.ring;
  if (fault_.delay_ms > 0) std::this_thread::sleep_for(std::chrono::milliseconds(fault_.delay_ms));
  if (job.type != proto::kEager && job.type != proto::kFrag) {
    std::uint64_t n = shm::align8(job.head.size());
    TORCH_CHECK(n <= ring.max_record(), "commux: control record of ", n,
                " bytes exceeds the ring's record limit; raise COMMUX_SHM_RING_BYTES");
    char* p = ring.reserve(n);
    if (p == nullptr) return false;
    std::memcpy(p, job.head.data(), job.head.size());
    auto* h = reinterpret_cast<shm::WireHdr*>(p);
    h->len = static_cast<std::uint32_t>(n);
    h->type = job.type;
    h->flags = 0;
    stats_.records_out++;
    return true;
  }
  // payload stream: EAGER head + FRAG continuation, or DATA (FRAG only).
  // To a TCP peer, a large payload in one host segment travels as indirect
  // records: the pump sends it straight from the request's memory, and the
  // request completes once the pump has sent its last record.
  constexpr std::uint64_t kIndirectMin = 64 << 10;
  const bool indirect = remote_[dst] && job.req && job.req->host.size() == 1 && job.total >= kIndirectMin &&
                        job.req->host[0].bytes >= job.total;
  while (indirect && (!job.head_sent || job.off < job.total)) {
    const std::uint64_t chunk = std::min<std::uint64_t>(job.total - job.off, frag_bytes_);
    const std::uint64_t hdr = job.head_sent ? sizeof(proto::FragRec) : sizeof(proto::EagerRec);
    const std::uint64_t n = shm::align8(sizeof(proto::IndirectRec));
    char* p = ring.reserve(n);
    if (p == nullptr) return false;
    auto* ir = reinterpret_cast<proto::IndirectRec*>(p);
    std::memset(ir, 0, sizeof(*ir));
    ir->h.len = static_cast<std::uint32_t>(n);
    ir->h.type = proto::kIndirect;
    ir->wire_len = static_cast<std::uint32_t>(shm::align8(hdr + chunk));
    ir->head_bytes = static_cast<std::uint32_t>(hdr);
    ir->payload = reinterpret_cast<std::uint64_t>(job.req->host[0].ptr + job.off);
    ir->payload_bytes = chunk;
    auto* wh = reinterpret_cast<shm::WireHdr*>(ir->head);
    wh->len = ir->wire_len;
    wh->flags = 0;
    if (!job.head_sent) {
      auto* rec = reinterpret_cast<proto::EagerRec*>(ir->head);
      wh->type = proto::kEager;
      rec->key = job.req->key;
      rec->total = job.total;
      rec->msg_id = job.msg_id;
      rec->nbytes = chunk;
      job.head_sent = true;
    } else {
      auto* rec = reinterpret_cast<proto::FragRec*>(ir->head);
      wh->type = proto::kFrag;
      rec->msg_id = job.msg_id;
      rec->offset = job.off;
      rec->nbytes = chunk;
    }
    job.off += chunk;
    if (job.off >= job.total && job.complete_req_when_done) {
      // registered before the ring is published, so the pump finds it
      std::lock_guard<std::mutex> lk(pump_mu_);
      pump_waiting_[job.req->id] = job.req;
      ir->h.flags = proto::kIndirectComplete;
      ir->done_id = job.req->id;
      job.completes_when_sent = true;
    }
    stats_.records_out++;
  }
  while (!job.head_sent || job.off < job.total) {
    std::uint64_t chunk = std::min<std::uint64_t>(job.total - job.off, frag_bytes_);
    std::uint64_t hdr = job.head_sent ? sizeof(proto::FragRec) : sizeof(proto::EagerRec);
    std::uint64_t n = shm::align8(hdr + chunk);
    char* p = ring.reserve(n);
    if (p == nullptr) return false;
    auto* h = reinterpret_cast<shm::WireHdr*>(p);
    h->len = static_cast<std::uint32_t>(n);
    h->flags = 0;
    if (!job.head_sent) {
      auto* rec = reinterpret_cast<proto::EagerRec*>(p);
      h->type = proto::kEager;
      rec->key = job.req->key;
      rec->total = job.total;
      rec->msg_id = job.msg_id;
      rec->nbytes = chunk;
      job.head_sent = true;
    } else {
      auto* rec = reinterpret_cast<proto::FragRec*>(p);
      h->type = proto::kFrag;
      rec->msg_id = job.msg_id;
      rec->offset = job.off;
      rec->nbytes = chunk;
    }
    // gather the payload bytes from the request's host segments
    char* dstp = p + hdr;
    std::uint64_t off = job.off, left = chunk;
    for (auto& s : job.req->host) {
      if (left == 0) break;
      if (off >= s.bytes) {
        off -= s.bytes;
        continue;
      }
      std::uint64_t k = std::min(left, s.bytes - off);
      std::memcpy(dstp, s.ptr + off, k);
      dstp += k;
      left -= k;
      off = 0;
    }
    job.off += chunk;
    stats_.records_out++;
    if (job.total == 0) break;
  }
  return true;
}

bool Engine::flush_out(int dst, bool blocking_lock) {
  auto& po = *out_[dst];
  if (po.pending.load(std::memory_order_acquire) == 0) return false;
  std::unique_lock<SpinMutex> lk(po.mu, std::defer_lock);
  if (blocking_lock)
    lk.lock();
  else if (!lk.try_lock())
    return false;
  bool wrote = false;
  std::vector<std::unique_ptr<OutJob>> finished;
  while (!po.ctrl.empty()) {
    bool done = write_job(dst, po, *po.ctrl.front());
    if (!done) {
      stats_.ring_full_stalls++;
      break;
    }
    wrote = true;
    finished.push_back(std::move(po.ctrl.front()));
    po.ctrl.pop_front();
    po.pending.fetch_sub(1);
  }
  while (po.ctrl.empty() && !po.jobs.empty()) {
    OutJob& job = *po.jobs.front();
    if (job.type == proto::kDrts && job.req && dev_ && !dev_->send_gate_open(job.req)) break;
    bool done = write_job(dst, po, job);
    wrote = true;  // a partial write still advanced the stream
    if (!done) {
      stats_.ring_full_stalls++;
      break;
    }
    finished.push_back(std::move(po.jobs.front()));
    po.jobs.pop_front();
    po.pending.fetch_sub(1);
  }
  if (wrote) {
    po.ring.publish();
    std::atomic_thread_fence(std::memory_order_seq_cst);
    if (remote_[dst]) {
      links_->notify();
    } else {
      auto* ph = segs_[dst]->header();
      if (ph->sleeping.load(std::memory_order_seq_cst)) {
        ph->doorbell.fetch_add(1);
        shm::futex_wake(&ph->doorbell, 1);
      }
    }
  }
  lk.unlock();
  for (auto& j : finished) {
    if (j->complete_req_when_done && j->req && !j->completes_when_sent) complete(j->req);
  }
  return wrote;
}

// ---------------------------------------------------------------------------
// inbound (progress thread)
// ---------------------------------------------------------------------------

bool Engine::drain(int src) {
  auto& rr = in_[src];
  int n = 0;
  while (n < 64) {
    const shm::WireHdr* h = rr.peek();
    if (h == nullptr) break;
    switch (h->type) {
      case proto::kEager:
        on_eager(src, reinterpret_cast<const proto::EagerRec*>(h));
        break;
      case proto::kFrag:
        on_frag(src, reinterpret_cast<const proto::FragRec*>(h));
        break;
      case proto::kRts:
        on_rts(src, reinterpret_cast<const proto::RtsRec*>(h));
        break;
      case proto::kCts:
        on_cts(src, reinterpret_cast<const proto::CtsRec*>(h));
        break;
      case proto::kDrts:
        on_drts(src, reinterpret_cast<const proto::DrtsRec*>(h));
        break;
      case proto::kFin:
        on_fin(src, reinterpret_cast<const proto::FinRec*>(h));
        break;
      case proto::kAbort:
        on_abort(src, reinterpret_cast<const proto::AbortRec*>(h));
        break;
      default:
        std::fprintf(stderr, "commux: rank %d: corrupt record type %u from rank %d\n",
                     rank_, h->type, src);
        abort_group("corrupt record from rank " + std::to_string(src));
        return false;
    }
    rr.pop(h);
    ++n;
  }
  if (n) {
    rr.release();
    stats_.records_in += n;
  }
  return n > 0;
}

void Engine::on_eager(int src, const proto::EagerRec* rec) {
  const char* payload = reinterpret_cast<const char*>(rec + 1);
  Inflight inf;
  inf.total = rec->total;
  ReqPtr r;
  UnexpPtr u;
  bool reject_device = false;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    r = match_posted(src, rec->key);
    if (r) {
      r->source = src;
      if (r->device) {
        reject_device = true;
      } else if (rec->total > r->total) {
        // truncation: drop the bytes
      } else {
        inf.recv = r;
      }
    } else {
      u = std::make_shared<Unexpected>();
      u->src = src;
      u->key = rec->key;
      u->type = proto::kEager;
      u->total = rec->total;
      u->msg_id = rec->msg_id;
      u->data.resize(rec->total);
      unexpected_[rec->key].push_back(u);
      ++unexpected_count_;
      stats_.unexpected_msgs++;
      if (unexpected_count_ > stats_.unexpected_peak.load())
        stats_.unexpected_peak.store(unexpected_count_);
      inf.unexp = u;
    }
  }
  if (r && !inf.recv) {
    if (reject_device)
      fail(r, "commux recv: a CPU tensor was sent to a CUDA receive buffer; "
              "send and receive tensors must live on the same kind of device");
    else
      fail(r, "commux recv: message of " + std::to_string(rec->total) +
                  " bytes does not fit the " + std::to_string(r->total) + "-byte buffer");
  }
  if (inf.recv)
    scatter(inf.recv, 0, payload, rec->nbytes);
  else if (inf.unexp && rec->nbytes)
    std::memcpy(inf.unexp->data.data(), payload, rec->nbytes);
  inf.got = rec->nbytes;
  if (inf.got < inf.total) {
    std::lock_guard<SpinMutex> lk(mu_);
    inflight_[src][rec->msg_id] = inf;
    return;
  }
  // message complete
  if (inf.recv) {
    inf.recv->landed = inf.total;
    stats_.bytes_recv += static_cast<std::int64_t>(inf.total);
    complete(inf.recv);
  } else if (inf.unexp) {
    ReqPtr b;
    {
      std::lock_guard<SpinMutex> lk(mu_);
      inf.unexp->arrived = inf.total;
      inf.unexp->complete = true;
      b = inf.unexp->bound;
    }
    if (b) deliver_unexpected(b, inf.unexp);
  }
}

void Engine::on_frag(int src, const proto::FragRec* rec) {
  const char* payload = reinterpret_cast<const char*>(rec + 1);
  Inflight* inf = nullptr;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    auto it = inflight_[src].find(rec->msg_id);
    if (it != inflight_[src].end()) inf = &it->second;
  }
  if (inf == nullptr) return;  // dropped (truncated / failed receive)
  if (inf->recv) {
    if (inf->recv->state.load() == kPending) scatter(inf->recv, rec->offset, payload, rec->nbytes);
  } else if (inf->unexp) {
    std::memcpy(inf->unexp->data.data() + rec->offset, payload, rec->nbytes);
  }
  inf->got += rec->nbytes;
  if (inf->got < inf->total) return;
  Inflight done = *inf;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    inflight_[src].erase(rec->msg_id);
  }
  if (done.recv) {
    done.recv->landed = done.total;
    stats_.bytes_recv += static_cast<std::int64_t>(done.total);
    complete(done.recv);
  } else if (done.unexp) {
    ReqPtr b;
    {
      std::lock_guard<SpinMutex> lk(mu_);
      done.unexp->arrived = done.total;
      done.unexp->complete = true;
      b = done.unexp->bound;
    }
    if (b) deliver_unexpected(b, done.unexp);
  }
}

void Engine::on_rts(int src, const proto::RtsRec* rec) {
  ReqPtr r;
  bool started = false, cma = false;
  const auto* segs = reinterpret_cast<const proto::CmaSeg*>(rec + 1);
  const bool has_segs = rec->nseg > 0 && rec->nseg <= proto::kCmaSegs &&
                        rec->h.len >= sizeof(proto::RtsRec) + rec->nseg * sizeof(proto::CmaSeg);
  {
    std::lock_guard<SpinMutex> lk(mu_);
    r = match_posted(src, rec->key);
    if (!r) {
      auto u = std::make_shared<Unexpected>();
      u->src = src;
      u->key = rec->key;
      u->type = proto::kRts;
      u->total = rec->total;
      u->msg_id = rec->send_id;
      u->pid = rec->pid;
      if (has_segs)
        u->data.assign(reinterpret_cast<const char*>(segs),
                       reinterpret_cast<const char*>(segs + rec->nseg));
      unexpected_[rec->key].push_back(u);
      ++unexpected_count_;
      stats_.unexpected_msgs++;
      return;
    }
    r->source = src;
    if (!r->device && rec->total <= r->total) {
      if (has_segs && !cma_off_[src].load()) {
        cma = true;  // single-copy read, outside the lock
      } else {
        // DATA fragments carry the sender's total; record it for completion.
        start_rndv_recv(r, src, rec->send_id, rec->total);
        started = true;
      }
    }
  }
  if (cma) {
    if (cma_read(src, r, rec->pid, segs, rec->nseg, rec->total)) {
      send_fin(src, rec->send_id, 0);
      complete(r);
      return;
    }
    {
      std::lock_guard<SpinMutex> lk(mu_);
      start_rndv_recv(r, src, rec->send_id, rec->total);
    }
    started = true;
  }
  if (started) {
    flush_out(src, true);
    return;
  }
  auto job = std::make_unique<OutJob>();
  job->type = proto::kCts;
  job->head.resize(sizeof(proto::CtsRec));
  auto* c = reinterpret_cast<proto::CtsRec*>(job->head.data());
  c->send_id = rec->send_id;
  c->recv_id = 0;
  enqueue(src, std::move(job));
  flush_out(src, true);
  if (r->device)
    fail(r, "commux recv: a CPU tensor was sent to a CUDA receive buffer; "
            "send and receive tensors must live on the same kind of device");
  else
    fail(r, "commux recv: message of " + std::to_string(rec->total) +
                " bytes does not fit the " + std::to_string(r->total) + "-byte buffer");
}

void Engine::on_cts(int src, const proto::CtsRec* rec) {
  ReqPtr s;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    auto it = sends_waiting_.find(rec->send_id);
    if (it == sends_waiting_.end()) return;
    s = it->second;
    sends_waiting_.erase(it);
  }
  if (rec->recv_id == 0) {
    fail(s, "commux send: rank " + std::to_string(src) +
                " rejected the message (buffer too small or device mismatch)");
    return;
  }
  auto job = std::make_unique<OutJob>();
  job->type = proto::kFrag;
  job->req = s;
  job->msg_id = rec->recv_id | proto::kDataBit;
  job->total = s->total;
  job->head_sent = true;
  job->complete_req_when_done = true;
  enqueue(src, std::move(job));
  flush_out(src, true);
}

void Engine::on_drts(int src, const proto::DrtsRec* rec) {
  const char* blob = reinterpret_cast<const char*>(rec + 1);
  ReqPtr r;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    r = match_posted(src, rec->key);
    if (!r) {
      auto u = std::make_shared<Unexpected>();
      u->src = src;
      u->key = rec->key;
      u->type = proto::kDrts;
      u->total = rec->total;
      u->msg_id = rec->send_id;
      u->data.assign(blob, blob + rec->blob_bytes);
      unexpected_[rec->key].push_back(u);
      ++unexpected_count_;
      stats_.unexpected_msgs++;
      return;
    }
    r->source = src;
  }
  if (!r->device) {
    send_fin(src, rec->send_id, -2);
    fail(r, "commux recv: a CUDA tensor was sent to a CPU receive buffer; "
            "send and receive tensors must live on the same kind of device");
    return;
  }
  device()->on_match(r, src, rec->send_id, blob, rec->blob_bytes);
}

void Engine::on_fin(int src, const proto::FinRec* rec) {
  ReqPtr s;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    auto it = sends_waiting_.find(rec->send_id);
    if (it == sends_waiting_.end()) return;
    s = it->second;
    // the copy of a device message was enqueued: its completion FIN follows
    if (rec->status != proto::kFinLaunched) sends_waiting_.erase(it);
  }
  if (rec->status == -2) {
    fail(s, "commux send: rank " + std::to_string(src) +
                " received this CUDA tensor into a CPU buffer (device mismatch)");
    return;
  }
  if (!s->device) {  // host rendezvous finished by the receiver's single-copy read
    complete(s);
    return;
  }
  if (dev_) dev_->on_fin(s, rec->status);
}

bool Engine::cma_read(int src, const ReqPtr& r, std::int32_t pid, const proto::CmaSeg* segs, std::uint32_t nseg,
                      std::uint64_t total) {
  // Pair the sender's segments with this request's host segments: pieces of
  // (local address, remote address, bytes).
  struct Piece {
    char* local;
    std::uint64_t remote;
    std::uint64_t bytes;
  };
  std::vector<Piece> pieces;
  std::uint32_t si = 0;
  std::uint64_t soff = 0, mapped = 0;
  std::size_t li = 0;
  std::uint64_t loff = 0;
  while (mapped < total) {
    while (si < nseg && soff >= segs[si].bytes) {
      ++si;
      soff = 0;
    }
    while (li < r->host.size() && loff >= r->host[li].bytes) {
      ++li;
      loff = 0;
    }
    if (si >= nseg || li >= r->host.size()) break;
    std::uint64_t n = std::min({segs[si].bytes - soff, r->host[li].bytes - loff, total - mapped});
    pieces.push_back({static_cast<char*>(r->host[li].ptr) + loff, segs[si].addr + soff, n});
    soff += n;
    loff += n;
    mapped += n;
  }
  if (mapped != total) {
    cma_off_[src].store(true);
    return false;
  }
  // Large reads are split into equal byte ranges, one per thread: the caller
  // and up to COMMUX_COPY_THREADS helpers, each range at least kMinShare.
  constexpr std::uint64_t kMinShare = std::uint64_t{1} << 20;
  std::uint64_t shares = 1;
  if (copy_threads_ > 0 && total >= 2 * kMinShare)
    shares = std::min<std::uint64_t>(static_cast<std::uint64_t>(copy_threads_) + 1, total / kMinShare);
  std::atomic<int> failed_errno{0};
  auto copy_range = [&, pid](std::uint64_t lo, std::uint64_t hi) {
    std::uint64_t at = 0;  // byte offset of the current piece in the message
    for (const Piece& pc : pieces) {
      const std::uint64_t a = std::max(lo, at), b = std::min(hi, at + pc.bytes);
      at += pc.bytes;
      if (a >= b) continue;
      std::uint64_t off = a - (at - pc.bytes);
      std::uint64_t left = b - a;
      while (left > 0) {
        if (failed_errno.load(std::memory_order_relaxed) != 0) return;
        iovec liov{pc.local + off, static_cast<std::size_t>(left)};
        iovec riov{reinterpret_cast<void*>(pc.remote + off), static_cast<std::size_t>(left)};
        ssize_t got = ::process_vm_readv(static_cast<pid_t>(pid), &liov, 1, &riov, 1, 0);
        if (got <= 0) {
          int e = errno != 0 ? errno : EIO;
          int zero = 0;
          failed_errno.compare_exchange_strong(zero, e);
          return;
        }
        off += static_cast<std::uint64_t>(got);
        left -= static_cast<std::uint64_t>(got);
      }
    }
  };
  if (shares > 1 && copy_pool() == nullptr) shares = 1;
  if (shares <= 1) {
    copy_range(0, total);
  } else {
    std::vector<std::function<void()>> tasks;
    const std::uint64_t step = (total + shares - 1) / shares;
    for (std::uint64_t lo = 0; lo < total; lo += step)
      tasks.push_back([&copy_range, lo, hi = std::min(total, lo + step)] { copy_range(lo, hi); });
    copy_pool_->run_all(tasks);
  }
  if (failed_errno.load() != 0) {
    // refused (ptrace policy, seccomp, another host): this peer uses the
    // two-copy path from now on
    cma_off_[src].store(true);
    logf(LogLevel::Info, rank_, "single-copy reads from rank %d refused (%s); using the ring", src,
         std::strerror(failed_errno.load()));
    return false;
  }
  stats_.single_copy_msgs++;
  stats_.bytes_recv += static_cast<std::int64_t>(total);
  return true;
}

void Engine::on_abort(int src, const proto::AbortRec* rec) {
  std::string why(rec->reason, strnlen(rec->reason, sizeof(rec->reason)));
  {
    std::lock_guard<SpinMutex> lk(mu_);
    if (abort_reason_.empty())
      abort_reason_ = "rank " + std::to_string(src) + " aborted: " + why;
  }
  aborted_.store(true);
  fail_all("commux: group aborted by rank " + std::to_string(src) + ": " + why);
}

// ---------------------------------------------------------------------------
// liveness, abort
// ---------------------------------------------------------------------------

void Engine::abort_group(const std::string& why) {
  {
    std::lock_guard<SpinMutex> lk(mu_);
    if (abort_reason_.empty()) abort_reason_ = "rank " + std::to_string(rank_) + ": " + why;
  }
  bool was = aborted_.exchange(true);
  if (!was) {
    for (int p = 0; p < size_; ++p) {
      if (remote_[p] && !dead_[p].load()) {
        auto job = std::make_unique<OutJob>();
        job->type = proto::kAbort;
        job->head.resize(sizeof(proto::AbortRec));
        auto* rec = reinterpret_cast<proto::AbortRec*>(job->head.data());
        rec->code = 1;
        std::strncpy(rec->reason, why.c_str(), sizeof(rec->reason) - 1);
        enqueue(p, std::move(job));
        flush_out(p, true);
        continue;
      }
      if (!segs_[p]) continue;
      auto* h = segs_[p]->header();
      std::uint32_t z = 0;
      h->abort_code.compare_exchange_strong(z, 1);
      h->abort_rank.store(rank_);
      h->doorbell.fetch_add(1);
      shm::futex_wake(&h->doorbell, 1);
    }
  }
  fail_all("commux: group aborted: " + why);
}

void Engine::fail_all(const std::string& why) {
  std::vector<ReqPtr> victims;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    for (auto& kv : posted_)
      for (auto& r : kv.second) victims.push_back(r);
    posted_.clear();
    for (auto& kv : sends_waiting_) victims.push_back(kv.second);
    sends_waiting_.clear();
    for (auto& per : inflight_)
      for (auto& kv : per)
        if (kv.second.recv) victims.push_back(kv.second.recv);
  }
  for (auto& r : victims) fail(r, why);
  std::lock_guard<std::mutex> lk(done_mu_);
  done_cv_.notify_all();
}

void Engine::fail_peer(int p, const std::string& why) {
  if (dead_[p].exchange(true)) return;
  std::vector<ReqPtr> victims;
  {
    std::lock_guard<SpinMutex> lk(mu_);
    for (auto it = posted_.begin(); it != posted_.end();) {
      auto& dq = it->second;
      for (auto q = dq.begin(); q != dq.end();) {
        if ((*q)->peer == p) {
          victims.push_back(*q);
          q = dq.erase(q);
        } else {
          ++q;
        }
      }
      it = dq.empty() ? posted_.erase(it) : std::next(it);
    }
    for (auto it = sends_waiting_.begin(); it != sends_waiting_.end();) {
      if (it->second->peer == p) {
        victims.push_back(it->second);
        it = sends_waiting_.erase(it);
      } else {
        ++it;
      }
    }
    for (auto& kv : inflight_[p])
      if (kv.second.recv) victims.push_back(kv.second.recv);
    inflight_[p].clear();
  }
  for (auto& r : victims) fail(r, why);
  std::lock_guard<std::mutex> lk(done_mu_);
  done_cv_.notify_all();
}

void Engine::check_liveness() {
  auto* mine = my_header();
  if (mine->abort_code.load() != 0 && !aborted_.load()) {
    int who = mine->abort_rank.load();
    {
      std::lock_guard<SpinMutex> lk(mu_);
      if (abort_reason_.empty()) abort_reason_ = "rank " + std::to_string(who) + " aborted the group";
    }
    aborted_.store(true);
    fail_all("commux: group aborted by rank " + std::to_string(who));
  }
  for (int p = 0; p < size_; ++p) {
    if (p == rank_ || dead_[p].load() || remote_[p]) continue;  // TCP: the socket reports loss
    auto* h = segs_[p]->header();
    if (h->closed.load() != 0) continue;
    if (!pid_alive(static_cast<pid_t>(h->pid))) {
      fail_peer(p, "commux: peer rank " + std::to_string(p) + " (pid " +
                       std::to_string(h->pid) + ") exited without closing the group");
    }
  }
}

// ---------------------------------------------------------------------------
// progress thread
// ---------------------------------------------------------------------------

void Engine::progress_loop() {
  auto last_busy = std::chrono::steady_clock::now();
  auto* hdr = my_header();
  while (!stop_.load(std::memory_order_acquire)) {
    bool busy = false;
    for (int p = 0; p < size_; ++p) {
      try {
        busy |= drain(p);
      } catch (const std::exception& e) {
        abort_group(std::string("progress error: ") + e.what());
      }
    }
    // Jobs the posting threads left behind (ring full, or their flush lost
    // the lock race). The progress thread keeps off a peer's queue while a
    // posting thread is between its enqueue and its own flush, and takes the
    // lock without blocking: competing for it would turn every post into a
    // contended mutex hand-off (two futex calls). The loop comes back while
    // anything is pending.
    bool out_pending = false;
    for (int p = 0; p < size_; ++p) {
      auto& po = *out_[p];
      if (po.pending.load(std::memory_order_acquire) > 0) {
        if (po.posters.load(std::memory_order_acquire) == 0) busy |= flush_out(p, false);
        out_pending |= po.pending.load() > 0;
      }
    }
    int dev_inflight = 0;
    if (dev_) {
      try {
        busy |= dev_->poll();
        dev_inflight = dev_->inflight();
      } catch (const std::exception& e) {
        abort_group(std::string("device progress error: ") + e.what());
      }
    }
    hdr->heartbeat.fetch_add(1, std::memory_order_relaxed);
    auto now = std::chrono::steady_clock::now();
    if (now - last_liveness_ > std::chrono::milliseconds(100)) {
      last_liveness_ = now;
      check_liveness();
    }
    if (busy) {
      last_busy = now;
      continue;
    }
    if (out_pending || dev_inflight > 0 ||
        now - last_busy < std::chrono::microseconds(spin_us_)) {
      COMMUX_PAUSE();
      if (dev_inflight > 0 && now - last_busy > std::chrono::microseconds(spin_us_))
        std::this_thread::yield();
      continue;
    }
    // Park until a producer rings the doorbell (bounded, for liveness checks).
    hdr->sleeping.store(1, std::memory_order_seq_cst);
    std::uint32_t db = hdr->doorbell.load(std::memory_order_seq_cst);
    std::atomic_thread_fence(std::memory_order_seq_cst);
    bool any = false;
    for (int p = 0; p < size_ && !any; ++p) {
      auto* c = segs_[rank_]->ring_ctl(p);
      any = c->tail.load(std::memory_order_acquire) != c->head.load(std::memory_order_relaxed);
    }
    if (!any && !stop_.load()) {
      stats_.futex_sleeps++;
      shm::futex_wait(&hdr->doorbell, db, 20000);
    }
    hdr->sleeping.store(0, std::memory_order_seq_cst);
    last_busy = std::chrono::steady_clock::now();
  }
}

// ---------------------------------------------------------------------------
// device transport loading
// ---------------------------------------------------------------------------

DeviceTransport* Engine::device(bool create) {
  std::lock_guard<std::mutex> lk(dev_mu_);
  if (dev_ || !create) return dev_.get();
  if (released_.load()) throw std::runtime_error("commux: the process is shutting down");
  // libcommux_cuda.so sits next to this library (found through dladdr), so
  // it resolves regardless of LD_LIBRARY_PATH; it is the only commux library
  // that links the CUDA runtime (reference keeps the same split:
  // src/process_group_ucx.cpp:81-129).
  std::string path = "libcommux_cuda.so";
  Dl_info info;
  if (dladdr(reinterpret_cast<void*>(&env_int), &info) && info.dli_fname != nullptr) {
    std::string self(info.dli_fname);
    auto slash = self.find_last_of('/');
    if (slash != std::string::npos) path = self.substr(0, slash + 1) + "libcommux_cuda.so";
  }
  void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) h = dlopen("libcommux_cuda.so", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr)
    throw std::runtime_error(std::string("commux: a CUDA tensor was passed but the CUDA "
                                         "transport (libcommux_cuda.so) could not be loaded: ") +
                             dlerror());
  auto fn = reinterpret_cast<DeviceTransportFactory>(dlsym(h, "commux_create_device_transport"));
  if (fn == nullptr)
    throw std::runtime_error("commux: libcommux_cuda.so lacks commux_create_device_transport");
  dev_lib_ = h;
  dev_.reset(fn(this));
  wake_progress();
  return dev_.get();
}

}  // namespace commux
