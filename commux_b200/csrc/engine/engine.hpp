#pragma once

// Host tag-matching engine.
//
// MPI matching semantics on a 64-bit key (the reference gets them from UCX's
// tag API, reference: src/process_group_ucx.cpp:474-526 and :696-732):
//   * a receive posted for (src, key) takes the oldest unmatched message from
//     src with that key; any-source receives (src == -1) take the oldest
//     message with that key from any rank;
//   * messages from one sender with one key are matched in send order (the
//     rings are FIFO per ordered pair);
//   * the receive that was posted first wins when several match.
//
// Posted receives and unexpected messages are kept in hash maps keyed by the
// 48-bit key (tag without the rank field) with FIFO deques per key. A single
// progress thread drains the inbound rings, matches, copies host payloads and
// streams rendezvous data; user threads post and match under `mu_` and never
// copy data that the progress thread may still be writing.

#include <ATen/core/Tensor.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <functional>
#include <list>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <unordered_map>
#include <vector>

#include "copy_pool.hpp"
#include "protocol.hpp"
#include "shm.hpp"
#include "tcp.hpp"

namespace commux {

using tag_t = std::uint64_t;

enum ReqState : int { kPending = 0, kDone = 1, kFailed = 2 };
enum class ReqKind : std::uint8_t { Send, Recv };

struct HostSeg {
  char* ptr;
  std::uint64_t bytes;
};

class Engine;
class DeviceTransport;

// One tagged message in flight (one per tensor, or one per tensor vector on
// the coalesced IOV path).
struct Request {
  ReqKind kind = ReqKind::Send;
  std::atomic<int> state{kPending};
  std::string error;      // set before state becomes kFailed
  int peer = -1;          // send: dst; recv: src (-1: any source)
  tag_t key = 0;          // tag with the rank field cleared
  std::uint64_t id = 0;   // engine-unique (send id / recv id)
  bool device = false;    // CUDA tensors
  std::vector<at::Tensor> tensors;  // data (kept alive until completion)
  std::vector<HostSeg> host;        // host byte segments, in order
  std::uint64_t total = 0;          // bytes
  std::atomic<int> source{-1};      // recv: rank the message came from (read by waiters)
  std::uint64_t landed = 0;         // recv: payload bytes written
  std::shared_ptr<void> dev;        // device-transport state
  std::chrono::steady_clock::time_point posted_at;
};
using ReqPtr = std::shared_ptr<Request>;

// Unexpected (arrived, not yet matched) message.
struct Unexpected {
  int src = -1;
  tag_t key = 0;
  std::uint16_t type = 0;     // proto::kEager / kRts / kDrts
  std::uint64_t total = 0;
  std::uint64_t msg_id = 0;   // sender's id
  std::vector<char> data;     // eager payload / device blob / single-copy segments
  std::int32_t pid = 0;       // rendezvous: sender pid for a single-copy read
  std::uint64_t arrived = 0;  // eager bytes landed
  bool complete = false;      // all eager bytes landed
  ReqPtr bound;               // recv matched while bytes were still landing
};
using UnexpPtr = std::shared_ptr<Unexpected>;

// Engine counters (exported through ProcessGroupUCX::stats()).
struct Stats {
  std::atomic<std::int64_t> sends{0}, recvs{0}, bytes_sent{0}, bytes_recv{0};
  std::atomic<std::int64_t> eager_msgs{0}, rndv_msgs{0}, device_msgs{0};
  std::atomic<std::int64_t> unexpected_msgs{0}, unexpected_peak{0};
  std::atomic<std::int64_t> ring_full_stalls{0}, futex_sleeps{0};
  std::atomic<std::int64_t> records_in{0}, records_out{0};
  std::atomic<std::int64_t> host_copies{0};
  std::atomic<std::int64_t> single_copy_msgs{0};  // host rendezvous read with process_vm_readv
  std::atomic<std::int64_t> faults_injected{0};
};

// Outbound record stream to one peer.
struct OutJob {
  std::uint16_t type = 0;
  std::vector<char> head;         // fixed record (control) or first header
  ReqPtr req;                     // payload source (EAGER / DATA)
  std::uint64_t msg_id = 0;       // id carried by FRAG records
  std::uint64_t off = 0;          // next payload byte to send
  std::uint64_t total = 0;        // payload bytes
  bool head_sent = false;
  bool complete_req_when_done = false;
  bool completes_when_sent = false;  // TCP pump completes req (indirect records)
};

// A mutex for short critical sections shared by a posting thread and the
// progress thread: a contended lock spins briefly (the holder is usually
// about to release it) before it parks in the kernel, which saves the futex
// wait/wake pair of a plain std::mutex hand-off.
class SpinMutex {
 public:
  void lock() {
    for (int i = 0; i < 256; ++i) {
      if (m_.try_lock()) return;
#if defined(__x86_64__) || defined(__i386__)
      __builtin_ia32_pause();
#else
      std::this_thread::yield();
#endif
    }
    m_.lock();
  }
  bool try_lock() { return m_.try_lock(); }
  void unlock() { m_.unlock(); }

 private:
  std::mutex m_;
};

struct PeerOut {
  SpinMutex mu;                   // serialises writers of this ring
  shm::RingWriter ring;
  std::deque<std::unique_ptr<OutJob>> ctrl;  // FIN/CTS/ABORT: never wait
  std::deque<std::unique_ptr<OutJob>> jobs;  // matched messages, FIFO
  std::atomic<int> pending{0};
  std::atomic<int> posters{0};    // posting threads between enqueue and their flush
};

// Fault injection (host side only): COMMUX_FAULT
//   drop:<rank>:<tag>   rank silently drops sends carrying user tag <tag>
//   kill:<rank>:<n>     rank exits (code 77) when it posts its n-th operation
//   delay:<ms>          every outbound record is delayed by <ms>
struct FaultSpec {
  int drop_rank = -1;
  std::int64_t drop_tag = -1;
  int kill_rank = -1;
  std::int64_t kill_after = -1;
  int delay_ms = 0;
  static FaultSpec from_env();
};

class Engine {
 public:
  Engine(c10::intrusive_ptr<c10d::Store> store, int rank, int size,
         std::chrono::milliseconds timeout);
  ~Engine();

  int rank() const { return rank_; }
  int size() const { return size_; }
  std::chrono::milliseconds timeout() const { return timeout_; }
  void set_timeout(std::chrono::milliseconds t) { timeout_ = t; }
  c10d::Store& store() { return *store_; }
  // Store key prefix unique to this group ("commux/<generation>/").
  const std::string& store_prefix() const { return prefix_; }

  // Post a send / receive of the given tensors. `iov` sends the vector as one
  // message (COMMUX_COALESCE); otherwise the caller passes one tensor.
  ReqPtr post_send(std::vector<at::Tensor> tensors, int dst, tag_t tag);
  ReqPtr post_recv(std::vector<at::Tensor> tensors, int src, tag_t tag);

  // Block until the request leaves kPending (host part); throws on failure or
  // timeout (timeout <= 0 uses the engine timeout).
  void wait(const ReqPtr& r, std::chrono::milliseconds timeout);
  bool test(const ReqPtr& r) const {
    return r->state.load(std::memory_order_acquire) != kPending;
  }

  // Request completion (progress thread or device transport).
  void complete(const ReqPtr& r);
  void fail(const ReqPtr& r, const std::string& why);

  // Control records for the device transport.
  void send_fin(int dst, std::uint64_t send_id, std::int64_t status);
  void wake_progress();

  // Aborts the whole group: every pending request fails and peers are told.
  void abort_group(const std::string& why);
  bool aborted() const { return aborted_.load(); }
  bool peer_dead(int p) const { return dead_[p].load(); }
  std::string failure_reason() const;

  DeviceTransport* device(bool create = true);
  Stats& stats() { return stats_; }

  // Drop every CUDA resource and every tensor reference this engine holds
  // while the CUDA context is still alive (Python calls release_all() from
  // an atexit hook). Afterwards the engine refuses new operations. Without
  // this, a group kept alive until interpreter exit would free CUDA memory
  // after the runtime tore its context down.
  void release_for_exit();
  static void release_all();
  const Stats& stats() const { return stats_; }
  // current sizes of the engine's queues and tables (all zero when no
  // message is in flight): posted receives, unexpected messages, messages
  // partly received, sends waiting for their FIN, sends the TCP pump has
  // still to send
  std::vector<std::pair<std::string, std::int64_t>> gauges();

  // Internal fault injection hook (counts operations for kill:<rank>:<n>).
  void count_op();

  // nullptr for a peer reached over TCP (another host)
  const shm::SegHeader* peer_header(int p) const { return segs_[p] ? segs_[p]->header() : nullptr; }
  // Peer p is reached over TCP (another host, or COMMUX_TRANSPORT=tcp).
  bool remote(int p) const { return !remote_.empty() && remote_[p]; }
  bool any_remote() const { return any_remote_; }
  shm::SegHeader* my_header() const { return segs_[rank_]->header(); }

 private:
  void bootstrap();
  void store_barrier(const std::string& key);
  void progress_loop();
  bool drain(int src);
  bool flush_out(int dst, bool blocking_lock);
  bool write_job(int dst, PeerOut& po, OutJob& job);
  void enqueue(int dst, std::unique_ptr<OutJob> job);
  // enqueue + flush from a posting thread (see progress_loop)
  void post_job(int dst, std::unique_ptr<OutJob> job);
  // the TCP pump has sent the last record of request `id` (indirect records)
  void on_pump_sent(std::uint64_t id);

 public:
  // fn(lo, hi) over [0, n) in at most 1 + COMMUX_COPY_THREADS ranges of at
  // least `grain`, on this thread and the copy helpers; returns when all are
  // done. Serial when the helpers are off or unavailable.
  void parallel_ranges(std::int64_t n, std::int64_t grain, const std::function<void(std::int64_t, std::int64_t)>& fn);

 private:
  CopyPool* copy_pool();  // created on first use; nullptr when unavailable
  void check_liveness();
  void fail_peer(int p, const std::string& why);
  void fail_all(const std::string& why);

  // inbound handlers (progress thread)
  void on_eager(int src, const proto::EagerRec* rec);
  void on_frag(int src, const proto::FragRec* rec);
  void on_rts(int src, const proto::RtsRec* rec);
  void on_cts(int src, const proto::CtsRec* rec);
  void on_drts(int src, const proto::DrtsRec* rec);
  void on_fin(int src, const proto::FinRec* rec);
  void on_abort(int src, const proto::AbortRec* rec);
  // Single-copy rendezvous: read the sender's segments straight into r's
  // host buffers; false (and the peer marked CTS-only) when the kernel
  // refuses the cross-process read.
  bool cma_read(int src, const ReqPtr& r, std::int32_t pid, const proto::CmaSeg* segs, std::uint32_t nseg,
                std::uint64_t total);

  // matching helpers (mu_ held)
  ReqPtr match_posted(int src, tag_t key);
  UnexpPtr match_unexpected(int src, tag_t key);
  void start_rndv_recv(const ReqPtr& r, int src, std::uint64_t send_id,
                       std::uint64_t total);
  void deliver_unexpected(const ReqPtr& r, const UnexpPtr& u);
  void scatter(const ReqPtr& r, std::uint64_t off, const char* data,
               std::uint64_t n);

  c10::intrusive_ptr<c10d::Store> store_;
  std::string prefix_;
  int rank_;
  int size_;
  std::chrono::milliseconds timeout_;
  std::uint64_t eager_limit_;
  std::uint64_t frag_bytes_;
  int spin_us_;
  int spin_wait_us_ = 100;  // COMMUX_WAIT_SPIN_US: spin of a waiting thread before it sleeps
  std::mutex pump_mu_;                                      // guards pump_waiting_
  std::unordered_map<std::uint64_t, ReqPtr> pump_waiting_;  // sends the TCP pump completes
  int wait_poll_ms_;
  FaultSpec fault_;
  std::atomic<std::int64_t> op_count_{0};

  std::vector<std::unique_ptr<shm::Segment>> segs_;  // [rank] own, others mapped (null: TCP peer)
  std::vector<bool> remote_;                         // remote_[p]: TCP peer
  std::unique_ptr<std::atomic<bool>[]> cma_off_;     // single-copy refused for peer p
  bool cma_enabled_ = true;                          // COMMUX_CMA
  int copy_threads_ = 2;                             // COMMUX_COPY_THREADS: helpers of large reads
  std::unique_ptr<CopyPool> copy_pool_;              // created on the first large read
  std::once_flag copy_pool_once_;
  bool any_remote_ = false;
  std::unique_ptr<tcp::Links> links_;                // TCP peers (null when none)
  std::vector<shm::RingReader> in_;                  // in_[src]
  std::vector<std::unique_ptr<PeerOut>> out_;        // out_[dst]

  // matching state
  mutable SpinMutex mu_;
  std::unordered_map<tag_t, std::deque<ReqPtr>> posted_;
  std::unordered_map<tag_t, std::deque<UnexpPtr>> unexpected_;
  std::int64_t unexpected_count_ = 0;
  std::unordered_map<std::uint64_t, ReqPtr> sends_waiting_;  // by send id
  std::atomic<std::uint64_t> next_id_{1};

  // inbound fragment streams (progress thread only)
  struct Inflight {
    ReqPtr recv;     // bound receive, or
    UnexpPtr unexp;  // unexpected buffer
    std::uint64_t total = 0;
    std::uint64_t got = 0;
  };
  std::vector<std::unordered_map<std::uint64_t, Inflight>> inflight_;

  // completion signalling
  mutable std::mutex done_mu_;
  std::condition_variable done_cv_;
  std::atomic<int> waiters_{0};

  // liveness
  std::vector<std::atomic<bool>> dead_;
  std::atomic<bool> aborted_{false};
  std::string abort_reason_;
  std::chrono::steady_clock::time_point last_liveness_;

  std::unique_ptr<DeviceTransport> dev_;
  std::mutex dev_mu_;
  void* dev_lib_ = nullptr;

  std::atomic<bool> stop_{false};
  std::atomic<bool> released_{false};
  std::thread progress_;
  Stats stats_;
};

// Reduction operators of the collectives (ReduceOp subset this backend runs).
enum class RedOp : int { Sum = 0, Prod = 1, Min = 2, Max = 3, Avg = 4 };

// Completion handle of a collective enqueued on a CUDA stream.
class DevCollResult {
 public:
  virtual ~DevCollResult() = default;
  virtual void stream_wait() = 0;  // caller's current stream waits for it
  virtual bool query() = 0;        // non-blocking
  virtual void host_wait() = 0;    // block the host until it is done
  virtual std::string error() = 0;  // device-side failure, "" if none
  // Complete `fut` with `value` so that consumers sync on the collective's
  // stream (CUDA-aware c10 Future semantics).
  virtual void mark_future(void* fut, void* value) = 0;
};
using DevCollPtr = std::shared_ptr<DevCollResult>;

// A persistent set of tagged CUDA messages, matched once (the analogue of
// MPI_Send_init/MPI_Recv_init + MPI_Startall). Every start() enqueues one
// exchange of the same buffers on the caller's current stream: no host
// matching, no host round trip, a few launches.
class DevicePlan {
 public:
  virtual ~DevicePlan() = default;
  virtual void start() = 0;
  virtual std::vector<std::pair<std::string, std::int64_t>> info() = 0;
  // Caps the CTAs of the plan's launches (0: the default grid). A smaller
  // grid leaves SMs to kernels that run beside the exchange.
  virtual void set_max_ctas(int ctas) = 0;
};
using DevicePlanPtr = std::shared_ptr<DevicePlan>;

// Device transport interface, implemented by libcommux_cuda.so (loaded on the
// first CUDA tensor; the host engine has no link-time CUDA dependency).
class DeviceTransport {
 public:
  virtual ~DeviceTransport() = default;
  // Sender: prepare a CUDA send; fills the descriptor blob carried by DRTS.
  // Sets *gate when the DRTS may only go out once send_gate_open() is true,
  // and *complete_on_post when the send's host part is complete as soon as
  // the DRTS is written (its device completion is then awaited on a stream).
  // For dst == own rank the blob never leaves the process.
  virtual void prepare_send(const ReqPtr& s, int dst, std::vector<char>& blob,
                            bool* gate, bool* complete_on_post) = 0;
  virtual bool send_gate_open(const ReqPtr& s) = 0;
  // Receiver: record the point on the consumer stream where the buffer may
  // be overwritten.
  virtual void prepare_recv(const ReqPtr& r) = 0;
  // A DRTS from `src` matched receive `r` (called with the engine lock
  // released). Arranges the pull; completes `r` (host part) once the copy is
  // enqueued on the device.
  virtual void on_match(const ReqPtr& r, int src, std::uint64_t send_id,
                        const char* blob, std::size_t len) = 0;
  // The receiver reported completion (FIN) of send `s`.
  virtual void on_fin(const ReqPtr& s, std::int64_t status) = 0;
  // Progress-thread hook: launch batched pulls, poll events, send FINs.
  // Returns true when it did work (keeps the progress thread spinning).
  virtual bool poll() = 0;
  // Order the caller's current stream after the request's device work.
  virtual void stream_wait(const ReqPtr& r) = 0;
  // Same for a set of requests (one wait launch covers many sends).
  virtual void stream_wait_all(const std::vector<ReqPtr>& rs) = 0;
  // Non-blocking: has the device work of `r` finished?
  virtual bool query(const ReqPtr& r) = 0;
  // Device-side error (timeout of a flag wait, ...) recorded so far.
  virtual std::string device_error() = 0;
  // Number of in-flight device transfers (keeps the progress thread awake).
  virtual int inflight() = 0;
  virtual std::vector<std::pair<std::string, std::int64_t>> stats() = 0;
  virtual void shutdown() = 0;

  // Batching hint: sends posted between begin_batch() and end_batch() (one
  // group window) share one readiness signal and one launch where possible.
  virtual void begin_batch() = 0;
  virtual void end_batch() = 0;

  // Collectives on CUDA tensors (all ranks call them in the same order). The
  // work is stream-ordered after the caller's current stream.
  virtual DevCollPtr allreduce(std::vector<at::Tensor>& ts, RedOp op) = 0;
  virtual DevCollPtr reduce(std::vector<at::Tensor>& ts, RedOp op, int root) = 0;
  virtual DevCollPtr broadcast(std::vector<at::Tensor>& ts, int root) = 0;
  virtual DevCollPtr allgather(at::Tensor& out, const at::Tensor& in) = 0;
  virtual DevCollPtr reduce_scatter(at::Tensor& out, const at::Tensor& in, RedOp op) = 0;
  virtual DevCollPtr barrier() = 0;
  // True if the device collectives can run on `dev` (every rank drives its
  // own GPU). False when ranks share a GPU: kernels of different processes
  // must never wait on each other on one GPU, so the caller stages through
  // the host collectives instead. The first call is collective (workspace
  // exchange): all ranks make it in the same order.
  virtual bool device_collectives(int dev) = 0;
  // True once the device collectives are set up on this group and run on
  // the device (the same on every rank: the set-up is collective).
  virtual bool collectives_ready() = 0;

  // Persistent plan over the given receives and sends (matched by (peer,
  // tag) in FIFO order, like the one-shot path). Collective among the ranks
  // the plan talks to: each must create its side, in the same order.
  virtual DevicePlanPtr create_plan(const std::vector<at::Tensor>& recv_t,
                                    const std::vector<int>& recv_peer,
                                    const std::vector<int>& recv_tag,
                                    const std::vector<at::Tensor>& send_t,
                                    const std::vector<int>& send_peer,
                                    const std::vector<int>& send_tag) = 0;
};

using DeviceTransportFactory = DeviceTransport* (*)(Engine*);

// Environment helpers shared by the native libraries.
std::int64_t env_int(const char* name, std::int64_t dflt);
bool env_flag(const char* name);

}  // namespace commux
