#pragma once

// CUDA transport: host-side state of tagged CUDA p2p and the device
// collectives, implemented over CUDA IPC mappings and the sm_100a kernels in
// p2p_kernels.cu / coll_kernels.cu.
//
// Tagged p2p protocol (receiver-matched pull):
//   sender   isend: record a ready event on the current stream, export the
//            tensor's allocation through CUDA IPC (cached per allocation id),
//            and queue a DRTS record; the progress thread lets the DRTS out
//            once the ready event has completed on the device.
//   receiver irecv: record a buffer-free event on the current stream and post
//            the receive. On match (DRTS arrival or post), the pull waits
//            until the buffer-free event completed, then one launch copies
//            every ready message (strided gather over NVLink from the
//            sender's mapping, strided scatter into the receive view), stores
//            each sender's "consumed" flag with release semantics, and
//            records a done event the receive's wait() orders its stream on.
//            The progress thread sends FIN once the done event completed.
//   sender   wait(): if the peer runs on another GPU, a one-warp kernel on the
//            caller's stream waits (bounded) for the consumed flag; if the
//            peer shares this GPU, the host waits for FIN instead (no device
//            spin between processes on one GPU).
//   self     (same process): matched in the posting thread; the copy is
//            launched straight on the caller's stream after both events.
// Pull kernels never wait on anything, so their launch order on the comm
// stream cannot deadlock, whatever the matching order.

#include <ATen/ATen.h>
#include <cuda_runtime.h>

#include <atomic>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../engine/engine.hpp"
#include "cuda_common.hpp"

namespace commux {
namespace cuda {

#define CMX_CUDA(expr)                                                                       \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("commux CUDA error: ") + cudaGetErrorString(_e) + \
                               " (" #expr ")");                                              \
  } while (0)

class DevCtx;

// Select `dev` without throwing; false once the CUDA context is gone (process
// teardown), in which case destructors skip their CUDA cleanup.
bool select_device_quiet(int dev);

// Pool of timing-free events of one device. Shared by every EventRef, so an
// event can outlive the transport (a Work collected after the group was
// destroyed still returns its event safely).
struct EventPool {
  explicit EventPool(int d) : dev(d) {}
  ~EventPool();
  int dev;
  std::mutex mu;
  std::vector<cudaEvent_t> free;
};

// Event returned to its pool when the last holder drops it.
struct EventRef {
  cudaEvent_t ev = nullptr;
  std::shared_ptr<EventPool> pool;
  ~EventRef();
};
using EventPtr = std::shared_ptr<EventRef>;

// Device buffers from cudaMalloc, which CUDA IPC can always export, for
// sends whose own memory cannot be exported (the caching allocator's
// expandable segments are cuMemCreate mappings). Buffers are kept for reuse,
// so a receiver maps each of them once. Shared with the tensors it lends out:
// a buffer returns here when the last tensor over it dies, after the transport
// may be gone.
struct ExportPool {
  explicit ExportPool(int d) : dev(d) {}
  ~ExportPool();
  int dev;
  std::mutex mu;
  std::multimap<std::size_t, void*> free;  // by capacity
  std::int64_t bytes = 0;                  // allocated in total
};

class DevCtx {
 public:
  explicit DevCtx(int dev);
  ~DevCtx();
  int dev;
  unsigned char uuid[16];
  int sm_count = 148;
  cudaStream_t comm = nullptr;     // pulls launched by the progress thread
  std::uint64_t* mbox = nullptr;   // consumed flags, one per send slot
  cudaIpcMemHandle_t mbox_handle;
  std::uint64_t mbox_id = 0;
  std::uint64_t mbox_base = 0;
  std::atomic<std::uint64_t> next_value{0};
  std::atomic<std::uint64_t> next_plan_slot{0};  // persistent-plan flags (second half of mbox)
  unsigned long long* status_h = nullptr;  // host-mapped error block (4 x u64)
  unsigned long long* status_d = nullptr;

  EventPtr event();                          // from the pool
  // An uninitialised contiguous tensor in an exportable pool buffer.
  at::Tensor exportable_empty(at::IntArrayRef sizes, at::ScalarType dtype);
  std::shared_ptr<ExportPool> export_pool;
  void release(cudaEvent_t e);
  std::uint32_t* scratch(cudaStream_t s);    // zeroed per-stream counters
  // first of `n` consecutive counter slots (mod kCounterSlots) on stream s
  std::uint32_t take_slots(cudaStream_t s, std::uint32_t n);

 private:
  std::mutex mu_;
  std::shared_ptr<EventPool> pool_;
  std::unordered_map<cudaStream_t, std::uint32_t*> scratch_;
  std::unordered_map<cudaStream_t, std::uint32_t> next_slot_;
};

struct SendState {
  int device = -1;
  cudaStream_t stream = nullptr;
  EventPtr ready;             // data produced
  bool local = false;
  bool device_wait = false;   // wait() polls the consumed flag on the GPU
  std::uint64_t slot = 0, value = 0;
  std::atomic<bool> fin{false};
  // device_wait sends: the receiver enqueued the copy that will store the
  // consumed flag (its FIN with proto::kFinLaunched); a wait kernel is only
  // launched after that, so no stream ever spins on a copy that is not yet
  // enqueued (see wait_sends_on_stream)
  std::atomic<bool> launched{false};
  std::atomic<std::int64_t> fin_status{0};  // an error FIN's status
  EventPtr local_done;        // self-send: copy finished (same process)
  std::vector<at::Tensor> staged;  // contiguous copies made for the wire
};

struct RecvState {
  int device = -1;
  cudaStream_t stream = nullptr;
  EventPtr ready;             // receive buffer free
  EventPtr done;              // pull finished
  std::vector<std::pair<at::Tensor, at::Tensor>> unpack;  // (temp, view)
};

struct PendingPull {
  ReqPtr r;
  int src = -1;
  std::uint64_t send_id = 0;
  bool sender_waits = false;  // the sender waits on the device flag (a FIN at launch too)
  DevCtx* ctx = nullptr;
  std::vector<PullDesc> descs;
  std::uint32_t msg_chunks = 0;
};

class CollImpl;

class CudaTransport final : public DeviceTransport {
 public:
  explicit CudaTransport(Engine* e);
  ~CudaTransport() override;

  void prepare_send(const ReqPtr& s, int dst, std::vector<char>& blob, bool* gate,
                    bool* complete_on_post) override;
  bool send_gate_open(const ReqPtr& s) override;
  void prepare_recv(const ReqPtr& r) override;
  void on_match(const ReqPtr& r, int src, std::uint64_t send_id, const char* blob,
                std::size_t len) override;
  void on_fin(const ReqPtr& s, std::int64_t status) override;
  bool poll() override;
  void stream_wait(const ReqPtr& r) override;
  bool query(const ReqPtr& r) override;
  std::string device_error() override;
  int inflight() override;
  std::vector<std::pair<std::string, std::int64_t>> stats() override;
  void shutdown() override;
  void begin_batch() override;
  void end_batch() override;

  DevCollPtr allreduce(std::vector<at::Tensor>& ts, RedOp op) override;
  DevCollPtr reduce(std::vector<at::Tensor>& ts, RedOp op, int root) override;
  DevCollPtr broadcast(std::vector<at::Tensor>& ts, int root) override;
  DevCollPtr allgather(at::Tensor& out, const at::Tensor& in) override;
  DevCollPtr reduce_scatter(at::Tensor& out, const at::Tensor& in, RedOp op) override;
  DevCollPtr barrier() override;
  bool device_collectives(int dev) override;
  bool collectives_ready() override;
  DevicePlanPtr create_plan(const std::vector<at::Tensor>& recv_t, const std::vector<int>& recv_peer,
                            const std::vector<int>& recv_tag, const std::vector<at::Tensor>& send_t,
                            const std::vector<int>& send_peer, const std::vector<int>& send_tag) override;
  // pull launch(es) of prebuilt per-message descriptors on `stream` (plans)
  // descriptors of one message from its wire description (plans)
  std::vector<PullDesc> plan_descs(const char* wire, std::size_t len, int src, bool local,
                                   const at::Tensor& dst, DevCtx* c);
  void stream_wait_all(const std::vector<ReqPtr>& rs) override;

  // shared with the collectives
  Engine* engine() { return eng_; }
  DevCtx* ctx(int dev);
  // Maps rank src's allocation `buffer_id` (cached per (src, buffer_id)).
  // `base`/`size` give its address range in the sender (size 0: unknown, as
  // for the mailboxes): an older mapping of the same sender whose range
  // overlaps it belongs to an allocation the sender has freed, and is closed.
  void* ipc_open(int src, std::uint64_t buffer_id, std::uint64_t base, std::uint64_t size,
                 const cudaIpcMemHandle_t& h, DevCtx* c);
  // false when CUDA IPC cannot export the allocation holding `ptr`
  bool exportable(const void* ptr);
  // `t` itself when the receiver can map it, else a copy (enqueued on the
  // current stream) in an exportable pool buffer
  at::Tensor export_or_stage(const at::Tensor& t, DevCtx* c);
  void ipc_export(const void* ptr, std::uint64_t* buffer_id, std::uint64_t* base,
                  std::uint64_t* size, cudaIpcMemHandle_t* handle);
  std::uint64_t device_timeout_ns() const { return timeout_ns_; }
  int pull_ctas(DevCtx* c) const;
  std::atomic<std::int64_t> kernel_launches{0};
  // which path the messages took (tests assert the intended one ran):
  // persistent-plan messages to a rank on another GPU (device flags) or on
  // this same GPU (host-gated), and plan starts
  std::atomic<std::int64_t> plan_device_msgs{0}, plan_shared_msgs{0}, plan_starts{0};

 private:
  void publish_uuid(DevCtx* c);
  void build_descs(const ReqPtr& r, const char* wire, std::size_t len, bool local,
                   PendingPull& pp);
  void launch_batch(DevCtx* c, std::vector<PendingPull>& pulls, cudaStream_t stream);
  void wait_sends_on_stream(const std::vector<ReqPtr>& sends);
  void wait_pull_launched(SendState& st);

  Engine* eng_;
  std::uint64_t timeout_ns_;
  std::mutex ctx_mu_;
  std::map<int, std::unique_ptr<DevCtx>> ctx_;
  bool uuid_published_ = false;

  SpinMutex ipc_mu_;  // shared by posting threads and the progress thread
  std::unordered_map<std::uint64_t, cudaIpcMemHandle_t> exported_;  // by buffer id
  struct Opened {
    void* ptr = nullptr;
    std::uint64_t base = 0, size = 0;  // the sender's address range (size 0: unknown)
  };
  std::map<std::pair<int, std::uint64_t>, Opened> opened_;
  std::unordered_set<std::uint64_t> unexportable_;  // allocation ids IPC refused

  std::mutex local_mu_;
  std::unordered_map<std::uint64_t, ReqPtr> local_sends_;  // self-sends awaiting a match

  SpinMutex pend_mu_;  // shared by posting threads and the progress thread
  std::vector<PendingPull> pending_;
  struct Flight {
    EventPtr done;
    std::vector<std::pair<int, std::uint64_t>> fins;  // FINs owed at completion
    std::vector<ReqPtr> reqs;
    int pulls = 0;  // counted in inflight_
  };
  std::deque<Flight> flights_;
  std::atomic<int> inflight_{0};

  // group window batching (self-sends launch at end_batch)
  SpinMutex batch_mu_;  // shared by posting threads and the progress thread
  int batch_depth_ = 0;
  std::map<int, EventPtr> batch_event_;  // one ready event per device per window
  std::vector<std::pair<PendingPull, cudaStream_t>> batch_local_;
  std::vector<ReqPtr> batch_local_sends_;

  std::string dev_error_;
  std::unique_ptr<CollImpl> coll_;

  std::atomic<std::int64_t> st_pulls_{0}, st_pull_bytes_{0}, st_wait_kernels_{0}, st_fins_{0},
      st_ipc_opens_{0}, st_ipc_exports_{0}, st_staged_{0}, st_ipc_closes_{0}, st_export_staged_{0};
  // sends to another process: completed by a device-side wait on this
  // stream (receiver on another GPU) or by the receiver's host FIN (same
  // GPU); pulls from a sender on another GPU or on this same GPU
  std::atomic<std::int64_t> st_sends_device_{0}, st_sends_host_{0}, st_pulls_peer_gpu_{0}, st_pulls_same_gpu_{0};
};

}  // namespace cuda
}  // namespace commux
