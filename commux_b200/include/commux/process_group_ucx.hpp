#pragma once

// commux (B200-native): a PyTorch c10d::Backend with MPI-style (sender, tag)
// matched point-to-point messaging plus collectives, for CPU and CUDA tensors.
//
// Public surface kept identical to the reference backend
// (reference: include/commux/process_group_ucx.hpp:30-80): the class is still
// named ProcessGroupUCX, getBackendName() is "ucx", and make_ucp_tag /
// kTagMaskAnySource keep their bit layout. Nothing here includes UCX: the
// transport underneath is this library's own engine (POSIX shared-memory rings
// for host bytes, CUDA IPC + sm_100a kernels over NVLink for device bytes).

#include <ATen/core/Tensor.h>
#include <c10/util/intrusive_ptr.h>

#include <chrono>
#include <cstdint>
#include <memory>
#include <string>
#include <torch/csrc/distributed/c10d/Backend.hpp>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <torch/csrc/distributed/c10d/Types.hpp>
#include <torch/csrc/distributed/c10d/Work.hpp>
#include <vector>

namespace commux {

// 64-bit match key (same layout as reference process_group_ucx.hpp:30-40):
//
//   bits [63:48] (16)  sender rank
//   bits [47:33] (15)  sub-index (tensor position within a std::vector arg)
//   bit  [32]          collective namespace (keeps collective traffic apart
//                      from user p2p tags)
//   bits [31:0]  (32)  user tag
//
// Out-of-range values are masked (rank & 0xFFFF, sub & 0x7FFF).
using tag_t = std::uint64_t;
tag_t make_ucp_tag(int sender_rank, std::uint32_t user_tag,
                   std::uint32_t sub_index, bool collective);

// Mask that wildcards the sender-rank field (any-source receive).
constexpr tag_t kTagMaskAnySource = 0x0000FFFFFFFFFFFFull;

class Engine;       // host tag-matching engine (opaque)
class CollEngine;   // collective algorithms (opaque)
struct GroupWindow;  // coalescing-window state (opaque)
struct Request;      // one message in flight (opaque)
class DevicePlan;    // persistent CUDA message plan (opaque)

class ProcessGroupUCX : public c10d::Backend {
 public:
  // `timeout` bounds every blocking wait of this backend (Work::wait without
  // an explicit timeout, bootstrap, device-side flag waits). Zero means the
  // c10d default (30 min) for host waits and COMMUX_DEVICE_TIMEOUT_MS for
  // device waits.
  ProcessGroupUCX(c10::intrusive_ptr<c10d::Store> store, int rank, int size,
                  std::chrono::milliseconds timeout =
                      std::chrono::milliseconds(0));
  ~ProcessGroupUCX() override;

  const std::string getBackendName() const override { return "ucx"; }

  // --- point-to-point (tagged) -------------------------------------------
  c10::intrusive_ptr<c10d::Work> send(std::vector<at::Tensor>& tensors,
                                      int dstRank, int tag) override;
  c10::intrusive_ptr<c10d::Work> recv(std::vector<at::Tensor>& tensors,
                                      int srcRank, int tag) override;
  c10::intrusive_ptr<c10d::Work> recvAnysource(std::vector<at::Tensor>& tensors,
                                               int tag) override;

  // --- collectives ---------------------------------------------------------
  c10::intrusive_ptr<c10d::Work> allreduce(
      std::vector<at::Tensor>& tensors,
      const c10d::AllreduceOptions& opts = c10d::AllreduceOptions()) override;
  c10::intrusive_ptr<c10d::Work> allreduce_coalesced(
      std::vector<at::Tensor>& tensors,
      const c10d::AllreduceCoalescedOptions& opts =
          c10d::AllreduceCoalescedOptions()) override;
  c10::intrusive_ptr<c10d::Work> reduce(
      std::vector<at::Tensor>& tensors,
      const c10d::ReduceOptions& opts = c10d::ReduceOptions()) override;
  c10::intrusive_ptr<c10d::Work> broadcast(
      std::vector<at::Tensor>& tensors,
      const c10d::BroadcastOptions& opts = c10d::BroadcastOptions()) override;
  c10::intrusive_ptr<c10d::Work> barrier(
      const c10d::BarrierOptions& opts = c10d::BarrierOptions()) override;
  // allgather family: needed by torch DDP (parameter-shape verification and
  // object collectives); absent from the reference backend.
  c10::intrusive_ptr<c10d::Work> allgather(
      std::vector<std::vector<at::Tensor>>& outputTensors,
      std::vector<at::Tensor>& inputTensors,
      const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> _allgather_base(
      at::Tensor& outputBuffer, at::Tensor& inputBuffer,
      const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> allgather_into_tensor_coalesced(
      std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
      const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> gather(
      std::vector<std::vector<at::Tensor>>& outputTensors,
      std::vector<at::Tensor>& inputTensors,
      const c10d::GatherOptions& opts = c10d::GatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> scatter(
      std::vector<at::Tensor>& outputTensors,
      std::vector<std::vector<at::Tensor>>& inputTensors,
      const c10d::ScatterOptions& opts = c10d::ScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> reduce_scatter(
      std::vector<at::Tensor>& outputTensors,
      std::vector<std::vector<at::Tensor>>& inputTensors,
      const c10d::ReduceScatterOptions& opts =
          c10d::ReduceScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> _reduce_scatter_base(
      at::Tensor& outputBuffer, at::Tensor& inputBuffer,
      const c10d::ReduceScatterOptions& opts =
          c10d::ReduceScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> alltoall_base(
      at::Tensor& outputBuffer, at::Tensor& inputBuffer,
      std::vector<int64_t>& outputSplitSizes,
      std::vector<int64_t>& inputSplitSizes,
      const c10d::AllToAllOptions& opts = c10d::AllToAllOptions()) override;
  // list form: outputTensors[p] receives rank p's inputTensors[me]
  c10::intrusive_ptr<c10d::Work> alltoall(
      std::vector<at::Tensor>& outputTensors, std::vector<at::Tensor>& inputTensors,
      const c10d::AllToAllOptions& opts = c10d::AllToAllOptions()) override;

  // --- coalescing (group) window: the c10d analog of ncclGroupStart/End ----
  // With COMMUX_GROUP=1, send()/recv() between startCoalescing() and
  // endCoalescing() are deferred and posted together; the CUDA path then
  // issues one batched kernel per exchange. With it off, ops post at once but
  // endCoalescing() still returns a Work covering every op of the window
  // (torch's batch_isend_irecv keeps only that Work).
  bool supportsCoalescing() const override { return true; }
  void startCoalescing() override;
  c10::intrusive_ptr<c10d::Work> endCoalescing() override;

  // Post a batch of tagged receives and sends (receives first) as one group
  // and return one Work covering all of them: the native form of
  // torch.distributed.batch_isend_irecv. On CUDA the whole batch shares one
  // readiness event and, for messages to self, one copy launch.
  c10::intrusive_ptr<c10d::Work> batch_p2p(
      std::vector<at::Tensor>& recv_tensors, const std::vector<int>& recv_peers,
      const std::vector<int>& recv_tags, std::vector<at::Tensor>& send_tensors,
      const std::vector<int>& send_peers, const std::vector<int>& send_tags);

  // Persistent plan of CUDA receives and sends (matched once; the analogue of
  // MPI_Send_init/MPI_Recv_init). plan->start() enqueues one exchange of the
  // same buffers on the current stream with no host round trip. Every rank
  // the plan talks to creates its side, in the same order, and starts it the
  // same number of times.
  std::shared_ptr<DevicePlan> p2p_plan(
      const std::vector<at::Tensor>& recv_tensors, const std::vector<int>& recv_peers,
      const std::vector<int>& recv_tags, const std::vector<at::Tensor>& send_tensors,
      const std::vector<int>& send_peers, const std::vector<int>& send_tags);

  void setTimeout(std::chrono::milliseconds timeout) override;
  c10::intrusive_ptr<Options> getBackendOptions() override;
  void abort() override;
  void shutdown() override;

  // --- introspection ---------------------------------------------------------
  // Counters (messages, bytes, eager vs rendezvous, unexpected-queue depth,
  // kernel launches, IPC cache entries, ...) as name/value pairs.
  std::vector<std::pair<std::string, std::int64_t>> stats() const;
  void reset_stats();
  Engine& engine() { return *engine_; }

 private:
  c10::intrusive_ptr<c10d::Work> post_p2p(std::vector<at::Tensor>& tensors,
                                          int peer, int tag, bool is_send);
  void post_now(std::vector<at::Tensor>& tensors, int peer, int tag, bool is_send,
                std::vector<std::shared_ptr<Request>>& reqs,
                std::vector<std::pair<at::Tensor, at::Tensor>>& unpack);
  bool device_coll(const at::Tensor& t);
  static std::vector<at::Tensor> to_host(const std::vector<at::Tensor>& ts);
  static void from_host(std::vector<at::Tensor>& ts,
                        const std::vector<at::Tensor>& h);

  c10::intrusive_ptr<c10d::Store> store_;
  std::unique_ptr<Engine> engine_;
  std::unique_ptr<CollEngine> coll_;
  std::unique_ptr<GroupWindow> group_;
};

}  // namespace commux
