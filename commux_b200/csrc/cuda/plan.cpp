// Persistent p2p plans: a fixed set of tagged CUDA sends and receives,
// matched once through host set-up records and replayed by every start()
// as one CUDA graph (see CudaPlan).

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "commux/process_group_ucx.hpp"
#include "transport.hpp"
#include "wire.hpp"

namespace commux {
namespace cuda {

// ---------------------------------------------------------------------------
// persistent plans
// ---------------------------------------------------------------------------

namespace {

constexpr std::uint32_t kPlanSub = 0x7FF0;       // sub-index of setup descriptors
constexpr std::uint32_t kPlanReplySub = 0x7FF1;  // sub-index of setup replies
constexpr std::uint32_t kPlanMagic = 0x4E414C50u;

// receiver -> sender at setup: where the sender stores "ready"
struct PlanReply {
  std::uint32_t magic;
  std::int32_t pid;
  unsigned char uuid[16];
  std::uint64_t mbox_id;
  cudaIpcMemHandle_t mbox_handle;
  std::uint64_t ready_slot;
};

enum class PlanMode { Local, Device, Shared };

}  // namespace

class CudaPlan final : public DevicePlan {
 public:
  struct Msg {
    at::Tensor t;
    int peer = -1;
    int tag = 0;
    PlanMode mode = PlanMode::Local;
    std::uint64_t* ready_remote = nullptr;    // send: where "ready" is stored
    std::uint64_t* consumed_local = nullptr;  // send: set by the receiver's pull
    const std::uint64_t* ready_local = nullptr;  // recv: set by the sender
    std::vector<PullDesc> descs;              // recv (local/device)
    bool matched = false;                     // self recv paired with a send
    at::Tensor stage;                         // send: packed copy the receiver reads
    std::vector<PullDesc> pack;               // send: view -> stage
  };

  CudaPlan(CudaTransport* tr, Engine* eng, DevCtx* c) : tr_(tr), eng_(eng), c_(c) {}
  ~CudaPlan() override {
    if (!select_device_quiet(c_->dev)) return;  // context gone at process exit
    // the last start may still run: its buffers (state_, staging) must not be
    // handed to other work before it is done
    if (last_stream_ != nullptr) cudaStreamSynchronize(last_stream_);
    if (exec_) cudaGraphExecDestroy(exec_);
    if (graph_) cudaGraphDestroy(graph_);
    if (trace_h_) cudaFreeHost(trace_h_);
    if (cta_trace_h_) cudaFreeHost(cta_trace_h_);
    cudaGetLastError();
  }
  std::vector<Msg> sends, recvs;

  // Builds the launches every start() replays (captured into a CUDA graph
  // at the first start): (1) pack + "ready" signals of
  // the sends to other GPUs (without packing, the signals are stored by the
  // first pull launch at entry instead), (2) the pulls of every receive; the
  // last CTA of the last launch then waits for the receivers' "consumed"
  // flags and advances the epoch.
  // Every flag value is
  // the plan's epoch, read from device memory, so the launches never change:
  // they are captured once into a CUDA graph and a start is one graph launch.
  void finalize() {
    // Sends to another GPU: packed ones (their "ready" is stored by the last
    // warp of the pack), the rest signal "ready" at the entry of the plan's
    // first launch.
    std::vector<std::vector<PullDesc>> packs, pull;
    std::vector<std::uint64_t*> ready_only;
    for (auto& m : sends) {
      if (m.mode != PlanMode::Device) continue;
      if (m.pack.empty()) {
        ready_only.push_back(m.ready_remote);
        continue;
      }
      std::vector<PullDesc> d = m.pack;
      for (auto& x : d) x.done = m.ready_remote;
      packs.push_back(std::move(d));
    }
    for (auto& m : recvs)
      if (m.mode != PlanMode::Shared && !m.descs.empty()) pull.push_back(m.descs);
    // COMMUX_PLAN_ORDER: chunk order of the pull launch (CTAs take chunks in
    // order). "plan" (default): the order the receives were given; "local":
    // copies within this GPU first, hiding the peers' signal latency; "remote":
    // receives from other GPUs first, starting the long NVLink reads early.
    {
      static const std::string order = [] {
        const char* e = std::getenv("COMMUX_PLAN_ORDER");
        return std::string(e != nullptr ? e : "plan");
      }();
      if (order == "local" || order == "remote") {
        const bool local_first = order == "local";
        std::stable_partition(pull.begin(), pull.end(), [&](const std::vector<PullDesc>& v) {
          return (v[0].ready == nullptr) == local_first;  // a receive from another GPU waits on "ready"
        });
      }
    }
    // The packs ride in the pull launch, ahead of every pull chunk, when all
    // of them share the pull launch's unit class: each CTA (all resident,
    // the grid is capped at residency) finishes its pack chunks before it
    // waits on any peer's "ready". Otherwise they get a launch of their own
    // before the pulls.
    bool merge = !packs.empty() && !pull.empty();
    // one launch only: a pack split into a later launch of the peer, behind
    // pulls that wait, could leave two ranks waiting on each other
    std::size_t ndesc = 0;
    for (auto* v : {&packs, &pull})
      for (auto& m : *v) ndesc += m.size();
    merge = merge && ndesc <= static_cast<std::size_t>(kMaxBatch);
    if (merge) {
      const int cls = pull_unit_class(pull[0][0]);
      for (auto& m : pull) merge = merge && pull_unit_class(m[0]) == cls;
      for (auto& m : packs) merge = merge && pull_unit_class(m[0]) == cls;
    }
    std::vector<std::vector<PullDesc>> pre;
    std::size_t lead = 0;  // pack messages at the head of the pull launch
    if (merge) {
      pull.insert(pull.begin(), packs.begin(), packs.end());
      lead = packs.size();
    } else {
      pre = packs;
    }
    // no launch at all would carry the entry signals: a pure-signal launch
    if (pre.empty() && pull.empty() && !ready_only.empty()) {
      PullDesc x{};
      x.ndim = 1;
      x.unit = 16;
      x.units = 0;
      x.nchunks = 1;
      pre.push_back({x});
    }
    // device state: [epoch u64, starts at 1][finished-CTA count u32][pad to
    // 64 bytes][counters u32 x kCounterSlots]
    const std::size_t state_bytes = 64 + kCounterSlots * sizeof(std::uint32_t);
    state_ = at::empty({static_cast<std::int64_t>(state_bytes)},
                       at::TensorOptions().dtype(at::kByte).device(at::kCUDA, c_->dev));
    epoch_d_ = reinterpret_cast<std::uint64_t*>(state_.data_ptr());
    cta_done_d_ = reinterpret_cast<unsigned int*>(static_cast<char*>(state_.data_ptr()) + 8);
    counters_d_ = reinterpret_cast<std::uint32_t*>(static_cast<char*>(state_.data_ptr()) + 64);
    std::vector<char> init(state_bytes, 0);
    const std::uint64_t one = 1;
    std::memcpy(init.data(), &one, sizeof(one));
    CMX_CUDA(cudaMemcpy(state_.data_ptr(), init.data(), state_bytes, cudaMemcpyHostToDevice));
    // a plan whose messages all stay on this GPU has no flags: its launches
    // skip the epoch (one dependent load less at kernel start)
    for (auto* v : {&sends, &recvs})
      for (auto& m : *v) has_flags_ |= m.mode == PlanMode::Device;
    pre_ = batches(pre, pre.size());
    pulls_ = batches(pull, lead);
    if (!ready_only.empty()) {
      TORCH_CHECK(ready_only.size() <= static_cast<std::size_t>(kMaxEntrySignals), "commux plan: more than ",
                  kMaxEntrySignals, " unpacked sends to other GPUs");
      PullBatch& first = pre_.empty() ? *pulls_[0] : *pre_[0];
      first.nsig = static_cast<std::uint32_t>(ready_only.size());
      for (std::size_t k = 0; k < ready_only.size(); ++k) first.sig[k] = ready_only[k];
    }
    std::vector<const std::uint64_t*> fins;  // the "consumed" flags of the sends to other GPUs
    for (auto& m : sends)
      if (m.mode == PlanMode::Device) {
        TORCH_CHECK(fins.size() < static_cast<std::size_t>(kMaxWaitFlags), "commux plan: more than ",
                    kMaxWaitFlags, " sends to other GPUs");
        fins.push_back(m.consumed_local);
      }
    // the receivers' "consumed" flags and the epoch bump ride on the last
    // launch: its last CTA waits for them and advances the epoch
    bool flags = !fins.empty();
    for (auto& m : recvs) flags |= m.mode == PlanMode::Device;
    PullBatch* last = !pulls_.empty() ? pulls_.back().get() : !pre_.empty() ? pre_.back().get() : nullptr;
    TORCH_CHECK(!flags || last != nullptr, "commux plan: internal error, flags without a launch");
    if (flags) {
      last->bump = epoch_d_;
      last->cta_done = cta_done_d_;
      last->nfin = static_cast<std::uint32_t>(fins.size());
      for (std::size_t k = 0; k < fins.size(); ++k) last->fin[k] = fins[k];
    }
    // COMMUX_PLAN_TRACE: span of every launch of a start (earliest CTA start,
    // latest CTA end), printed after each start (which then synchronises)
    if (env_int("COMMUX_PLAN_TRACE", 0) != 0) {
      const std::size_t n = pre_.size() + pulls_.size();
      CMX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&trace_h_), n * 2 * sizeof(unsigned long long),
                             cudaHostAllocMapped));
      unsigned long long* d = nullptr;
      CMX_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), trace_h_, 0));
      std::size_t k = 0;
      // the last message-counter slot is the launches' CTA counter (reset
      // by the last CTA of each launch)
      std::uint32_t* count = counters_d_ + (kCounterSlots - 1);
      for (auto* ls : {&pre_, &pulls_})
        for (auto& b : *ls) {
          b->trace = d + 2 * k++;
          b->trace_count = count;
        }
      trace_n_ = n;
      // COMMUX_PLAN_TRACE=2: per-CTA stamps of the last launch (the pulls)
      if (env_int("COMMUX_PLAN_TRACE", 0) >= 2 && (!pulls_.empty() || !pre_.empty())) {
        cta_trace_n_ = static_cast<std::size_t>(8 * c_->sm_count);
        CMX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&cta_trace_h_), cta_trace_n_ * 4 * sizeof(unsigned long long),
                               cudaHostAllocMapped));
        unsigned long long* dd = nullptr;
        CMX_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dd), cta_trace_h_, 0));
        (pulls_.empty() ? pre_.back() : pulls_.back())->cta_trace = dd;
      }
    }
    // every batch goes to device memory once: a launch passes one pointer,
    // and each CTA stages the batch into shared memory (pull_kernel_staged)
    const std::size_t nb = pre_.size() + pulls_.size();
    if (nb > 0) {
      batches_d_ = at::empty({static_cast<std::int64_t>(nb * sizeof(PullBatch))},
                             at::TensorOptions().dtype(at::kByte).device(at::kCUDA, c_->dev));
      std::size_t k = 0;
      for (auto* ls : {&pre_, &pulls_})
        for (auto& b : *ls) CMX_CUDA(cudaMemcpy(dev_batch(k++), b.get(), sizeof(PullBatch), cudaMemcpyHostToDevice));
    }
  }

  PullBatch* dev_batch(std::size_t k) {
    return reinterpret_cast<PullBatch*>(static_cast<char*>(batches_d_.data_ptr()) + k * sizeof(PullBatch));
  }

  // Grid cap of the launches. A launch whose CTAs wait on peers keeps every
  // CTA resident at once, so a CTA never waits while another CTA of the
  // launch that still has pack work waits for an SM; launches without waits
  // keep the wider grid.
  int grid_ctas() const {
    bool waits = false;
    for (auto& m : recvs) waits |= m.mode == PlanMode::Device;
    int ctas = waits ? std::min(tr_->pull_ctas(c_), 4 * c_->sm_count) : tr_->pull_ctas(c_);
    if (max_ctas_ > 0) ctas = std::min(ctas, max_ctas_);
    return ctas;
  }


  void start() override {
    ++starts_;
    tr_->plan_starts++;
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c_->dev));
    cudaStream_t cur = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(c_->dev)).stream();
    // messages to/from a rank on this same GPU go through the host-gated path
    std::vector<ReqPtr> shared;
    if (n_shared_) {
      tr_->begin_batch();
      try {
        auto tag = [](const Msg& m) { return make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), 0, false); };
        for (auto& m : recvs)
          if (m.mode == PlanMode::Shared) shared.push_back(eng_->post_recv({m.t}, m.peer, tag(m)));
        for (auto& m : sends)
          if (m.mode == PlanMode::Shared) shared.push_back(eng_->post_send({m.t}, m.peer, tag(m)));
      } catch (...) {
        tr_->end_batch();
        throw;
      }
      tr_->end_batch();
    }
    last_stream_ = cur;
    if (trace_h_ != nullptr)
      for (std::size_t k = 0; k < trace_n_; ++k) {
        trace_h_[2 * k] = ~0ull;
        trace_h_[2 * k + 1] = 0;
      }
    if (pre_.size() + pulls_.size() > 0) {
      if (!exec_) capture();
      CMX_CUDA(cudaGraphLaunch(exec_, cur));
      tr_->kernel_launches += nodes_;
    }
    if (trace_h_ != nullptr) report_trace(cur);
    if (!shared.empty()) {
      for (auto& r : shared) eng_->wait(r, std::chrono::milliseconds(0));
      tr_->stream_wait_all(shared);
    }
    std::string e = tr_->device_error();
    if (!e.empty()) C10_THROW_ERROR(DistBackendError, e);
  }

  void set_max_ctas(int ctas) override {
    TORCH_CHECK(ctas >= 0, "commux plan: max_ctas must be >= 0");
    if (ctas == max_ctas_) return;
    max_ctas_ = ctas;
    if (exec_) {  // captured with the old grid: capture again at the next start
      c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c_->dev));
      if (last_stream_ != nullptr) CMX_CUDA(cudaStreamSynchronize(last_stream_));
      cudaGraphExecDestroy(exec_);
      cudaGraphDestroy(graph_);
      exec_ = nullptr;
      graph_ = nullptr;
    }
  }

  std::vector<std::pair<std::string, std::int64_t>> info() override {
    std::int64_t loc = 0, dev = 0, packed = 0;
    for (auto* v : {&sends, &recvs})
      for (auto& m : *v) (m.mode == PlanMode::Local ? loc : dev) += m.mode != PlanMode::Shared;
    for (auto& m : sends) packed += (m.mode == PlanMode::Device && !m.pack.empty()) ? 1 : 0;
    return {{"local", loc},      {"device", dev},       {"shared", n_shared_}, {"packed_sends", packed},
            {"graph_nodes", nodes_}, {"starts", static_cast<std::int64_t>(starts_)}, {"max_ctas", max_ctas_}};
  }

  std::int64_t n_shared_ = 0;

 private:
  void report_trace(cudaStream_t cur) {
    CMX_CUDA(cudaStreamSynchronize(cur));
    unsigned long long t0 = ~0ull;
    for (std::size_t k = 0; k < trace_n_; ++k) t0 = std::min(t0, trace_h_[2 * k]);
    std::string line;
    char buf[160];
    std::size_t k = 0;
    auto span = [&](const char* what) {
      const unsigned long long a = trace_h_[2 * k], b = trace_h_[2 * k + 1];
      ++k;
      if (a == ~0ull || b == 0) return;  // launch left out of this plan's graph
      std::snprintf(buf, sizeof(buf), " %s %.1f-%.1f", what, (a - t0) / 1e3, (b - t0) / 1e3);
      line += buf;
    };
    for (std::size_t i = 0; i < pre_.size(); ++i) span("pack");
    for (std::size_t i = 0; i < pulls_.size(); ++i) span("pull");
    if (cta_trace_h_ != nullptr) {
      // CTAs that ran (end stamp set): spans, ready-flag waits, flagged chunks
      std::vector<double> span_us;
      double wait_sum = 0, wait_max = 0, first = 1e300, last = 0;
      unsigned long long flagged = 0;
      int waited_ctas = 0;
      for (std::size_t k = 0; k < cta_trace_n_; ++k) {
        const unsigned long long* r = cta_trace_h_ + 4 * k;
        if (r[1] == 0) continue;
        span_us.push_back((r[1] - r[0]) / 1e3);
        first = std::min(first, static_cast<double>(r[0]));
        last = std::max(last, static_cast<double>(r[1]));
        wait_sum += r[2] / 1e3;
        wait_max = std::max(wait_max, r[2] / 1e3);
        flagged += r[3];
        waited_ctas += r[3] > 0 ? 1 : 0;
      }
      if (!span_us.empty()) {
        std::sort(span_us.begin(), span_us.end());
        std::snprintf(buf, sizeof(buf), " | ctas %zu span p50 %.1f max %.1f us, first-to-last %.1f us",
                      span_us.size(), span_us[span_us.size() / 2], span_us.back(), (last - first) / 1e3);
        line += buf;
        std::snprintf(buf, sizeof(buf), ", flagged chunks %llu on %d ctas, ready wait sum %.1f max %.1f us",
                      flagged, waited_ctas, wait_sum, wait_max);
        line += buf;
      }
      for (std::size_t k = 0; k < cta_trace_n_ * 4; ++k) cta_trace_h_[k] = 0;
    }
    std::fprintf(stderr, "[commux plan trace rank %d] start %llu, us from the first CTA:%s\n", eng_->rank(),
                 static_cast<unsigned long long>(starts_), line.c_str());
  }

  // Messages -> batches of at most kMaxBatch descriptors, one unit class
  // each; every message counts into its own counter slot (the plan's
  // launches run one after another and each message returns its counter to
  // zero, so the slots are reused by the next start). Messages of one
  // descriptor and equal chunk count (a halo's six faces) after the first
  // `lead` messages (the packs, which run first) form an interleaved group
  // placed where its first member was: their chunks go round robin, so row k
  // of every face is copied at about the same time and faces that share
  // DRAM sectors (the 16-byte x-face rows of both sides of a row) meet in L2
  // (COMMUX_PLAN_INTERLEAVE=0 keeps the message order).
  std::vector<std::unique_ptr<PullBatch>> batches(const std::vector<std::vector<PullDesc>>& msgs,
                                                  std::size_t lead = 0) {
    static const bool interleave = env_int("COMMUX_PLAN_INTERLEAVE", 1) != 0;
    struct Unit {
      std::vector<PullDesc> descs;  // one message, or an interleaved group
      std::uint32_t ilv = 1;
    };
    std::map<int, std::vector<Unit>> by_cls;
    std::map<std::pair<int, std::uint32_t>, std::size_t> group_at;  // (class, chunks) -> unit index
    std::uint32_t slot = 0;
    for (std::size_t mi = 0; mi < msgs.size(); ++mi) {
      const auto& m = msgs[mi];
      if (m.empty()) continue;
      const int cls = pull_unit_class(m[0]);
      std::uint32_t chunks = 0;
      for (auto& d : m) {
        TORCH_CHECK(pull_unit_class(d) == cls, "commux plan: a message mixes unit classes");
        chunks += d.nchunks;
      }
      TORCH_CHECK(slot < kCounterSlots - 1, "commux plan: too many messages");
      auto& v = by_cls[cls];
      std::vector<PullDesc> ds(m);
      for (auto& d : ds) {
        d.counter_idx = slot;
        d.msg_chunks = chunks;
        d.ilv = 1;
      }
      ++slot;
      if (interleave && mi >= lead && ds.size() == 1 && chunks >= 2) {
        auto key = std::make_pair(cls, chunks);
        auto it = group_at.find(key);
        if (it != group_at.end() && v[it->second].ilv < 32) {
          v[it->second].descs.push_back(ds[0]);
          v[it->second].ilv++;
          continue;
        }
        group_at[key] = v.size();
      }
      v.push_back(Unit{std::move(ds), 1});
    }
    std::vector<std::unique_ptr<PullBatch>> out;
    auto fresh = [&]() {
      auto b = std::make_unique<PullBatch>();
      b->n = 0;
      b->total_chunks = 0;
      b->counters = counters_d_;
      b->status = c_->status_d;
      b->timeout_ns = tr_->device_timeout_ns();
      b->epoch = has_flags_ ? epoch_d_ : nullptr;
      b->nsig = 0;
      return b;
    };
    for (auto& kv : by_cls) {
      std::unique_ptr<PullBatch> b = fresh();
      for (auto& u : kv.second) {
        if (b->n + u.descs.size() > static_cast<std::size_t>(kMaxBatch)) {
          out.push_back(std::move(b));
          b = fresh();
        }
        const std::uint32_t first = b->n, c0 = b->total_chunks;
        for (auto d : u.descs) {
          if (u.ilv > 1) {  // the group's members share chunk0 and their chunk range
            d.chunk0 = c0;
            d.ilv = u.ilv;
            d.ilv_first = first;
          } else {
            d.chunk0 = b->total_chunks;
          }
          b->total_chunks += d.nchunks;
          b->d[b->n++] = d;
        }
      }
      if (b->n > 0) out.push_back(std::move(b));
    }
    return out;
  }

  void capture() {
    cudaStream_t cs = nullptr;
    CMX_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    const int ctas = grid_ctas();
    nodes_ = 0;
    CMX_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    std::size_t k = 0;
    for (auto* ls : {&pre_, &pulls_})
      for (auto& b : *ls) {
        if (e == cudaSuccess) e = launch_pull_staged(*b, dev_batch(k), ctas, cs);
        ++k;
        ++nodes_;
      }
    // the receivers' "consumed" flags and the epoch bump ride on the last
    // launch (its last CTA waits and bumps; see PullBatch::bump); a plan
    // whose every message stays on this GPU has no flags and no epoch
    cudaGraph_t g = nullptr;
    cudaError_t e2 = cudaStreamEndCapture(cs, &g);
    cudaStreamDestroy(cs);  // holds no tensors: safe to destroy
    CMX_CUDA(e);
    CMX_CUDA(e2);
    graph_ = g;
    CMX_CUDA(cudaGraphInstantiate(&exec_, graph_, 0));
  }

  CudaTransport* tr_;
  Engine* eng_;
  DevCtx* c_;
  std::uint64_t starts_ = 0;
  at::Tensor state_;
  std::uint64_t* epoch_d_ = nullptr;
  unsigned int* cta_done_d_ = nullptr;
  at::Tensor batches_d_;  // the launches' batches in device memory
  int max_ctas_ = 0;      // set_max_ctas (0: the default grid)
  bool has_flags_ = false;  // some message crosses to another GPU
  std::uint32_t* counters_d_ = nullptr;
  std::vector<std::unique_ptr<PullBatch>> pre_, pulls_;
  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t exec_ = nullptr;
  std::int64_t nodes_ = 0;
  unsigned long long* trace_h_ = nullptr;  // COMMUX_PLAN_TRACE (host-mapped)
  unsigned long long* cta_trace_h_ = nullptr;  // COMMUX_PLAN_TRACE=2: per-CTA stamps
  std::size_t cta_trace_n_ = 0;
  std::size_t trace_n_ = 0;
  cudaStream_t last_stream_ = nullptr;      // stream of the last start
};

std::vector<PullDesc> CudaTransport::plan_descs(const char* wire, std::size_t len, int src, bool local,
                                                const at::Tensor& dst, DevCtx* c) {
  auto r = std::make_shared<Request>();
  r->kind = ReqKind::Recv;
  r->device = true;
  r->tensors = {dst};
  r->total = static_cast<std::uint64_t>(dst.numel()) * dst.element_size();
  auto rs = std::make_shared<RecvState>();
  rs->device = c->dev;
  r->dev = rs;
  PendingPull pp;
  pp.r = r;
  pp.src = src;
  pp.ctx = c;
  build_descs(r, wire, len, local, pp);
  TORCH_CHECK(rs->unpack.empty(), "commux plan: this receive layout needs a staged copy; persistent plans "
              "take views whose strides merge to at most 4 dims on both sides");
  return pp.descs;
}

DevicePlanPtr CudaTransport::create_plan(const std::vector<at::Tensor>& recv_t, const std::vector<int>& recv_peer,
                                         const std::vector<int>& recv_tag, const std::vector<at::Tensor>& send_t,
                                         const std::vector<int>& send_peer, const std::vector<int>& send_tag) {
  TORCH_CHECK(!recv_t.empty() || !send_t.empty(), "commux plan: no messages");
  const at::Tensor& any = recv_t.empty() ? send_t[0] : recv_t[0];
  const int dev = any.device().index();
  for (auto* v : {&recv_t, &send_t})
    for (auto& t : *v)
      TORCH_CHECK(t.is_cuda() && t.device().index() == dev, "commux plan: all tensors must be on one CUDA device");
  DevCtx* c = ctx(dev);
  publish_uuid(c);
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
  const int me = eng_->rank();
  auto plan = std::make_shared<CudaPlan>(this, eng_, c);

  // wire description of one tensor (DrtsWire + one SegWire), as a send would
  auto wire_of = [&](const at::Tensor& t, bool local, std::uint64_t consumed_slot) {
    std::vector<std::int64_t> sz(t.sizes().begin(), t.sizes().end()), sd(t.strides().begin(), t.strides().end());
    auto d = dims_of(sz.data(), sd.data(), t.dim());
    std::vector<Dim> merged;
    TORCH_CHECK(t.dim() <= kWireDims && refine(d, d, merged) && merged.size() <= static_cast<std::size_t>(kMaxPullDims),
                "commux plan: send views must merge to at most 4 dims (send a contiguous tensor)");
    std::vector<char> blob(sizeof(DrtsWire) + sizeof(SegWire), 0);
    auto* w = reinterpret_cast<DrtsWire*>(blob.data());
    w->magic = kWireMagic;
    w->nseg = 1;
    w->pid = static_cast<std::int32_t>(::getpid());
    w->device = dev;
    std::memcpy(w->uuid, c->uuid, 16);
    w->mbox_id = c->mbox_id;
    w->mbox_base = c->mbox_base;
    w->mbox_handle = c->mbox_handle;
    w->slot = consumed_slot;
    auto* sw = reinterpret_cast<SegWire*>(blob.data() + sizeof(DrtsWire));
    sw->elem = static_cast<std::uint32_t>(t.element_size());
    sw->ndim = static_cast<std::int32_t>(t.dim());
    for (int k = 0; k < t.dim(); ++k) {
      sw->sizes[k] = t.size(k);
      sw->strides[k] = t.stride(k);
    }
    if (t.numel() > 0) {
      const char* p = static_cast<const char*>(t.data_ptr());
      if (local) {
        CUpointer_attribute attrs[2] = {CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, CU_POINTER_ATTRIBUTE_RANGE_SIZE};
        CUdeviceptr start = 0;
        std::size_t asz = 0;
        void* data[2] = {&start, &asz};
        cu_check(cuPointerGetAttributes(2, attrs, data, reinterpret_cast<CUdeviceptr>(p)), "cuPointerGetAttributes");
        sw->base = static_cast<std::uint64_t>(start);
        sw->alloc_size = asz;
      } else {
        ipc_export(p, &sw->buffer_id, &sw->base, &sw->alloc_size, &sw->handle);
      }
      sw->offset = reinterpret_cast<std::uint64_t>(p) - sw->base;
    }
    return blob;
  };
  auto plan_slot = [&]() {
    std::uint64_t s = kSlots + c->next_plan_slot.fetch_add(1);
    TORCH_CHECK(s < 2 * kSlots, "commux plan: out of persistent flag slots");
    return s;
  };
  auto bytes_tensor = [](const void* p, std::size_t n) {
    at::Tensor t = at::empty({static_cast<std::int64_t>(n)}, at::TensorOptions().dtype(at::kByte));
    std::memcpy(t.data_ptr(), p, n);
    return t;
  };
  const std::size_t wire_len = sizeof(DrtsWire) + sizeof(SegWire);

  std::vector<ReqPtr> pending_sends;
  struct RecvSetup {
    std::size_t idx;
    ReqPtr req;
    at::Tensor buf;
  };
  std::vector<RecvSetup> desc_recvs, reply_recvs;
  // sends: descriptor to the receiver, then expect its reply
  for (std::size_t i = 0; i < send_t.size(); ++i) {
    CudaPlan::Msg m;
    m.t = send_t[i];
    m.peer = send_peer[i];
    m.tag = send_tag[i];
    TORCH_CHECK(m.peer >= 0 && m.peer < eng_->size(), "commux plan: invalid send peer ", m.peer);
    if (m.peer == me) {
      m.mode = PlanMode::Local;
    } else {
      std::uint64_t slot = plan_slot();
      m.consumed_local = c->mbox + slot;
      // narrow rows: the receiver reads a contiguous copy packed here (the
      // pack descriptors run in the plan's first launch; a receiver that
      // turns out to share this GPU reads the view itself)
      at::Tensor wire_src = m.t;
      // also staged: memory that CUDA IPC cannot export; the stage then comes
      // from the exportable pool
      const bool unexportable = m.t.numel() > 0 && !exportable(m.t.data_ptr());
      if (narrow_rows(m.t) || unexportable) {
        m.stage = at::empty(m.t.sizes(), m.t.options().memory_format(at::MemoryFormat::Contiguous));
        if (!exportable(m.stage.data_ptr())) m.stage = c->exportable_empty(m.t.sizes(), m.t.scalar_type());
        auto self_blob = wire_of(m.t, true, 0);
        m.pack = plan_descs(self_blob.data(), self_blob.size(), me, true, m.stage, c);
        wire_src = m.stage;
      }
      auto blob = wire_of(wire_src, false, slot);
      pending_sends.push_back(eng_->post_send({bytes_tensor(blob.data(), blob.size())}, m.peer,
                                              make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), kPlanSub, true)));
      at::Tensor rb = at::empty({static_cast<std::int64_t>(sizeof(PlanReply))}, at::TensorOptions().dtype(at::kByte));
      const auto rtag = make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), kPlanReplySub, true);
      reply_recvs.push_back({plan->sends.size(), eng_->post_recv({rb}, m.peer, rtag), rb});
    }
    plan->sends.push_back(std::move(m));
  }
  // receives: expect the sender's descriptor
  for (std::size_t j = 0; j < recv_t.size(); ++j) {
    CudaPlan::Msg m;
    m.t = recv_t[j];
    m.peer = recv_peer[j];
    m.tag = recv_tag[j];
    TORCH_CHECK(m.peer >= 0 && m.peer < eng_->size(), "commux plan: invalid recv peer ", m.peer);
    if (m.peer == me) {
      m.mode = PlanMode::Local;
    } else {
      at::Tensor db = at::empty({static_cast<std::int64_t>(wire_len)}, at::TensorOptions().dtype(at::kByte));
      const auto dtag = make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), kPlanSub, true);
      desc_recvs.push_back({plan->recvs.size(), eng_->post_recv({db}, m.peer, dtag), db});
    }
    plan->recvs.push_back(std::move(m));
  }
  // self messages pair up locally, FIFO per tag
  for (auto& s : plan->sends) {
    if (s.peer != me) continue;
    CudaPlan::Msg* r = nullptr;
    for (auto& x : plan->recvs)
      if (x.peer == me && !x.matched && x.tag == s.tag) {
        r = &x;
        break;
      }
    TORCH_CHECK(r != nullptr, "commux plan: self-send with tag ", s.tag, " has no matching self-receive");
    r->matched = true;
    auto blob = wire_of(s.t, true, 0);
    r->descs = plan_descs(blob.data(), blob.size(), me, true, r->t, c);
  }
  for (auto& x : plan->recvs)
    TORCH_CHECK(x.peer != me || x.matched, "commux plan: self-receive with tag ", x.tag, " has no matching self-send");
  // remote receives: build the pull, allocate "ready", reply to the sender
  for (auto& rs : desc_recvs) {
    eng_->wait(rs.req, std::chrono::milliseconds(0));
    CudaPlan::Msg& m = plan->recvs[rs.idx];
    const char* blob = static_cast<const char*>(rs.buf.data_ptr());
    auto* w = reinterpret_cast<const DrtsWire*>(blob);
    TORCH_CHECK(w->magic == kWireMagic, "commux plan: malformed setup descriptor from rank ", m.peer);
    const bool same_gpu = std::memcmp(w->uuid, c->uuid, 16) == 0;
    PlanReply rep;
    std::memset(&rep, 0, sizeof(rep));
    rep.magic = kPlanMagic;
    rep.pid = static_cast<std::int32_t>(::getpid());
    std::memcpy(rep.uuid, c->uuid, 16);
    rep.mbox_id = c->mbox_id;
    rep.mbox_handle = c->mbox_handle;
    if (same_gpu) {
      m.mode = PlanMode::Shared;
      plan->n_shared_++;
    } else {
      m.mode = PlanMode::Device;
      std::uint64_t slot = plan_slot();
      m.ready_local = c->mbox + slot;
      rep.ready_slot = slot;
      m.descs = plan_descs(blob, wire_len, m.peer, false, m.t, c);
      for (auto& d : m.descs) d.ready = m.ready_local;
    }
    pending_sends.push_back(eng_->post_send({bytes_tensor(&rep, sizeof(rep))}, m.peer,
                                            make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), kPlanReplySub, true)));
  }
  // remote sends: learn where to store "ready"
  for (auto& rr : reply_recvs) {
    eng_->wait(rr.req, std::chrono::milliseconds(0));
    CudaPlan::Msg& m = plan->sends[rr.idx];
    PlanReply rep;
    std::memcpy(&rep, rr.buf.data_ptr(), sizeof(rep));
    TORCH_CHECK(rep.magic == kPlanMagic, "commux plan: malformed setup reply from rank ", m.peer);
    if (std::memcmp(rep.uuid, c->uuid, 16) == 0) {
      m.mode = PlanMode::Shared;
      plan->n_shared_++;
    } else {
      m.mode = PlanMode::Device;
      auto* mb = static_cast<std::uint64_t*>(ipc_open(m.peer, rep.mbox_id, 0, 0, rep.mbox_handle, c));
      m.ready_remote = mb + rep.ready_slot;
    }
  }
  for (auto& s : pending_sends) eng_->wait(s, std::chrono::milliseconds(0));
  for (auto* v : {&plan->sends, &plan->recvs})
    for (auto& m : *v) {
      if (m.mode == PlanMode::Device) plan_device_msgs++;
      if (m.mode == PlanMode::Shared) plan_shared_msgs++;
    }
  plan->finalize();
  return plan;
}

}  // namespace cuda
}  // namespace commux
