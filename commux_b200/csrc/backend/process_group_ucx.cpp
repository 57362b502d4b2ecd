// c10d::Backend facade of commux: p2p (tagged, coalesced, grouped) and the
// collectives, for CPU and CUDA tensors.
//
// Parity map with the reference backend (reference: src/process_group_ucx.cpp):
//   send/recv/recvAnysource    :568-732   -> post_p2p / recvAnysource below
//   COMMUX_COALESCE IOV path   :596-622   -> one multi-segment message
//   COMMUX_GROUP window        :825-883   -> startCoalescing/endCoalescing
//   allreduce/reduce/broadcast/barrier :734-823 -> CollEngine (host) or the
//                                                  CUDA transport (device)
//   check_reduce_op (#13)      :236-247   -> validate_op, before any message
// New here: allgather/_allgather_base (torch DDP), gather, scatter,
// reduce_scatter, alltoall_base, Work::getFuture, timeouts, abort.

#include "commux/process_group_ucx.hpp"
#include "../engine/log.hpp"

#include <ATen/ATen.h>
#include <ATen/core/ivalue.h>
#include <c10/util/Exception.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../engine/engine.hpp"
#include "reduce_cpu.hpp"

namespace commux {

tag_t make_ucp_tag(int sender_rank, std::uint32_t user_tag, std::uint32_t sub_index,
                   bool collective) {
  tag_t t = 0;
  t |= static_cast<tag_t>(static_cast<std::uint32_t>(sender_rank) & 0xFFFFu) << 48;
  t |= static_cast<tag_t>(sub_index & 0x7FFFu) << 33;
  t |= static_cast<tag_t>(collective ? 1u : 0u) << 32;
  t |= static_cast<tag_t>(user_tag);
  return t;
}

namespace {

bool coalesce_enabled() {
  static const bool v = env_flag("COMMUX_COALESCE");
  return v;
}
bool group_enabled() {
  static const bool v = env_flag("COMMUX_GROUP");
  return v;
}

[[noreturn]] void throw_backend(const std::string& msg) { C10_THROW_ERROR(DistBackendError, msg); }

RedOp to_redop(const c10d::ReduceOp& op, const char* what) {
  switch (op.op_) {
    case c10d::ReduceOp::SUM:
      return RedOp::Sum;
    case c10d::ReduceOp::PRODUCT:
      return RedOp::Prod;
    case c10d::ReduceOp::MIN:
      return RedOp::Min;
    case c10d::ReduceOp::MAX:
      return RedOp::Max;
    case c10d::ReduceOp::AVG:
      return RedOp::Avg;
    default:
      TORCH_CHECK(false, "commux ", what, ": unsupported ReduceOp ", static_cast<int>(op.op_));
  }
}

// Validate op and dtypes of every tensor before any rank sends anything, so an
// unsupported combination raises on every rank (reference issue #13).
RedOp validate_op(const c10d::ReduceOp& op, const std::vector<at::Tensor>& ts, const char* what) {
  RedOp r = to_redop(op, what);
  for (auto& t : ts) {
    std::string e = check_reduce(t.scalar_type(), r);
    TORCH_CHECK(e.empty(), "commux ", what, ": ", e);
  }
  return r;
}

void check_same_device_kind(const std::vector<at::Tensor>& ts, const char* what) {
  TORCH_CHECK(!ts.empty(), "commux ", what, ": empty tensor list");
  bool cuda = ts[0].is_cuda();
  for (auto& t : ts)
    TORCH_CHECK(t.is_cuda() == cuda && (t.is_cuda() || t.is_cpu()), "commux ", what,
                ": tensors must all be CPU or all be CUDA");
}

}  // namespace

// ---------------------------------------------------------------------------
// Work
// ---------------------------------------------------------------------------

class CommuxWork : public c10d::Work {
 public:
  CommuxWork(Engine* eng, c10d::OpType op, std::vector<ReqPtr> reqs, std::vector<at::Tensor> outs,
             int source_rank = -1)
      : c10d::Work(-1, op),
        eng_(eng),
        reqs_(std::move(reqs)),
        outs_(std::move(outs)),
        source_rank_(source_rank) {}

  void add(std::vector<ReqPtr> reqs, std::vector<at::Tensor> outs) {
    std::lock_guard<std::mutex> lk(mu_);
    for (auto& r : reqs) reqs_.push_back(std::move(r));
    for (auto& t : outs) outs_.push_back(std::move(t));
  }
  void add_device(DevCollPtr d) {
    std::lock_guard<std::mutex> lk(mu_);
    dev_.push_back(std::move(d));
  }
  // CPU receive into a strided view: the bytes land in `tmp`, copied into
  // `view` once the receive completed.
  void add_unpack(at::Tensor tmp, at::Tensor view) {
    std::lock_guard<std::mutex> lk(mu_);
    unpack_.push_back({std::move(tmp), std::move(view)});
  }
  void set_source(int s) { source_rank_ = s; }

  bool isCompleted() override {
    std::lock_guard<std::mutex> lk(mu_);
    for (auto& r : reqs_) {
      int st = r->state.load(std::memory_order_acquire);
      if (st == kPending) return false;
      if (st == kFailed) {
        record_error(r->error);
        continue;
      }
      if (r->device) {
        auto* d = eng_->device(false);
        if (d && !d->query(r)) return false;
      }
    }
    for (auto& d : dev_)
      if (!d->query()) return false;
    unpack_locked();
    return true;
  }

  bool isSuccess() const override {
    std::lock_guard<std::mutex> lk(mu_);
    return !err_;
  }

  std::exception_ptr exception() const override {
    std::lock_guard<std::mutex> lk(mu_);
    return err_;
  }

  int sourceRank() const override {
    if (source_rank_ >= 0) return source_rank_;
    return reqs_.size() == 1 ? reqs_[0]->source.load() : -1;
  }

  std::vector<at::Tensor> result() override { return outs_; }

  bool wait(std::chrono::milliseconds timeout = kNoTimeout) override {
    std::vector<ReqPtr> reqs;
    std::vector<DevCollPtr> devs;
    {
      std::lock_guard<std::mutex> lk(mu_);
      reqs = reqs_;
      devs = dev_;
    }
    auto to = timeout == kNoTimeout ? std::chrono::milliseconds(0) : timeout;
    try {
      for (auto& r : reqs) eng_->wait(r, to);
      std::vector<ReqPtr> dev_reqs;
      for (auto& r : reqs)
        if (r->device) dev_reqs.push_back(r);
      if (!dev_reqs.empty()) eng_->device()->stream_wait_all(dev_reqs);
      for (auto& d : devs) {
        std::string e = d->error();
        if (!e.empty()) throw_backend(e);
        d->stream_wait();
      }
      if (!reqs.empty() && reqs[0]->device) {
        std::string e = eng_->device()->device_error();
        if (!e.empty()) throw_backend(e);
      }
    } catch (...) {
      std::lock_guard<std::mutex> lk(mu_);
      if (!err_) err_ = std::current_exception();
      throw;
    }
    std::lock_guard<std::mutex> lk(mu_);
    unpack_locked();
    return true;
  }

  void synchronize() override {
    std::vector<ReqPtr> reqs;
    std::vector<DevCollPtr> devs;
    {
      std::lock_guard<std::mutex> lk(mu_);
      reqs = reqs_;
      devs = dev_;
    }
    for (auto& r : reqs)
      if (r->device && r->state.load() == kDone) eng_->device()->stream_wait(r);
    for (auto& d : devs) d->stream_wait();
  }

  c10::intrusive_ptr<c10::ivalue::Future> getFuture() override {
    std::vector<c10::Device> devices;
    bool cuda = false;
    DevCollPtr dev_last;
    bool has_reqs = false;
    c10::intrusive_ptr<c10::ivalue::Future> fut;
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (future_) return future_;
      for (auto& t : outs_)
        if (t.is_cuda()) {
          cuda = true;
          if (std::find(devices.begin(), devices.end(), t.device()) == devices.end())
            devices.push_back(t.device());
        }
      if (!dev_.empty()) dev_last = dev_.back();
      has_reqs = !reqs_.empty();
      future_ = c10::make_intrusive<c10::ivalue::Future>(
          c10::ListType::create(c10::TensorType::get()), devices);
      fut = future_;
    }
    if (dev_last && !has_reqs && cuda) {
      // Collective on a CUDA stream: complete now, synchronised through the
      // collective's stream (consumers wait on its event, not on the host).
      c10::IValue value(outs_);
      dev_last->mark_future(fut.get(), &value);
      return fut;
    }
    try {
      wait();
    } catch (...) {
      fut->setError(std::current_exception());
      return fut;
    }
    fut->markCompleted(c10::IValue(outs_));
    return fut;
  }

 private:
  void unpack_locked() {
    for (auto& tv : unpack_) tv.second.copy_(tv.first.view(tv.second.sizes()));
    unpack_.clear();
  }

  void record_error(const std::string& e) {
    if (!err_) err_ = std::make_exception_ptr(c10::DistBackendError(
                   c10::SourceLocation{__func__, __FILE__, static_cast<uint32_t>(__LINE__)}, e));
  }

  Engine* eng_;
  mutable std::mutex mu_;
  std::vector<ReqPtr> reqs_;
  std::vector<DevCollPtr> dev_;
  std::vector<at::Tensor> outs_;
  std::vector<std::pair<at::Tensor, at::Tensor>> unpack_;
  int source_rank_;
  std::exception_ptr err_;
  c10::intrusive_ptr<c10::ivalue::Future> future_;
};

c10::intrusive_ptr<CommuxWork> completed_work(Engine* e, c10d::OpType op,
                                              std::vector<at::Tensor> outs) {
  return c10::make_intrusive<CommuxWork>(e, op, std::vector<ReqPtr>{}, std::move(outs));
}

// ---------------------------------------------------------------------------
// Host collectives over tagged p2p (collective tag namespace)
// ---------------------------------------------------------------------------

class CollEngine {
 public:
  explicit CollEngine(Engine* e) : e_(e), P_(e->size()), me_(e->rank()) {}

  // User-tag field of collective messages: kind*16 + phase.
  enum Kind : std::uint32_t { kAllreduce = 1, kReduce, kBcast, kBarrier, kAllgather, kGather,
                              kScatter, kRedScat, kAllToAll };

  tag_t tag(Kind k, int phase, std::size_t sub) const {
    return make_ucp_tag(0, static_cast<std::uint32_t>(k) * 16 + static_cast<std::uint32_t>(phase),
                        static_cast<std::uint32_t>(sub), true);
  }

  void wait_all(std::vector<ReqPtr>& reqs) {
    for (auto& r : reqs) e_->wait(r, std::chrono::milliseconds(0));
    reqs.clear();
  }

  ReqPtr send(const at::Tensor& t, int dst, tag_t tg) { return e_->post_send({t}, dst, tg); }
  ReqPtr recv(const at::Tensor& t, int src, tag_t tg) { return e_->post_recv({t}, src, tg); }

  static std::int64_t lo(std::int64_t n, int P, int j) { return n * j / P; }

  // fold_ranks over disjoint element ranges on the engine's copy helpers for
  // large tensors: every element still folds in rank order, so the result is
  // the same bit for bit
  void pfold(at::ScalarType dt, RedOp op, void* out, const void* const* bufs, int nb, std::int64_t n,
             int nranks) {
    const std::int64_t es = static_cast<std::int64_t>(c10::elementSize(dt));
    e_->parallel_ranges(n, std::max<std::int64_t>(1, (512 << 10) / es), [&](std::int64_t a, std::int64_t b) {
      std::vector<const void*> part(static_cast<std::size_t>(nb));
      for (int k = 0; k < nb; ++k) part[k] = static_cast<const char*>(bufs[k]) + a * es;
      fold_ranks(dt, op, static_cast<char*>(out) + a * es, part.data(), nb, b - a, nranks);
    });
  }

  // In-place allreduce of a contiguous 1-D view.
  void allreduce(at::Tensor& t, RedOp op, std::size_t sub) {
    const std::int64_t n = t.numel();
    const auto dt = t.scalar_type();
    const std::int64_t bytes = n * static_cast<std::int64_t>(t.element_size());
    std::vector<ReqPtr> reqs;
    if (bytes <= kSmall || n < P_) {
      // one round: everyone sends its whole buffer to everyone and folds
      std::vector<at::Tensor> tmp(P_);
      std::vector<const void*> bufs(P_);
      at::Tensor mine = t.clone();
      for (int p = 0; p < P_; ++p) {
        if (p == me_) continue;
        tmp[p] = at::empty_like(t);
        reqs.push_back(recv(tmp[p], p, tag(kAllreduce, 0, sub)));
      }
      for (int p = 0; p < P_; ++p)
        if (p != me_) reqs.push_back(send(mine, p, tag(kAllreduce, 0, sub)));
      wait_all(reqs);
      for (int p = 0; p < P_; ++p) bufs[p] = p == me_ ? mine.data_ptr() : tmp[p].data_ptr();
      pfold(dt, op, t.data_ptr(), bufs.data(), P_, n, P_);
      return;
    }
    // reduce-scatter (rank j folds chunk j in rank order) + allgather
    std::int64_t mlo = lo(n, P_, me_), mhi = lo(n, P_, me_ + 1);
    std::vector<at::Tensor> tmp(P_);
    for (int p = 0; p < P_; ++p) {
      if (p == me_) continue;
      tmp[p] = at::empty({mhi - mlo}, t.options());
      reqs.push_back(recv(tmp[p], p, tag(kAllreduce, 1, sub)));
    }
    for (int j = 0; j < P_; ++j)
      if (j != me_) reqs.push_back(send(t.narrow(0, lo(n, P_, j), lo(n, P_, j + 1) - lo(n, P_, j)), j,
                                        tag(kAllreduce, 1, sub)));
    wait_all(reqs);
    at::Tensor own = t.narrow(0, mlo, mhi - mlo);
    std::vector<const void*> bufs(P_);
    for (int p = 0; p < P_; ++p) bufs[p] = p == me_ ? own.data_ptr() : tmp[p].data_ptr();
    pfold(dt, op, own.data_ptr(), bufs.data(), P_, mhi - mlo, P_);
    for (int p = 0; p < P_; ++p)
      if (p != me_)
        reqs.push_back(recv(t.narrow(0, lo(n, P_, p), lo(n, P_, p + 1) - lo(n, P_, p)), p,
                            tag(kAllreduce, 2, sub)));
    for (int p = 0; p < P_; ++p)
      if (p != me_) reqs.push_back(send(own, p, tag(kAllreduce, 2, sub)));
    wait_all(reqs);
  }

  void reduce(at::Tensor& t, RedOp op, int root, std::size_t sub) {
    const std::int64_t n = t.numel();
    const auto dt = t.scalar_type();
    std::vector<ReqPtr> reqs;
    if (me_ != root) {
      reqs.push_back(send(t, root, tag(kReduce, 0, sub)));
      wait_all(reqs);
      return;
    }
    std::vector<at::Tensor> tmp(P_);
    std::vector<const void*> bufs(P_);
    for (int p = 0; p < P_; ++p) {
      if (p == me_) continue;
      tmp[p] = at::empty_like(t);
      reqs.push_back(recv(tmp[p], p, tag(kReduce, 0, sub)));
    }
    wait_all(reqs);
    for (int p = 0; p < P_; ++p) bufs[p] = p == me_ ? t.data_ptr() : tmp[p].data_ptr();
    pfold(dt, op, t.data_ptr(), bufs.data(), P_, n, P_);
  }

  void broadcast(at::Tensor& t, int root, std::size_t sub) {
    std::vector<ReqPtr> reqs;
    if (me_ == root) {
      for (int p = 0; p < P_; ++p)
        if (p != me_) reqs.push_back(send(t, p, tag(kBcast, 0, sub)));
    } else {
      reqs.push_back(recv(t, root, tag(kBcast, 0, sub)));
    }
    wait_all(reqs);
  }

  void barrier() {
    auto token = at::empty({0}, at::TensorOptions().dtype(at::kByte));
    std::vector<ReqPtr> reqs;
    if (me_ == 0) {
      for (int p = 1; p < P_; ++p) reqs.push_back(recv(token, p, tag(kBarrier, 0, 0)));
      wait_all(reqs);
      for (int p = 1; p < P_; ++p) reqs.push_back(send(token, p, tag(kBarrier, 1, 0)));
    } else {
      reqs.push_back(send(token, 0, tag(kBarrier, 0, 0)));
      reqs.push_back(recv(token, 0, tag(kBarrier, 1, 0)));
    }
    wait_all(reqs);
  }

  // outs[p] receives rank p's `in` (outs[me] gets a local copy).
  void allgather(std::vector<at::Tensor>& outs, const at::Tensor& in, std::size_t sub) {
    std::vector<ReqPtr> reqs;
    for (int p = 0; p < P_; ++p)
      if (p != me_) reqs.push_back(recv(outs[p], p, tag(kAllgather, 0, sub)));
    for (int p = 0; p < P_; ++p)
      if (p != me_) reqs.push_back(send(in, p, tag(kAllgather, 0, sub)));
    outs[me_].copy_(in);
    wait_all(reqs);
  }

  void gather(std::vector<at::Tensor>& outs, const at::Tensor& in, int root) {
    std::vector<ReqPtr> reqs;
    if (me_ == root) {
      for (int p = 0; p < P_; ++p)
        if (p != me_) reqs.push_back(recv(outs[p], p, tag(kGather, 0, 0)));
      outs[me_].copy_(in);
    } else {
      reqs.push_back(send(in, root, tag(kGather, 0, 0)));
    }
    wait_all(reqs);
  }

  void scatter(at::Tensor& out, const std::vector<at::Tensor>& ins, int root) {
    std::vector<ReqPtr> reqs;
    if (me_ == root) {
      for (int p = 0; p < P_; ++p)
        if (p != me_) reqs.push_back(send(ins[p], p, tag(kScatter, 0, 0)));
      out.copy_(ins[me_]);
    } else {
      reqs.push_back(recv(out, root, tag(kScatter, 0, 0)));
    }
    wait_all(reqs);
  }

  // out = fold over ranks of ins_p[me] (ins[j] is this rank's block for j).
  void reduce_scatter(at::Tensor& out, const std::vector<at::Tensor>& ins, RedOp op) {
    std::vector<ReqPtr> reqs;
    std::vector<at::Tensor> tmp(P_);
    for (int p = 0; p < P_; ++p) {
      if (p == me_) continue;
      tmp[p] = at::empty_like(out);
      reqs.push_back(recv(tmp[p], p, tag(kRedScat, 0, 0)));
    }
    for (int j = 0; j < P_; ++j)
      if (j != me_) reqs.push_back(send(ins[j], j, tag(kRedScat, 0, 0)));
    wait_all(reqs);
    std::vector<const void*> bufs(P_);
    at::Tensor own = ins[me_].contiguous();
    for (int p = 0; p < P_; ++p) bufs[p] = p == me_ ? own.data_ptr() : tmp[p].data_ptr();
    pfold(out.scalar_type(), op, out.data_ptr(), bufs.data(), P_, out.numel(), P_);
  }

  void alltoall(const std::vector<at::Tensor>& outs, const std::vector<at::Tensor>& ins) {
    std::vector<ReqPtr> reqs;
    for (int p = 0; p < P_; ++p)
      if (p != me_) reqs.push_back(recv(outs[p], p, tag(kAllToAll, 0, 0)));
    for (int p = 0; p < P_; ++p)
      if (p != me_) reqs.push_back(send(ins[p], p, tag(kAllToAll, 0, 0)));
    outs[me_].copy_(ins[me_]);
    wait_all(reqs);
  }

 private:
  static constexpr std::int64_t kSmall = 64 << 10;
  Engine* e_;
  int P_;
  int me_;
};

// ---------------------------------------------------------------------------
// ProcessGroupUCX
// ---------------------------------------------------------------------------

struct GroupWindow {
  std::mutex mu;
  bool open = false;
  struct Deferred {
    bool is_send;
    std::vector<at::Tensor> keep;
    int peer;
    int tag;
  };
  std::vector<Deferred> deferred;
  c10::intrusive_ptr<CommuxWork> pending;
};

ProcessGroupUCX::ProcessGroupUCX(c10::intrusive_ptr<c10d::Store> store, int rank, int size,
                                 std::chrono::milliseconds timeout)
    : c10d::Backend(rank, size), store_(std::move(store)) {
  engine_ = std::make_unique<Engine>(store_, rank, size, timeout);
  coll_ = std::make_unique<CollEngine>(engine_.get());
  group_ = std::make_unique<GroupWindow>();
}

ProcessGroupUCX::~ProcessGroupUCX() {
  group_.reset();
  coll_.reset();
  engine_.reset();
}

void ProcessGroupUCX::setTimeout(std::chrono::milliseconds timeout) { engine_->set_timeout(timeout); }

std::shared_ptr<DevicePlan> ProcessGroupUCX::p2p_plan(
    const std::vector<at::Tensor>& recv_tensors, const std::vector<int>& recv_peers,
    const std::vector<int>& recv_tags, const std::vector<at::Tensor>& send_tensors,
    const std::vector<int>& send_peers, const std::vector<int>& send_tags) {
  TORCH_CHECK(recv_tensors.size() == recv_peers.size() && recv_peers.size() == recv_tags.size() &&
                  send_tensors.size() == send_peers.size() && send_peers.size() == send_tags.size(),
              "commux p2p_plan: tensors, peers and tags must have equal lengths");
  for (auto* v : {&recv_tensors, &send_tensors})
    for (auto& t : *v)
      TORCH_CHECK(t.is_cuda(), "commux p2p_plan: persistent plans take CUDA tensors (use batch_p2p on CPU)");
  for (auto* v : {&recv_peers, &send_peers})
    for (int p : *v)
      TORCH_CHECK(p >= 0 && p < getSize() && !engine_->remote(p), "commux p2p_plan: rank ", p,
                  " is not on this host (persistent plans map peer memory; use batch_p2p)");
  return engine_->device()->create_plan(recv_tensors, recv_peers, recv_tags, send_tensors, send_peers,
                                        send_tags);
}

bool ProcessGroupUCX::device_coll(const at::Tensor& t) {
  // peers on other hosts: the device kernels need every peer's memory mapped
  if (engine_->any_remote()) return false;
  return engine_->device()->device_collectives(t.device().index());
}

std::vector<at::Tensor> ProcessGroupUCX::to_host(const std::vector<at::Tensor>& ts) {
  // Host staging for ranks that share a GPU (the device collectives would
  // need kernels of two processes to wait on each other on one GPU) and for
  // groups that span hosts.
  std::vector<at::Tensor> h;
  for (auto& t : ts) h.push_back(t.cpu().contiguous());
  return h;
}

void ProcessGroupUCX::from_host(std::vector<at::Tensor>& ts, const std::vector<at::Tensor>& h) {
  for (std::size_t i = 0; i < ts.size(); ++i) ts[i].copy_(h[i]);
}

c10::intrusive_ptr<c10d::Backend::Options> ProcessGroupUCX::getBackendOptions() {
  return c10::make_intrusive<c10d::Backend::Options>("ucx", engine_->timeout());
}

void ProcessGroupUCX::abort() { engine_->abort_group("abort() called"); }
void ProcessGroupUCX::shutdown() {}

std::vector<std::pair<std::string, std::int64_t>> ProcessGroupUCX::stats() const {
  auto& s = engine_->stats();
  std::vector<std::pair<std::string, std::int64_t>> v = {
      {"sends", s.sends.load()},
      {"recvs", s.recvs.load()},
      {"bytes_sent", s.bytes_sent.load()},
      {"bytes_recv", s.bytes_recv.load()},
      {"eager_msgs", s.eager_msgs.load()},
      {"rndv_msgs", s.rndv_msgs.load()},
      {"device_msgs", s.device_msgs.load()},
      {"unexpected_msgs", s.unexpected_msgs.load()},
      {"unexpected_peak", s.unexpected_peak.load()},
      {"ring_full_stalls", s.ring_full_stalls.load()},
      {"futex_sleeps", s.futex_sleeps.load()},
      {"records_in", s.records_in.load()},
      {"records_out", s.records_out.load()},
      {"host_copies", s.host_copies.load()},
      {"single_copy_msgs", s.single_copy_msgs.load()},
      {"faults_injected", s.faults_injected.load()},
  };
  for (auto& kv : engine_->gauges()) v.push_back(kv);
  if (auto* d = engine_->device(false))
    for (auto& kv : d->stats()) v.push_back(kv);
  return v;
}

void ProcessGroupUCX::reset_stats() {
  auto& s = engine_->stats();
  for (auto* a : {&s.sends, &s.recvs, &s.bytes_sent, &s.bytes_recv, &s.eager_msgs, &s.rndv_msgs,
                  &s.device_msgs, &s.unexpected_msgs, &s.unexpected_peak, &s.ring_full_stalls,
                  &s.futex_sleeps, &s.records_in, &s.records_out, &s.host_copies, &s.single_copy_msgs,
                  &s.faults_injected})
    a->store(0);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::post_p2p(std::vector<at::Tensor>& tensors, int peer,
                                                         int tag, bool is_send) {
  const int P = getSize();
  TORCH_CHECK(peer >= 0 && peer < P, "commux ", is_send ? "send" : "recv", ": invalid ",
              is_send ? "dst" : "src", " rank ", peer);
  check_same_device_kind(tensors, is_send ? "send" : "recv");
  auto& g = *group_;
  std::unique_lock<std::mutex> glk(g.mu);
  if (g.open && group_enabled()) {
    GroupWindow::Deferred d;
    d.is_send = is_send;
    d.peer = peer;
    d.tag = tag;
    for (auto& t : tensors) {
      if (is_send) {
        d.keep.push_back(t.is_contiguous() || t.is_cuda() ? t : t.contiguous());
      } else if (t.is_cuda() || t.is_contiguous()) {
        d.keep.push_back(t);
      } else {
        at::Tensor tmp = at::empty(t.sizes(), t.options());
        g.pending->add_unpack(tmp, t);
        d.keep.push_back(tmp);
      }
    }
    g.deferred.push_back(std::move(d));
    return g.pending;
  }
  glk.unlock();

  std::vector<ReqPtr> reqs;
  std::vector<std::pair<at::Tensor, at::Tensor>> unpack;
  post_now(tensors, peer, tag, is_send, reqs, unpack);
  auto work = c10::make_intrusive<CommuxWork>(engine_.get(), is_send ? c10d::OpType::SEND : c10d::OpType::RECV,
                                              reqs, is_send ? std::vector<at::Tensor>{} : tensors);
  for (auto& tv : unpack) work->add_unpack(tv.first, tv.second);
  glk.lock();
  if (g.open && g.pending) {
    g.pending->add(reqs, {});
    for (auto& tv : unpack) g.pending->add_unpack(tv.first, tv.second);
  }
  return work;
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::batch_p2p(
    std::vector<at::Tensor>& recv_tensors, const std::vector<int>& recv_peers,
    const std::vector<int>& recv_tags, std::vector<at::Tensor>& send_tensors,
    const std::vector<int>& send_peers, const std::vector<int>& send_tags) {
  TraceRange trace_("commux.batch_p2p");
  TORCH_CHECK(recv_tensors.size() == recv_peers.size() && recv_peers.size() == recv_tags.size() &&
                  send_tensors.size() == send_peers.size() && send_peers.size() == send_tags.size(),
              "commux batch_p2p: tensors, peers and tags must have equal lengths");
  const int P = getSize();
  bool any_cuda = false;
  for (auto* v : {&recv_tensors, &send_tensors})
    for (auto& t : *v) any_cuda |= t.is_cuda();
  auto work = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::COALESCED,
                                              std::vector<ReqPtr>{}, recv_tensors);
  DeviceTransport* dev = any_cuda ? engine_->device() : nullptr;
  if (dev) dev->begin_batch();
  try {
    for (int pass = 0; pass < 2; ++pass) {
      const bool is_send = pass == 1;
      auto& ts = is_send ? send_tensors : recv_tensors;
      auto& peers = is_send ? send_peers : recv_peers;
      auto& tags = is_send ? send_tags : recv_tags;
      for (std::size_t i = 0; i < ts.size(); ++i) {
        TORCH_CHECK(peers[i] >= 0 && peers[i] < P, "commux batch_p2p: invalid peer rank ", peers[i]);
        std::vector<at::Tensor> one{ts[i]};
        std::vector<ReqPtr> reqs;
        std::vector<std::pair<at::Tensor, at::Tensor>> unpack;
        post_now(one, peers[i], tags[i], is_send, reqs, unpack);
        work->add(reqs, {});
        for (auto& tv : unpack) work->add_unpack(tv.first, tv.second);
      }
    }
  } catch (...) {
    if (dev) dev->end_batch();
    throw;
  }
  if (dev) dev->end_batch();
  return work;
}

void ProcessGroupUCX::post_now(std::vector<at::Tensor>& tensors, int peer, int tag, bool is_send,
                               std::vector<ReqPtr>& reqs,
                               std::vector<std::pair<at::Tensor, at::Tensor>>& unpack) {
  std::vector<at::Tensor> keep;
  keep.reserve(tensors.size());
  // CUDA tensors to or from a rank on another host travel through host
  // memory (the TCP transport carries host bytes only)
  const bool stage = peer >= 0 ? engine_->remote(peer) : engine_->any_remote();
  for (auto& t : tensors) {
    // CPU sends go from a contiguous copy (the reference does the same,
    // :586-588); CPU receives into strided views land in a contiguous temp.
    // CUDA sends and receives may be strided views: the device transport
    // gathers and scatters inside its copy kernel.
    if (t.is_cuda() && stage) {
      if (is_send) {
        keep.push_back(t.to(at::kCPU).contiguous());
      } else {
        at::Tensor tmp = at::empty(t.sizes(), t.options().device(at::kCPU));
        unpack.push_back({tmp, t});
        keep.push_back(tmp);
      }
    } else if (t.is_cuda()) {
      keep.push_back(t);
    } else if (is_send) {
      keep.push_back(t.contiguous());
    } else if (t.is_contiguous()) {
      keep.push_back(t);
    } else {
      at::Tensor tmp = at::empty(t.sizes(), t.options());
      unpack.push_back({tmp, t});
      keep.push_back(tmp);
    }
  }
  const std::uint32_t ut = static_cast<std::uint32_t>(tag);
  if (keep.size() > 1 && coalesce_enabled()) {
    // one message for the whole vector, sub-index 0 (both sides decide from
    // tensor metadata only, so they always agree on the layout)
    tag_t tg = make_ucp_tag(0, ut, 0, false);
    reqs.push_back(is_send ? engine_->post_send(keep, peer, tg) : engine_->post_recv(keep, peer, tg));
  } else {
    for (std::size_t i = 0; i < keep.size(); ++i) {
      tag_t tg = make_ucp_tag(0, ut, static_cast<std::uint32_t>(i), false);
      reqs.push_back(is_send ? engine_->post_send({keep[i]}, peer, tg)
                             : engine_->post_recv({keep[i]}, peer, tg));
    }
  }
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::send(std::vector<at::Tensor>& tensors, int dstRank,
                                                     int tag) {
  TraceRange trace_("commux.send");
  return post_p2p(tensors, dstRank, tag, true);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::recv(std::vector<at::Tensor>& tensors, int srcRank,
                                                     int tag) {
  TraceRange trace_("commux.recv");
  return post_p2p(tensors, srcRank, tag, false);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::recvAnysource(std::vector<at::Tensor>& tensors,
                                                              int tag) {
  TraceRange trace_("commux.recvAnysource");
  check_same_device_kind(tensors, "recvAnysource");
  if (tensors[0].is_cuda() && engine_->any_remote()) {
    // a sender on another host sends host bytes: receive into host temps
    std::vector<at::Tensor> host;
    for (auto& t : tensors) host.push_back(at::empty(t.sizes(), t.options().device(at::kCPU)));
    auto w = c10::static_intrusive_pointer_cast<CommuxWork>(recvAnysource(host, tag));
    for (std::size_t i = 0; i < tensors.size(); ++i) w->add_unpack(host[i], tensors[i]);
    return w;
  }
  // Non-blocking here (the reference probes and blocks, :696-732); the source
  // is known once the first tensor has matched. Tensor i > 0 is then received
  // from that same source, as the sender sends the whole vector.
  std::vector<ReqPtr> reqs;
  const std::uint32_t ut = static_cast<std::uint32_t>(tag);
  if (tensors.size() > 1 && coalesce_enabled()) {
    reqs.push_back(engine_->post_recv(tensors, -1, make_ucp_tag(0, ut, 0, false)));
  } else {
    reqs.push_back(engine_->post_recv({tensors[0]}, -1, make_ucp_tag(0, ut, 0, false)));
    if (tensors.size() > 1) {
      engine_->wait(reqs[0], std::chrono::milliseconds(0));
      int src = reqs[0]->source;
      for (std::size_t i = 1; i < tensors.size(); ++i)
        reqs.push_back(
            engine_->post_recv({tensors[i]}, src, make_ucp_tag(0, ut, static_cast<std::uint32_t>(i), false)));
    }
  }
  return c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::RECVANYSOURCE, reqs, tensors);
}

void ProcessGroupUCX::startCoalescing() {
  auto& g = *group_;
  std::lock_guard<std::mutex> lk(g.mu);
  g.open = true;
  g.deferred.clear();
  g.pending = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::COALESCED,
                                              std::vector<ReqPtr>{}, std::vector<at::Tensor>{});
  if (group_enabled()) {
    // nothing posted yet
  }
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::endCoalescing() {
  TraceRange trace_("commux.endCoalescing");
  auto& g = *group_;
  std::vector<GroupWindow::Deferred> deferred;
  c10::intrusive_ptr<CommuxWork> work;
  {
    std::lock_guard<std::mutex> lk(g.mu);
    if (!g.open) return completed_work(engine_.get(), c10d::OpType::COALESCED, {});
    g.open = false;
    deferred = std::move(g.deferred);
    g.deferred.clear();
    work = std::move(g.pending);
    g.pending.reset();
  }
  if (deferred.empty()) return work;
  // Flush the window: every op keeps its usual per-tensor tags, so a grouping
  // rank interoperates with a non-grouping peer (reference :825-883).
  bool any_cuda = false;
  for (auto& d : deferred)
    for (auto& t : d.keep) any_cuda |= t.is_cuda();
  DeviceTransport* dev = any_cuda ? engine_->device() : nullptr;
  if (dev) dev->begin_batch();
  try {
    for (auto& d : deferred) {
      std::vector<ReqPtr> reqs;
      std::vector<std::pair<at::Tensor, at::Tensor>> unpack;
      post_now(d.keep, d.peer, d.tag, d.is_send, reqs, unpack);
      work->add(reqs, d.is_send ? std::vector<at::Tensor>{} : d.keep);
      for (auto& tv : unpack) work->add_unpack(tv.first, tv.second);
    }
  } catch (...) {
    if (dev) dev->end_batch();
    throw;
  }
  if (dev) dev->end_batch();
  return work;
}

// ---------------------------------------------------------------------------
// collectives
// ---------------------------------------------------------------------------

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::allreduce(std::vector<at::Tensor>& tensors,
                                                          const c10d::AllreduceOptions& opts) {
  TraceRange trace_("commux.allreduce");
  check_same_device_kind(tensors, "allreduce");
  RedOp op = validate_op(opts.reduceOp, tensors, "allreduce");
  if (tensors[0].is_cuda()) {
    if (getSize() == 1) return completed_work(engine_.get(), c10d::OpType::ALLREDUCE, tensors);
    if (!device_coll(tensors[0])) {
      std::vector<at::Tensor> h = to_host(tensors);
      allreduce(h, opts);
      from_host(tensors, h);
      return completed_work(engine_.get(), c10d::OpType::ALLREDUCE, tensors);
    }
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::ALLREDUCE,
                                             std::vector<ReqPtr>{}, tensors);
    w->add_device(engine_->device()->allreduce(tensors, op));
    return w;
  }
  if (getSize() > 1) {
    for (std::size_t i = 0; i < tensors.size(); ++i) {
      at::Tensor& t = tensors[i];
      at::Tensor flat = t.is_contiguous() ? t.view({-1}) : t.contiguous().view({-1});
      coll_->allreduce(flat, op, i);
      if (!t.is_contiguous()) t.copy_(flat.view(t.sizes()));
    }
  }
  return completed_work(engine_.get(), c10d::OpType::ALLREDUCE, tensors);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::allreduce_coalesced(
    std::vector<at::Tensor>& tensors, const c10d::AllreduceCoalescedOptions& opts) {
  TraceRange trace_("commux.allreduce_coalesced");
  c10d::AllreduceOptions o;
  o.reduceOp = opts.reduceOp;
  o.timeout = opts.timeout;
  return allreduce(tensors, o);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::reduce(std::vector<at::Tensor>& tensors,
                                                       const c10d::ReduceOptions& opts) {
  TraceRange trace_("commux.reduce");
  check_same_device_kind(tensors, "reduce");
  RedOp op = validate_op(opts.reduceOp, tensors, "reduce");
  int root = static_cast<int>(opts.rootRank);
  TORCH_CHECK(root >= 0 && root < getSize(), "commux reduce: root out of range");
  if (tensors[0].is_cuda()) {
    if (getSize() == 1) return completed_work(engine_.get(), c10d::OpType::REDUCE, tensors);
    if (!device_coll(tensors[0])) {
      std::vector<at::Tensor> h = to_host(tensors);
      reduce(h, opts);
      if (getRank() == root) from_host(tensors, h);
      return completed_work(engine_.get(), c10d::OpType::REDUCE, tensors);
    }
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::REDUCE,
                                             std::vector<ReqPtr>{}, tensors);
    w->add_device(engine_->device()->reduce(tensors, op, root));
    return w;
  }
  if (getSize() > 1) {
    for (std::size_t i = 0; i < tensors.size(); ++i) {
      at::Tensor& t = tensors[i];
      TORCH_CHECK(t.is_contiguous(), "commux reduce: tensor must be contiguous");
      at::Tensor flat = t.view({-1});
      coll_->reduce(flat, op, root, i);
    }
  }
  return completed_work(engine_.get(), c10d::OpType::REDUCE, tensors);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::broadcast(std::vector<at::Tensor>& tensors,
                                                          const c10d::BroadcastOptions& opts) {
  TraceRange trace_("commux.broadcast");
  check_same_device_kind(tensors, "broadcast");
  int root = static_cast<int>(opts.rootRank);
  TORCH_CHECK(root >= 0 && root < getSize(), "commux broadcast: root out of range");
  if (tensors[0].is_cuda()) {
    if (getSize() == 1) return completed_work(engine_.get(), c10d::OpType::BROADCAST, tensors);
    if (!device_coll(tensors[0])) {
      std::vector<at::Tensor> h = to_host(tensors);
      broadcast(h, opts);
      from_host(tensors, h);
      return completed_work(engine_.get(), c10d::OpType::BROADCAST, tensors);
    }
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::BROADCAST,
                                             std::vector<ReqPtr>{}, tensors);
    w->add_device(engine_->device()->broadcast(tensors, root));
    return w;
  }
  if (getSize() > 1) {
    for (std::size_t i = 0; i < tensors.size(); ++i) {
      at::Tensor& t = tensors[i];
      TORCH_CHECK(t.is_contiguous(), "commux broadcast: tensor must be contiguous");
      coll_->broadcast(t, root, i);
    }
  }
  return completed_work(engine_.get(), c10d::OpType::BROADCAST, tensors);
}

// The reference's barrier is a token reduce + broadcast over its transport
// (reference: src/process_group_ucx.cpp:813-823). Here: a group whose device
// collectives are set up (or a call naming device_ids) runs a device flag
// round on the current stream, ordered after the work already on it, and
// the call returns once every rank's stream reached it -- so what any
// rank's kernels wrote before the barrier is visible to every rank's kernels
// after it. Other groups use the host barrier over shared memory.
c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::barrier(const c10d::BarrierOptions& opts) {
  TraceRange trace_("commux.barrier");
  if (getSize() == 1) return completed_work(engine_.get(), c10d::OpType::BARRIER, {});
  DeviceTransport* dev = engine_->any_remote() ? nullptr : engine_->device(false);
  bool on_device = dev != nullptr && dev->collectives_ready();
  if (!on_device && !opts.device_ids.empty() && !engine_->any_remote()) {
    const auto idx = static_cast<c10::DeviceIndex>(opts.device_ids[0]);
    at::Tensor probe = at::empty({0}, at::TensorOptions().device(at::kCUDA, idx));
    on_device = device_coll(probe);
    dev = engine_->device(false);
  }
  if (!on_device) {
    coll_->barrier();
    return completed_work(engine_.get(), c10d::OpType::BARRIER, {});
  }
  DevCollPtr r = dev->barrier();
  r->stream_wait();
  r->host_wait();
  std::string e = r->error();
  if (!e.empty()) C10_THROW_ERROR(DistBackendError, "commux barrier: " + e);
  return completed_work(engine_.get(), c10d::OpType::BARRIER, {});
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::allgather(
    std::vector<std::vector<at::Tensor>>& outputTensors, std::vector<at::Tensor>& inputTensors,
    const c10d::AllgatherOptions& /*opts*/) {
  TraceRange trace_("commux.allgather");
  TORCH_CHECK(inputTensors.size() == 1 && outputTensors.size() == 1,
              "commux allgather: one input tensor and one output list per call");
  auto& outs = outputTensors[0];
  auto& in = inputTensors[0];
  TORCH_CHECK(static_cast<int>(outs.size()) == getSize(), "commux allgather: output list needs ",
              getSize(), " tensors");
  for (auto& o : outs)
    TORCH_CHECK(o.numel() == in.numel() && o.scalar_type() == in.scalar_type(),
                "commux allgather: output tensors must match the input's numel and dtype");
  if (in.is_cuda()) {
    if (getSize() > 1 && !device_coll(in)) {
      std::vector<std::vector<at::Tensor>> ho{to_host(outs)};
      std::vector<at::Tensor> hi = to_host(inputTensors);
      allgather(ho, hi, c10d::AllgatherOptions());
      from_host(outs, ho[0]);
      return completed_work(engine_.get(), c10d::OpType::ALLGATHER, outs);
    }
    // gather into one flat buffer on the device, then split into the list
    at::Tensor flat = at::empty({getSize() * in.numel()}, in.options());
    at::Tensor src = in.contiguous().view({-1});
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::ALLGATHER,
                                             std::vector<ReqPtr>{}, outs);
    if (getSize() > 1) {
      auto d = engine_->device()->allgather(flat, src);
      d->stream_wait();
      w->add_device(d);
    } else {
      flat.copy_(src);
    }
    for (int p = 0; p < getSize(); ++p)
      outs[p].copy_(flat.narrow(0, p * in.numel(), in.numel()).view(outs[p].sizes()));
    return w;
  }
  std::vector<at::Tensor> douts;
  for (auto& o : outs) douts.push_back(o.is_contiguous() ? o : at::empty_like(o, at::MemoryFormat::Contiguous));
  at::Tensor src = in.contiguous();
  if (getSize() > 1)
    coll_->allgather(douts, src, 0);
  else
    douts[0].copy_(src);
  for (std::size_t p = 0; p < outs.size(); ++p)
    if (!outs[p].is_same(douts[p])) outs[p].copy_(douts[p]);
  return completed_work(engine_.get(), c10d::OpType::ALLGATHER, outs);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::_allgather_base(at::Tensor& outputBuffer,
                                                                at::Tensor& inputBuffer,
                                                                const c10d::AllgatherOptions& /*opts*/) {
  TraceRange trace_("commux.allgather_base");
  TORCH_CHECK(outputBuffer.numel() == inputBuffer.numel() * getSize(),
              "commux _allgather_base: output must hold world_size * input elements");
  TORCH_CHECK(outputBuffer.is_contiguous(), "commux _allgather_base: output must be contiguous");
  at::Tensor flat = outputBuffer.view({-1});
  at::Tensor src = inputBuffer.contiguous().view({-1});
  if (inputBuffer.is_cuda()) {
    if (getSize() > 1 && !device_coll(inputBuffer)) {
      at::Tensor ho = outputBuffer.cpu(), hi = inputBuffer.cpu();
      _allgather_base(ho, hi, c10d::AllgatherOptions());
      outputBuffer.copy_(ho);
      return completed_work(engine_.get(), c10d::OpType::_ALLGATHER_BASE, {outputBuffer});
    }
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::_ALLGATHER_BASE,
                                             std::vector<ReqPtr>{}, std::vector<at::Tensor>{outputBuffer});
    if (getSize() > 1)
      w->add_device(engine_->device()->allgather(flat, src));
    else
      flat.copy_(src);
    return w;
  }
  std::vector<at::Tensor> outs;
  for (int p = 0; p < getSize(); ++p) outs.push_back(flat.narrow(0, p * src.numel(), src.numel()));
  if (getSize() > 1)
    coll_->allgather(outs, src, 0);
  else
    outs[0].copy_(src);
  return completed_work(engine_.get(), c10d::OpType::_ALLGATHER_BASE, {outputBuffer});
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::allgather_into_tensor_coalesced(
    std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
    const c10d::AllgatherOptions& opts) {
  TraceRange trace_("commux.allgather_coalesced");
  TORCH_CHECK(outputs.size() == inputs.size(), "commux allgather_into_tensor_coalesced: size mismatch");
  c10::intrusive_ptr<c10d::Work> last;
  auto agg = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::COALESCED,
                                             std::vector<ReqPtr>{}, outputs);
  for (std::size_t i = 0; i < inputs.size(); ++i) {
    auto w = _allgather_base(outputs[i], inputs[i], opts);
    w->wait();
  }
  return agg;
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::gather(std::vector<std::vector<at::Tensor>>& outputTensors,
                                                       std::vector<at::Tensor>& inputTensors,
                                                       const c10d::GatherOptions& opts) {
  TraceRange trace_("commux.gather");
  TORCH_CHECK(inputTensors.size() == 1, "commux gather: one input tensor");
  int root = static_cast<int>(opts.rootRank);
  TORCH_CHECK(!inputTensors[0].is_cuda(), "commux gather: CUDA tensors are not supported; use allgather");
  std::vector<at::Tensor> outs;
  if (getRank() == root) {
    TORCH_CHECK(outputTensors.size() == 1 && static_cast<int>(outputTensors[0].size()) == getSize(),
                "commux gather: root needs world_size output tensors");
    for (auto& o : outputTensors[0]) {
      TORCH_CHECK(o.is_contiguous(), "commux gather: outputs must be contiguous");
      outs.push_back(o);
    }
  }
  at::Tensor in = inputTensors[0].contiguous();
  if (getSize() > 1)
    coll_->gather(outs, in, root);
  else if (!outs.empty())
    outs[0].copy_(in);
  return completed_work(engine_.get(), c10d::OpType::GATHER, outs);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::scatter(std::vector<at::Tensor>& outputTensors,
                                                        std::vector<std::vector<at::Tensor>>& inputTensors,
                                                        const c10d::ScatterOptions& opts) {
  TraceRange trace_("commux.scatter");
  TORCH_CHECK(outputTensors.size() == 1, "commux scatter: one output tensor");
  TORCH_CHECK(!outputTensors[0].is_cuda(), "commux scatter: CUDA tensors are not supported");
  int root = static_cast<int>(opts.rootRank);
  std::vector<at::Tensor> ins;
  if (getRank() == root) {
    TORCH_CHECK(inputTensors.size() == 1 && static_cast<int>(inputTensors[0].size()) == getSize(),
                "commux scatter: root needs world_size input tensors");
    for (auto& t : inputTensors[0]) ins.push_back(t.contiguous());
  }
  TORCH_CHECK(outputTensors[0].is_contiguous(), "commux scatter: output must be contiguous");
  if (getSize() > 1)
    coll_->scatter(outputTensors[0], ins, root);
  else
    outputTensors[0].copy_(ins[0]);
  return completed_work(engine_.get(), c10d::OpType::SCATTER, outputTensors);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::reduce_scatter(
    std::vector<at::Tensor>& outputTensors, std::vector<std::vector<at::Tensor>>& inputTensors,
    const c10d::ReduceScatterOptions& opts) {
  TraceRange trace_("commux.reduce_scatter");
  TORCH_CHECK(outputTensors.size() == 1 && inputTensors.size() == 1, "commux reduce_scatter: one output");
  auto& out = outputTensors[0];
  RedOp op = validate_op(opts.reduceOp, {out}, "reduce_scatter");
  TORCH_CHECK(static_cast<int>(inputTensors[0].size()) == getSize(),
              "commux reduce_scatter: needs world_size inputs");
  if (out.is_cuda()) {
    if (getSize() == 1 || !device_coll(out)) {
      std::vector<at::Tensor> ho = to_host(outputTensors);
      std::vector<std::vector<at::Tensor>> hi{to_host(inputTensors[0])};
      reduce_scatter(ho, hi, opts);
      from_host(outputTensors, ho);
      return completed_work(engine_.get(), c10d::OpType::REDUCE_SCATTER, outputTensors);
    }
    at::Tensor flat = at::empty({getSize() * out.numel()}, out.options());
    for (int p = 0; p < getSize(); ++p)
      flat.narrow(0, p * out.numel(), out.numel()).copy_(inputTensors[0][p].reshape({-1}));
    at::Tensor o = out.is_contiguous() ? out.view({-1}) : at::empty({out.numel()}, out.options());
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::REDUCE_SCATTER,
                                             std::vector<ReqPtr>{}, outputTensors);
    w->add_device(engine_->device()->reduce_scatter(o, flat, op));
    if (!out.is_contiguous()) {
      w->wait();
      out.copy_(o.view(out.sizes()));
    }
    return w;
  }
  TORCH_CHECK(out.is_contiguous(), "commux reduce_scatter: output must be contiguous");
  std::vector<at::Tensor> ins;
  for (auto& t : inputTensors[0]) ins.push_back(t.contiguous());
  if (getSize() > 1)
    coll_->reduce_scatter(out, ins, op);
  else {
    const void* b = ins[0].data_ptr();
    fold_ranks(out.scalar_type(), op, out.data_ptr(), &b, 1, out.numel(), 1);
  }
  return completed_work(engine_.get(), c10d::OpType::REDUCE_SCATTER, outputTensors);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::_reduce_scatter_base(at::Tensor& outputBuffer,
                                                                     at::Tensor& inputBuffer,
                                                                     const c10d::ReduceScatterOptions& opts) {
  TraceRange trace_("commux.reduce_scatter_base");
  TORCH_CHECK(inputBuffer.numel() == outputBuffer.numel() * getSize(),
              "commux _reduce_scatter_base: input must hold world_size * output elements");
  RedOp op = validate_op(opts.reduceOp, {outputBuffer}, "reduce_scatter");
  if (outputBuffer.is_cuda() && (getSize() == 1 || !device_coll(outputBuffer))) {
    at::Tensor ho = outputBuffer.cpu(), hi = inputBuffer.cpu();
    _reduce_scatter_base(ho, hi, opts);
    outputBuffer.copy_(ho);
    return completed_work(engine_.get(), c10d::OpType::_REDUCE_SCATTER_BASE, {outputBuffer});
  }
  if (outputBuffer.is_cuda()) {
    TORCH_CHECK(outputBuffer.is_contiguous(), "commux _reduce_scatter_base: output must be contiguous");
    at::Tensor o = outputBuffer.view({-1});
    at::Tensor in = inputBuffer.contiguous().view({-1});
    auto w = c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::_REDUCE_SCATTER_BASE,
                                             std::vector<ReqPtr>{}, std::vector<at::Tensor>{outputBuffer});
    w->add_device(engine_->device()->reduce_scatter(o, in, op));
    return w;
  }
  at::Tensor flat = inputBuffer.contiguous().view({-1});
  std::vector<at::Tensor> ins;
  for (int p = 0; p < getSize(); ++p)
    ins.push_back(flat.narrow(0, p * outputBuffer.numel(), outputBuffer.numel()));
  std::vector<at::Tensor> outs{outputBuffer};
  std::vector<std::vector<at::Tensor>> vin{ins};
  return reduce_scatter(outs, vin, opts);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::alltoall_base(at::Tensor& outputBuffer,
                                                              at::Tensor& inputBuffer,
                                                              std::vector<int64_t>& outputSplitSizes,
                                                              std::vector<int64_t>& inputSplitSizes,
                                                              const c10d::AllToAllOptions& /*opts*/) {
  TraceRange trace_("commux.alltoall");
  const int P = getSize();
  TORCH_CHECK(outputBuffer.is_contiguous(), "commux alltoall: output must be contiguous");
  at::Tensor in = inputBuffer.contiguous();
  auto split = [&](const at::Tensor& t, const std::vector<int64_t>& sizes) {
    std::vector<at::Tensor> parts;
    std::int64_t row = t.dim() > 0 ? t.numel() / std::max<std::int64_t>(1, t.size(0)) : 1;
    std::int64_t off = 0;
    for (int p = 0; p < P; ++p) {
      std::int64_t rows = sizes.empty() ? t.size(0) / P : sizes[p];
      parts.push_back(t.view({-1}).narrow(0, off * row, rows * row));
      off += rows;
    }
    return parts;
  };
  if (outputBuffer.is_cuda() && engine_->any_remote()) {
    // a group spanning hosts: stage through host memory
    at::Tensor hin = in.cpu(), hout = at::empty(outputBuffer.sizes(), outputBuffer.options().device(at::kCPU));
    auto w = alltoall_base(hout, hin, outputSplitSizes, inputSplitSizes, c10d::AllToAllOptions());
    w->wait();
    outputBuffer.copy_(hout);
    return completed_work(engine_.get(), c10d::OpType::ALLTOALL_BASE, {outputBuffer});
  }
  auto outs = split(outputBuffer, outputSplitSizes);
  auto ins = split(in, inputSplitSizes);
  if (outputBuffer.is_cuda()) {
    // tagged device p2p: one batch of sends and receives
    auto* dev = engine_->device();
    dev->begin_batch();
    std::vector<ReqPtr> reqs;
    for (int p = 0; p < P; ++p) {
      tag_t tg = make_ucp_tag(0, CollEngine::kAllToAll * 16, 0, true);
      reqs.push_back(engine_->post_recv({outs[p]}, p, tg));
      reqs.push_back(engine_->post_send({ins[p]}, p, tg));
    }
    dev->end_batch();
    return c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::ALLTOALL_BASE, reqs,
                                           std::vector<at::Tensor>{outputBuffer});
  }
  if (P > 1)
    coll_->alltoall(outs, ins);
  else
    outs[0].copy_(ins[0]);
  return completed_work(engine_.get(), c10d::OpType::ALLTOALL_BASE, {outputBuffer});
}

c10::intrusive_ptr<c10d::Work> ProcessGroupUCX::alltoall(std::vector<at::Tensor>& outputTensors,
                                                         std::vector<at::Tensor>& inputTensors,
                                                         const c10d::AllToAllOptions& /*opts*/) {
  TraceRange trace_("commux.alltoall_list");
  const int P = getSize();
  TORCH_CHECK(static_cast<int>(outputTensors.size()) == P && static_cast<int>(inputTensors.size()) == P,
              "commux alltoall: needs world_size input and output tensors");
  check_same_device_kind(outputTensors, "alltoall");
  check_same_device_kind(inputTensors, "alltoall");
  TORCH_CHECK(outputTensors[0].is_cuda() == inputTensors[0].is_cuda(),
              "commux alltoall: inputs and outputs must live on the same kind of device");
  if (outputTensors[0].is_cuda() && engine_->any_remote()) {
    // a group spanning hosts: stage through host memory
    std::vector<at::Tensor> hout, hin;
    for (int p = 0; p < P; ++p) {
      hout.push_back(at::empty(outputTensors[p].sizes(), outputTensors[p].options().device(at::kCPU)));
      hin.push_back(inputTensors[p].cpu());
    }
    alltoall(hout, hin, c10d::AllToAllOptions())->wait();
    for (int p = 0; p < P; ++p) outputTensors[p].copy_(hout[p]);
    return completed_work(engine_.get(), c10d::OpType::ALLTOALL, outputTensors);
  }
  const tag_t tg = make_ucp_tag(0, CollEngine::kAllToAll * 16 + 1, 0, true);
  if (outputTensors[0].is_cuda()) {
    // tagged device p2p, one batch (strided views are gathered and scattered
    // inside the copy)
    auto* dev = engine_->device();
    dev->begin_batch();
    std::vector<ReqPtr> reqs;
    try {
      for (int p = 0; p < P; ++p) {
        reqs.push_back(engine_->post_recv({outputTensors[p]}, p, tg));
        reqs.push_back(engine_->post_send({inputTensors[p]}, p, tg));
      }
    } catch (...) {
      dev->end_batch();
      throw;
    }
    dev->end_batch();
    return c10::make_intrusive<CommuxWork>(engine_.get(), c10d::OpType::ALLTOALL, reqs, outputTensors);
  }
  // host: contiguous sends, contiguous temps for strided outputs
  std::vector<at::Tensor> outs(P), ins(P);
  for (int p = 0; p < P; ++p) {
    ins[p] = inputTensors[p].contiguous();
    outs[p] = outputTensors[p].is_contiguous() ? outputTensors[p] : at::empty(outputTensors[p].sizes(),
                                                                               outputTensors[p].options());
  }
  std::vector<ReqPtr> reqs;
  for (int p = 0; p < P; ++p)
    if (p != getRank()) reqs.push_back(engine_->post_recv({outs[p]}, p, tg));
  for (int p = 0; p < P; ++p)
    if (p != getRank()) reqs.push_back(engine_->post_send({ins[p]}, p, tg));
  outs[getRank()].copy_(ins[getRank()]);
  for (auto& r : reqs) engine_->wait(r, std::chrono::milliseconds(0));
  for (int p = 0; p < P; ++p)
    if (!outs[p].is_same(outputTensors[p])) outputTensors[p].copy_(outs[p]);
  return completed_work(engine_.get(), c10d::OpType::ALLTOALL, outputTensors);
}

}  // namespace commux
