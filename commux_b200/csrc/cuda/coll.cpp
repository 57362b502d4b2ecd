#include "coll.hpp"

#include "engine/log.hpp"

#include <ATen/core/ivalue.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace commux {
namespace cuda {

namespace {

cudaStream_t current_stream(int dev) {
  return c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream();
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat:
      return kF32;
    case at::kDouble:
      return kF64;
    case at::kHalf:
      return kF16;
    case at::kBFloat16:
      return kBF16;
    case at::kInt:
      return kI32;
    case at::kLong:
      return kI64;
    case at::kByte:
    case at::kBool:
      return kU8;
    case at::kChar:
      return kI8;
    default:
      throw std::runtime_error(std::string("commux: unsupported dtype for a CUDA collective: ") +
                               c10::toString(t));
  }
}

int op_code(RedOp op) { return static_cast<int>(op); }

struct ExchangeRecord {
  std::int32_t pid;
  std::int32_t nvls_ok;  // this rank can and may join an NVLS group
  unsigned char uuid[16];
  cudaIpcMemHandle_t handle;
};

class CollResult final : public DevCollResult {
 public:
  CollResult(CudaTransport* tr, int dev, cudaStream_t s, EventPtr done)
      : tr_(tr), dev_(dev), stream_(s), done_(std::move(done)) {}
  void stream_wait() override {
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev_));
    CMX_CUDA(cudaStreamWaitEvent(current_stream(dev_), done_->ev, 0));
  }
  bool query() override { return cudaEventQuery(done_->ev) == cudaSuccess; }
  void host_wait() override { CMX_CUDA(cudaEventSynchronize(done_->ev)); }
  std::string error() override { return tr_->device_error(); }
  void mark_future(void* fut, void* value) override {
    c10::cuda::CUDAStreamGuard g(
        c10::cuda::getStreamFromExternal(stream_, static_cast<c10::DeviceIndex>(dev_)));
    static_cast<c10::ivalue::Future*>(fut)->markCompleted(*static_cast<c10::IValue*>(value));
  }

 private:
  CudaTransport* tr_;
  int dev_;
  cudaStream_t stream_;
  EventPtr done_;
};

}  // namespace

CollImpl::CollImpl(CudaTransport* tr, int dev)
    : tr_(tr), eng_(tr->engine()), ctx_(tr->ctx(dev)), dev_(dev), P_(tr->engine()->size()),
      me_(tr->engine()->rank()) {
  TORCH_CHECK(P_ <= kMaxCollRanks, "commux: CUDA collectives support up to ", kMaxCollRanks,
              " ranks per group (one NVLink domain)");
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
  region_bytes_ = env_int("COMMUX_CUDA_WS_BYTES", 64ll << 20);
  region_bytes_ = std::max<std::int64_t>(region_bytes_ & ~std::int64_t(4095), 1 << 20);
  // one-shot moves (P-1) x the message out of every rank but needs a single
  // flag round: it wins up to a few MB at 2 ranks, less as P grows
  if (env_int("COMMUX_COLL_TRACE", 0) != 0) {
    CMX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&trace_h_),
                           kTracePoints * kTraceChunks * sizeof(unsigned long long), cudaHostAllocMapped));
    CMX_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&trace_d_), trace_h_, 0));
  }
  oneshot_bytes_ = env_int("COMMUX_ONESHOT_BYTES", P_ <= 2 ? 4ll << 20 : P_ <= 4 ? 2ll << 20 : 1ll << 20);
  chain_ranks_ = static_cast<int>(env_int("COMMUX_CHAIN_RANKS", 0));
  // COMMUX_ALGO=oneshot|twoshot|nvls forces an algorithm for the reductions
  // where it applies (the others keep the size-based choice)
  if (const char* f = std::getenv("COMMUX_ALGO")) {
    const std::string v(f);
    forced_algo_ = v == "oneshot" ? kAlgoOneShot : v == "twoshot" ? kAlgoTwoShot : v == "nvls" ? kAlgoNvls : -1;
  }
  int lo = 0, hi = 0;
  CMX_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
  CMX_CUDA(cudaStreamCreateWithPriority(&stream_, cudaStreamNonBlocking, hi));
  const std::size_t total = kFlagBytes + 2 * static_cast<std::size_t>(region_bytes_);
  CMX_CUDA(cudaMalloc(reinterpret_cast<void**>(&ws_), total));
  CMX_CUDA(cudaMemsetAsync(ws_, 0, kFlagBytes, stream_));
  CMX_CUDA(cudaStreamSynchronize(stream_));

  // exchange workspace handles (collective: every rank creates its workspace
  // at its first CUDA collective, in the same order)
  ExchangeRecord mine;
  std::memset(&mine, 0, sizeof(mine));
  mine.pid = static_cast<std::int32_t>(::getpid());
  mine.nvls_ok = env_int("COMMUX_NVLS", 1) != 0 && NvlsBuffer::device_supported(dev) ? 1 : 0;
  std::memcpy(mine.uuid, ctx_->uuid, 16);
  CMX_CUDA(cudaIpcGetMemHandle(&mine.handle, ws_));
  const std::string key = eng_->store_prefix() + "cws/";
  std::vector<std::uint8_t> blob(reinterpret_cast<std::uint8_t*>(&mine),
                                 reinterpret_cast<std::uint8_t*>(&mine) + sizeof(mine));
  eng_->store().set(key + std::to_string(me_), blob);
  data_.assign(P_, nullptr);
  flags_.assign(P_, nullptr);
  std::vector<ExchangeRecord> recs(P_);
  for (int p = 0; p < P_; ++p) {
    if (p == me_) {
      recs[p] = mine;
      continue;
    }
    eng_->store().wait({key + std::to_string(p)}, eng_->timeout());
    auto v = eng_->store().get(key + std::to_string(p));
    TORCH_CHECK(v.size() == sizeof(ExchangeRecord), "commux: malformed workspace record");
    std::memcpy(&recs[p], v.data(), sizeof(ExchangeRecord));
  }
  // any two ranks of the group on one GPU: every rank decides alike (a
  // rank alone on its GPU must not take the device path while the others
  // stage through the host)
  for (int p = 0; p < P_ && !shared_gpu_; ++p)
    for (int q = p + 1; q < P_; ++q)
      if (std::memcmp(recs[p].uuid, recs[q].uuid, 16) == 0) {
        shared_gpu_ = true;
        break;
      }
  if (shared_gpu_) {  // kernels of two processes on one GPU must not wait on each other
    logf(LogLevel::Info, me_, "device collectives: ranks share a GPU, collectives are staged through the host");
    return;
  }
  for (int p = 0; p < P_; ++p) {
    char* base = ws_;
    if (p != me_) {
      void* q = nullptr;
      CMX_CUDA(cudaIpcOpenMemHandle(&q, recs[p].handle, cudaIpcMemLazyEnablePeerAccess));
      base = static_cast<char*>(q);
    }
    flags_[p] = reinterpret_cast<std::uint64_t*>(base);
    data_[p] = base + kFlagBytes;
  }
  // NVLS: every rank on its own GPU and able to join (the same records on
  // every rank, so the decision and the collective set-up are shared)
  // NVLS moves (P+1)/P of the message over each NVLink (the switch also
  // reads and writes this rank's own copy) against 2(P-1)/P for two-shot:
  // it loses at 2 ranks, and measured below two-shot at 4, so it is chosen
  // from 8 ranks up unless COMMUX_NVLS_MIN_RANKS says otherwise.
  bool nvls = P_ >= std::max<std::int64_t>(2, env_int("COMMUX_NVLS_MIN_RANKS", 8));
  for (int p = 0; p < P_; ++p) nvls = nvls && recs[p].nvls_ok != 0;
  nvls_min_bytes_ = env_int("COMMUX_NVLS_MIN_BYTES", 1ll << 20);
  if (nvls) {
    const std::int64_t bytes = std::max<std::int64_t>(env_int("COMMUX_NVLS_BYTES", 2 * region_bytes_), 4 << 20);
    nvls_ = NvlsBuffer::create(eng_, dev, static_cast<std::size_t>(bytes), &nvls_why_);
    if (!nvls_)
      logf(LogLevel::Warn, me_, "NVLS collectives unavailable (%s); using peer-to-peer kernels", nvls_why_.c_str());
  } else {
    nvls_why_ = "too few ranks, COMMUX_NVLS=0, or no multicast support on some rank";
  }
  logf(LogLevel::Info, me_,
       "device collectives on GPU %d: workspace 2 x %lld bytes (IPC), one-shot <= %lld bytes, NVLS %s%s "
       "(>= %lld bytes), COMMUX_ALGO %s",
       dev_, static_cast<long long>(region_bytes_), static_cast<long long>(oneshot_bytes_),
       nvls_ ? "on" : "off: ", nvls_ ? "" : nvls_why_.c_str(), static_cast<long long>(nvls_min_bytes_),
       forced_algo_ < 0                ? "auto"
       : forced_algo_ == kAlgoOneShot ? "oneshot"
       : forced_algo_ == kAlgoTwoShot ? "twoshot"
                                      : "nvls");
}

// COMMUX_COLL_TRACE=1: after each collective (synchronously), one line per
// call with the phase durations of CTA 0, averaged over the chunks: push =
// stores into peers' workspaces, sig = the flag store (waits for those
// stores to land), wait = until every peer's flag arrived, fold, push2 =
// folded segment out, wait2, out = copy-out.
void CollImpl::report_trace(int algo, int mode, std::int64_t bytes, int ctas) {
  CMX_CUDA(cudaStreamSynchronize(stream_));
  const unsigned long long* t = trace_h_;
  double sum[kTracePoints] = {0};
  int nch = 0;
  for (int c = 0; c < kTraceChunks; ++c) {
    const unsigned long long* r = t + c * kTracePoints;
    if (r[0] == 0) break;
    for (int k = 1; k < kTracePoints; ++k)
      if (r[k] != 0 && r[k - 1] != 0) sum[k] += static_cast<double>(r[k] - r[k - 1]) / 1000.0;
    ++nch;
  }
  if (nch == 0) return;
  double total = 0;
  for (int c = nch - 1; c >= 0; --c) {
    const unsigned long long* r = t + c * kTracePoints;
    unsigned long long last = 0;
    for (int k = kTracePoints - 1; k >= 0 && last == 0; --k) last = r[k];
    total = static_cast<double>(last - t[0]) / 1000.0;
    break;
  }
  std::fprintf(stderr,
               "[commux trace rank %d] algo %d mode %d bytes %lld ctas %d chunks %d total %.1f us | per chunk: "
               "push %.1f sig %.1f wait %.1f fold %.1f push2 %.1f wait2 %.1f out %.1f\n",
               me_, algo, mode, static_cast<long long>(bytes), ctas, nch, total, sum[1] / nch, sum[2] / nch,
               sum[3] / nch, sum[4] / nch, sum[5] / nch, sum[6] / nch, sum[7] / nch);
}

CollImpl::~CollImpl() {
  if (!select_device_quiet(dev_)) return;  // context gone at process exit
  if (trace_h_) cudaFreeHost(trace_h_);
  if (stream_) cudaStreamSynchronize(stream_);
  nvls_.reset();
  for (int p = 0; p < P_; ++p)
    if (p != me_ && flags_[p]) cudaIpcCloseMemHandle(flags_[p]);
  if (ws_) cudaFree(ws_);
  // stream_ stays: tensors freed later may carry stream-use records of it
  cudaGetLastError();
}

int CollImpl::choose_ctas(int mode, int algo, std::int64_t bytes) const {
  static const std::int64_t forced = env_int("COMMUX_COLL_CTAS", 0);
  // Every CTA of a launch must be resident at once (CTA b waits for CTA b of
  // the peers): the copy kernels fit two 512-thread CTAs per SM (<= 64
  // registers), the NVLS kernel one. Two per SM measured 8-10 % faster than
  // one on large two-shot allreduces (1 GiB at 2 GPUs: 2.06 vs 2.23 ms).
  const int one = std::min(ctx_->sm_count, kMaxCollCtas);
  const int two = std::min(2 * ctx_->sm_count, kMaxCollCtas);
  // COMMUX_COLL_CTAS overrides the choice, within residency
  if (forced > 0) return static_cast<int>(std::min<std::int64_t>(forced, algo == kAlgoNvls ? one : two));
  if (algo == kAlgoNvls) return one;
  if (mode == kModeAllreduce || mode == kModeReduce || mode == kModeReduceScatter) {
    if (algo == kAlgoOneShot)
      return static_cast<int>(std::max<std::int64_t>(1, std::min<std::int64_t>(one, bytes / (16 << 10))));
    return two;
  }
  return static_cast<int>(std::max<std::int64_t>(1, std::min<std::int64_t>(two, bytes / (16 << 10))));
}

void CollImpl::fill(CollArgs& a, const Launch& l, const at::Tensor& in, const at::Tensor& out) {
  std::memset(&a, 0, sizeof(a));
  a.P = P_;
  a.me = me_;
  a.root = l.root;
  a.mode = l.mode;
  a.op = l.op;
  a.dtype = dtype_code(in.scalar_type());
  a.elem_bytes = static_cast<int>(in.element_size());
  // COMMUX_CHAIN_RANKS: group size from which broadcasts, and reduces of
  // messages beyond one-shot, run along a chain of the ranks (0: never, the
  // default; the chain measured slower than scatter + allgather and two-shot)
  a.bcast_chain_ranks = chain_ranks_;
  a.n = l.n;
  a.in = in.data_ptr();
  a.out = out.data_ptr();
  for (int p = 0; p < P_; ++p) {
    a.data[p] = data_[p];
    a.flags[p] = flags_[p];
  }
  a.region_bytes = region_bytes_;
  ++epoch_;
  a.half_off = (epoch_ & 1) ? region_bytes_ / 2 : 0;
  a.seq_base = epoch_ << 20;
  a.timeout_ns = tr_->device_timeout_ns();
  a.status = ctx_->status_d;
  a.trace = trace_d_;
  if (nvls_) {
    a.nvls_uc = nvls_->uc();
    a.nvls_mc = nvls_->mc();
    a.nvls_bytes = static_cast<std::int64_t>(nvls_->size());
    a.nvls_half_off = (epoch_ & 1) ? a.nvls_bytes / 2 : 0;
  }
}

DevCollPtr CollImpl::run(const std::vector<Launch>& launches) {
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev_));
  cudaStream_t cur = current_stream(dev_);
  auto c10s = c10::cuda::getStreamFromExternal(stream_, static_cast<c10::DeviceIndex>(dev_));
  // contiguous, 16B-aligned inputs and outputs (copies made on the caller's
  // stream so they are ordered before the collective)
  std::vector<at::Tensor> ins, outs;
  for (auto& l : launches) {
    at::Tensor i = *l.in, o = *l.out;
    auto good = [](const at::Tensor& t) {
      return t.is_contiguous() && (reinterpret_cast<std::uintptr_t>(t.data_ptr()) & 15u) == 0;
    };
    if (!good(i)) i = i.contiguous().clone();
    if (l.in == l.out)
      o = i;
    else if (!good(o))
      o = at::empty(o.sizes(), o.options());
    ins.push_back(i);
    outs.push_back(o);
  }
  auto ready = ctx_->event();
  CMX_CUDA(cudaEventRecord(ready->ev, cur));
  CMX_CUDA(cudaStreamWaitEvent(stream_, ready->ev, 0));
  for (std::size_t k = 0; k < launches.size(); ++k) {
    const Launch& l = launches[k];
    // nothing to move: no launch (a launch without a flag round would break
    // the rule that every call proves the peers finished the call before)
    if (l.n == 0) continue;
    CollArgs a;
    fill(a, l, ins[k], outs[k]);
    std::int64_t bytes = l.n * a.elem_bytes;
    const bool reduce_like = l.mode == kModeAllreduce || l.mode == kModeReduce;
    const bool oneshot_fits = reduce_like && l.n * a.elem_bytes * P_ <= region_bytes_ / 2;
    const bool nvls_fits = nvls_ && l.mode == kModeAllreduce && nvls_supported(a.dtype, a.op);
    int algo = kAlgoTwoShot;
    if (forced_algo_ == kAlgoOneShot && oneshot_fits)
      algo = kAlgoOneShot;
    else if (forced_algo_ == kAlgoNvls && nvls_fits)
      algo = kAlgoNvls;
    else if (forced_algo_ == kAlgoTwoShot)
      algo = kAlgoTwoShot;
    else if (oneshot_fits && bytes <= oneshot_bytes_)
      algo = kAlgoOneShot;
    else if (l.mode == kModeReduce && chain_ranks_ > 0 && P_ >= chain_ranks_)
      algo = kAlgoChain;
    else if (nvls_fits && bytes >= nvls_min_bytes_)
      algo = kAlgoNvls;
    a.algo = algo;
    int ctas = choose_ctas(l.mode, algo, bytes);
    if (trace_h_ != nullptr) std::memset(trace_h_, 0, kTracePoints * kTraceChunks * sizeof(unsigned long long));
    CMX_CUDA(launch_coll(a, ctas, stream_));
    tr_->kernel_launches++;
    if (trace_h_ != nullptr) report_trace(algo, l.mode, bytes, ctas);
    st_calls_++;
    st_bytes_ += bytes;
    if (l.mode == kModeBroadcast && chain_ranks_ > 0 && P_ >= chain_ranks_)
      st_chain_++;
    else if (l.mode == kModeAllgather || l.mode == kModeBroadcast)
      st_gather_++;
    else if (algo == kAlgoChain)
      st_chain_++;
    else if (algo == kAlgoOneShot)
      st_oneshot_++;
    else if (algo == kAlgoNvls)
      st_nvls_++;
    else
      st_twoshot_++;
  }
  // copy back results that went through a temporary
  {
    c10::cuda::CUDAStreamGuard sg(c10s);
    for (std::size_t k = 0; k < launches.size(); ++k) {
      at::Tensor& user_out = *launches[k].out;
      if (!outs[k].is_same(user_out) && outs[k].data_ptr() != user_out.data_ptr())
        user_out.copy_(outs[k].view(user_out.sizes()));
    }
  }
  for (std::size_t k = 0; k < launches.size(); ++k) {
    c10::cuda::CUDACachingAllocator::recordStream(ins[k].storage().data_ptr(), c10s);
    c10::cuda::CUDACachingAllocator::recordStream(outs[k].storage().data_ptr(), c10s);
    c10::cuda::CUDACachingAllocator::recordStream(launches[k].out->storage().data_ptr(), c10s);
  }
  auto done = ctx_->event();
  CMX_CUDA(cudaEventRecord(done->ev, stream_));
  return std::make_shared<CollResult>(tr_, dev_, stream_, done);
}

DevCollPtr CollImpl::allreduce(std::vector<at::Tensor>& ts, RedOp op) {
  std::vector<Launch> ls;
  for (auto& t : ts) ls.push_back({kModeAllreduce, op_code(op), 0, &t, &t, t.numel()});
  return run(ls);
}

DevCollPtr CollImpl::reduce(std::vector<at::Tensor>& ts, RedOp op, int root) {
  std::vector<Launch> ls;
  for (auto& t : ts) ls.push_back({kModeReduce, op_code(op), root, &t, &t, t.numel()});
  return run(ls);
}

DevCollPtr CollImpl::broadcast(std::vector<at::Tensor>& ts, int root) {
  std::vector<Launch> ls;
  for (auto& t : ts) ls.push_back({kModeBroadcast, 0, root, &t, &t, t.numel()});
  return run(ls);
}

DevCollPtr CollImpl::allgather(at::Tensor& out, const at::Tensor& in) {
  std::vector<Launch> ls{{kModeAllgather, 0, 0, &in, &out, in.numel()}};
  return run(ls);
}

DevCollPtr CollImpl::reduce_scatter(at::Tensor& out, const at::Tensor& in, RedOp op) {
  std::vector<Launch> ls{{kModeReduceScatter, op_code(op), 0, &in, &out, out.numel()}};
  return run(ls);
}

DevCollPtr CollImpl::barrier() {
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev_));
  cudaStream_t cur = current_stream(dev_);
  auto ready = ctx_->event();
  CMX_CUDA(cudaEventRecord(ready->ev, cur));
  CMX_CUDA(cudaStreamWaitEvent(stream_, ready->ev, 0));
  CollArgs a;
  std::memset(&a, 0, sizeof(a));
  a.P = P_;
  a.me = me_;
  a.mode = kModeBarrier;
  for (int p = 0; p < P_; ++p) a.flags[p] = flags_[p];
  ++epoch_;
  a.seq_base = epoch_ << 20;
  a.timeout_ns = tr_->device_timeout_ns();
  a.status = ctx_->status_d;
  CMX_CUDA(launch_barrier(a, stream_));
  tr_->kernel_launches++;
  st_barriers_++;
  auto done = ctx_->event();
  CMX_CUDA(cudaEventRecord(done->ev, stream_));
  return std::make_shared<CollResult>(tr_, dev_, stream_, done);
}

std::vector<std::pair<std::string, std::int64_t>> CollImpl::stats() const {
  return {{"coll_calls", st_calls_},   {"coll_oneshot", st_oneshot_}, {"coll_twoshot", st_twoshot_},
          {"coll_gather", st_gather_}, {"coll_bytes", st_bytes_},     {"coll_shared_gpu", shared_gpu_ ? 1 : 0},
          {"coll_nvls", st_nvls_},     {"coll_nvls_enabled", nvls_ ? 1 : 0},
          {"coll_barriers", st_barriers_}, {"coll_chain", st_chain_}};
}

// ---------------------------------------------------------------------------
// transport entry points
// ---------------------------------------------------------------------------

bool CudaTransport::device_collectives(int dev) {
  if (!coll_) coll_ = std::make_unique<CollImpl>(this, dev);
  TORCH_CHECK(coll_->device() == dev, "commux: CUDA collectives of one group must use one device "
              "per rank (got device ", dev, " after ", coll_->device(), ")");
  return !coll_->shared_gpu();
}

DevCollPtr CudaTransport::allreduce(std::vector<at::Tensor>& ts, RedOp op) {
  device_collectives(ts[0].device().index());
  return coll_->allreduce(ts, op);
}
DevCollPtr CudaTransport::reduce(std::vector<at::Tensor>& ts, RedOp op, int root) {
  device_collectives(ts[0].device().index());
  return coll_->reduce(ts, op, root);
}
DevCollPtr CudaTransport::broadcast(std::vector<at::Tensor>& ts, int root) {
  device_collectives(ts[0].device().index());
  return coll_->broadcast(ts, root);
}
DevCollPtr CudaTransport::allgather(at::Tensor& out, const at::Tensor& in) {
  device_collectives(in.device().index());
  return coll_->allgather(out, in);
}
DevCollPtr CudaTransport::reduce_scatter(at::Tensor& out, const at::Tensor& in, RedOp op) {
  device_collectives(in.device().index());
  return coll_->reduce_scatter(out, in, op);
}
DevCollPtr CudaTransport::barrier() {
  TORCH_CHECK(collectives_ready(), "commux: the device barrier needs the group's device collectives");
  return coll_->barrier();
}

bool CudaTransport::collectives_ready() { return coll_ && !coll_->shared_gpu(); }

}  // namespace cuda
}  // namespace commux
