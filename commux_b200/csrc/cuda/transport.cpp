#include "transport.hpp"

#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <cstdio>
#include <cstring>
#include <thread>
#include <sstream>

#include "coll.hpp"
#include "commux/process_group_ucx.hpp"
#include "wire.hpp"

namespace commux {
namespace cuda {


// ---------------------------------------------------------------------------
// device context
// ---------------------------------------------------------------------------

bool select_device_quiet(int dev) {
  if (cudaSetDevice(dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

EventPool::~EventPool() {
  if (!select_device_quiet(dev)) return;  // context already gone at exit
  for (auto e : free) cudaEventDestroy(e);
}

ExportPool::~ExportPool() {
  if (!select_device_quiet(dev)) return;  // context already gone at exit
  for (auto& kv : free) cudaFree(kv.second);
  cudaGetLastError();
}

at::Tensor DevCtx::exportable_empty(at::IntArrayRef sizes, at::ScalarType dtype) {
  std::int64_t numel = 1;
  for (auto v : sizes) numel *= v;
  constexpr std::size_t kGrain = std::size_t{1} << 21;  // cudaMalloc's own granularity
  const std::size_t need = std::max<std::size_t>(1, static_cast<std::size_t>(numel) * at::elementSize(dtype));
  const std::size_t cap = (need + kGrain - 1) / kGrain * kGrain;
  void* p = nullptr;
  std::size_t got = 0;
  {
    std::lock_guard<std::mutex> lk(export_pool->mu);
    auto it = export_pool->free.lower_bound(cap);
    if (it != export_pool->free.end() && it->first <= 2 * cap) {  // reuse up to twice the size
      p = it->second;
      got = it->first;
      export_pool->free.erase(it);
    }
  }
  if (p == nullptr) {
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
    CMX_CUDA(cudaMalloc(&p, cap));
    got = cap;
    std::lock_guard<std::mutex> lk(export_pool->mu);
    export_pool->bytes += static_cast<std::int64_t>(cap);
  }
  std::shared_ptr<ExportPool> pool = export_pool;
  return at::from_blob(
      p, sizes,
      [pool, got](void* q) {
        std::lock_guard<std::mutex> lk(pool->mu);
        pool->free.emplace(got, q);
      },
      at::TensorOptions().dtype(dtype).device(at::kCUDA, dev));
}

EventRef::~EventRef() {
  if (pool && ev != nullptr) {
    std::lock_guard<std::mutex> lk(pool->mu);
    pool->free.push_back(ev);
  }
}

DevCtx::DevCtx(int d)
    : dev(d), export_pool(std::make_shared<ExportPool>(d)), pool_(std::make_shared<EventPool>(d)) {
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(d));
  cudaDeviceProp prop;
  CMX_CUDA(cudaGetDeviceProperties(&prop, d));
  std::memcpy(uuid, prop.uuid.bytes, 16);
  sm_count = prop.multiProcessorCount;
  int lo = 0, hi = 0;
  CMX_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
  CMX_CUDA(cudaStreamCreateWithPriority(&comm, cudaStreamNonBlocking, hi));
  // [0, kSlots): consumed flags of one-shot sends; [kSlots, 2 kSlots): flags
  // of persistent plans (never reused)
  CMX_CUDA(cudaMalloc(reinterpret_cast<void**>(&mbox), 2 * kSlots * sizeof(std::uint64_t)));
  CMX_CUDA(cudaMemsetAsync(mbox, 0, 2 * kSlots * sizeof(std::uint64_t), comm));
  CMX_CUDA(cudaStreamSynchronize(comm));
  CMX_CUDA(cudaIpcGetMemHandle(&mbox_handle, mbox));
  unsigned long long id = 0;
  cu_check(cuPointerGetAttribute(&id, CU_POINTER_ATTRIBUTE_BUFFER_ID,
                                 reinterpret_cast<CUdeviceptr>(mbox)),
           "cuPointerGetAttribute(mailbox)");
  mbox_id = id;
  mbox_base = reinterpret_cast<std::uint64_t>(mbox);
  CMX_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&status_h), 64,
                         cudaHostAllocMapped | cudaHostAllocPortable));
  std::memset(status_h, 0, 64);
  CMX_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_d), status_h, 0));
}

DevCtx::~DevCtx() {
  // At process exit the context may already be destroyed: then leave the
  // resources to the driver instead of calling into a dead context.
  if (!select_device_quiet(dev)) return;
  cudaStreamSynchronize(comm);
  for (auto& kv : scratch_) cudaFree(kv.second);
  if (mbox) cudaFree(mbox);
  if (status_h) cudaFreeHost(status_h);
  // `comm` is not destroyed: tensors freed later may still carry stream-use
  // records of it in torch's caching allocator, which then records events on
  // it. A stream lives until process exit anyway.
  cudaGetLastError();
}

EventPtr DevCtx::event() {
  cudaEvent_t e = nullptr;
  {
    std::lock_guard<std::mutex> lk(pool_->mu);
    if (!pool_->free.empty()) {
      e = pool_->free.back();
      pool_->free.pop_back();
    }
  }
  if (e == nullptr) {
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
    CMX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  auto p = std::make_shared<EventRef>();
  p->ev = e;
  p->pool = pool_;
  return p;
}

void DevCtx::release(cudaEvent_t e) {
  std::lock_guard<std::mutex> lk(pool_->mu);
  pool_->free.push_back(e);
}

std::uint32_t* DevCtx::scratch(cudaStream_t s) {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = scratch_.find(s);
  if (it != scratch_.end()) return it->second;
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
  std::uint32_t* p = nullptr;
  CMX_CUDA(cudaMalloc(reinterpret_cast<void**>(&p), kCounterSlots * sizeof(std::uint32_t)));
  CMX_CUDA(cudaMemsetAsync(p, 0, kCounterSlots * sizeof(std::uint32_t), s));
  scratch_[s] = p;
  return p;
}

std::uint32_t DevCtx::take_slots(cudaStream_t s, std::uint32_t n) {
  std::lock_guard<std::mutex> lk(mu_);
  std::uint32_t& next = next_slot_[s];
  std::uint32_t first = next;
  next = (next + n) % kCounterSlots;
  return first;
}

// ---------------------------------------------------------------------------
// transport
// ---------------------------------------------------------------------------

CudaTransport::CudaTransport(Engine* e) : eng_(e) {
  std::int64_t ms = env_int("COMMUX_DEVICE_TIMEOUT_MS", 60000);
  std::int64_t host_ms = e->timeout().count();
  if (host_ms > 0) ms = std::min(ms, host_ms);
  timeout_ns_ = static_cast<std::uint64_t>(std::max<std::int64_t>(ms, 1)) * 1000000ull;
}

CudaTransport::~CudaTransport() { shutdown(); }

void CudaTransport::shutdown() {
  coll_.reset();
  {
    std::lock_guard<SpinMutex> lk(pend_mu_);
    pending_.clear();
  }
  bool alive = true;
  {
    std::lock_guard<std::mutex> lk(ctx_mu_);
    for (auto& kv : ctx_) {
      // pulls read peer mappings: let them finish before the mappings go
      // (pull kernels never wait on anything, so this returns)
      alive = alive && select_device_quiet(kv.first);
      if (alive) cudaStreamSynchronize(kv.second->comm);
    }
  }
  flights_.clear();
  std::lock_guard<SpinMutex> lk(ipc_mu_);
  if (alive)
    for (auto& kv : opened_) cudaIpcCloseMemHandle(kv.second.ptr);
  opened_.clear();
  cudaGetLastError();
}

DevCtx* CudaTransport::ctx(int dev) {
  std::lock_guard<std::mutex> lk(ctx_mu_);
  auto& p = ctx_[dev];
  if (!p) p = std::make_unique<DevCtx>(dev);
  return p.get();
}

void CudaTransport::publish_uuid(DevCtx* c) {
  if (uuid_published_) return;
  auto* h = eng_->my_header();
  std::memcpy(h->cuda_uuid, c->uuid, 16);
  h->cuda_uuid_valid.store(1, std::memory_order_release);
  uuid_published_ = true;
}

int CudaTransport::pull_ctas(DevCtx* c) const {
  static const std::int64_t v = env_int("COMMUX_P2P_CTAS", 0);
  return v > 0 ? static_cast<int>(v) : c->sm_count * 8;
}

bool CudaTransport::exportable(const void* ptr) {
  std::uint64_t id = 0, base = 0, size = 0;
  cudaIpcMemHandle_t h;
  try {
    ipc_export(ptr, &id, &base, &size, &h);
    return true;
  } catch (const std::runtime_error&) {
    cudaGetLastError();
    return false;
  }
}

at::Tensor CudaTransport::export_or_stage(const at::Tensor& t, DevCtx* c) {
  if (t.numel() == 0 || exportable(t.data_ptr())) return t;
  at::Tensor s = c->exportable_empty(t.sizes(), t.scalar_type());
  s.copy_(t);  // on the current stream, ahead of the send's ready event
  st_export_staged_++;
  return s;
}

void CudaTransport::ipc_export(const void* ptr, std::uint64_t* buffer_id, std::uint64_t* base,
                               std::uint64_t* size, cudaIpcMemHandle_t* handle) {
  CUpointer_attribute attrs[3] = {CU_POINTER_ATTRIBUTE_BUFFER_ID,
                                  CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                  CU_POINTER_ATTRIBUTE_RANGE_SIZE};
  unsigned long long id = 0;
  CUdeviceptr start = 0;
  std::size_t sz = 0;
  void* data[3] = {&id, &start, &sz};
  cu_check(cuPointerGetAttributes(3, attrs, data, reinterpret_cast<CUdeviceptr>(ptr)),
           "cuPointerGetAttributes");
  *buffer_id = id;
  *base = static_cast<std::uint64_t>(start);
  *size = sz;
  std::lock_guard<SpinMutex> lk(ipc_mu_);
  auto it = exported_.find(id);
  if (it != exported_.end()) {
    *handle = it->second;
    return;
  }
  cudaError_t e = unexportable_.count(id) != 0 ? cudaErrorInvalidValue
                                               : cudaIpcGetMemHandle(handle, reinterpret_cast<void*>(start));
  if (e != cudaSuccess) {
    // e.g. the caching allocator's expandable segments (cuMemCreate
    // mappings); callers stage such memory through the export pool
    cudaGetLastError();
    unexportable_.insert(id);  // allocation ids are never reused
    throw std::runtime_error(std::string("commux: this CUDA allocation cannot be exported through CUDA IPC (") +
                             cudaGetErrorString(e) + ")");
  }
  exported_[id] = *handle;
  st_ipc_exports_++;
}

void* CudaTransport::ipc_open(int src, std::uint64_t buffer_id, std::uint64_t base, std::uint64_t size,
                              const cudaIpcMemHandle_t& h, DevCtx* c) {
  std::lock_guard<SpinMutex> lk(ipc_mu_);
  auto key = std::make_pair(src, buffer_id);
  auto it = opened_.find(key);
  if (it != opened_.end()) return it->second.ptr;
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c->dev));
  // The sender reuses an address range only after freeing the allocation that
  // held it, and it frees a tensor only after every receive of it completed
  // (the receiver's copy kernel stored its completion flag after its last
  // load), and a persistent plan keeps its tensors alive. So no copy of this
  // rank will read an overlapping older mapping again: close it, instead of
  // keeping one mapping per allocation the sender ever had.
  if (size != 0) {
    for (auto o = opened_.lower_bound({src, 0}); o != opened_.end() && o->first.first == src;) {
      const Opened& m = o->second;
      if (m.size != 0 && m.base < base + size && base < m.base + m.size) {
        cudaIpcCloseMemHandle(m.ptr);
        cudaGetLastError();
        st_ipc_closes_++;
        o = opened_.erase(o);
      } else {
        ++o;
      }
    }
  }
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("commux: cudaIpcOpenMemHandle for rank ") +
                             std::to_string(src) + " failed: " + cudaGetErrorString(e));
  opened_[key] = Opened{p, base, size};
  st_ipc_opens_++;
  return p;
}

EventPtr ready_event_for(DevCtx* c, cudaStream_t s, int batch_depth,
                         std::map<int, EventPtr>& batch_events) {
  if (batch_depth > 0) {
    auto it = batch_events.find(c->dev);
    if (it != batch_events.end()) return it->second;
  }
  auto ev = c->event();
  CMX_CUDA(cudaEventRecord(ev->ev, s));
  if (batch_depth > 0) batch_events[c->dev] = ev;
  return ev;
}

void CudaTransport::prepare_send(const ReqPtr& s, int dst, std::vector<char>& blob, bool* gate,
                                 bool* complete_on_post) {
  const int dev = s->tensors[0].device().index();
  for (auto& t : s->tensors)
    TORCH_CHECK(t.device().index() == dev, "commux send: a coalesced CUDA message spans devices");
  DevCtx* c = ctx(dev);
  publish_uuid(c);
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
  auto st = std::make_shared<SendState>();
  st->device = dev;
  st->stream = current_stream(dev);
  st->local = dst == eng_->rank();

  // peer on another GPU (known once it published its device): narrow-row
  // views are packed here so the receiver's NVLink reads are contiguous
  bool peer_other_gpu = false;
  if (!st->local) {
    const auto* ph = eng_->peer_header(dst);
    bool known = ph->cuda_uuid_valid.load(std::memory_order_acquire) != 0;
    peer_other_gpu = known && std::memcmp(ph->cuda_uuid, c->uuid, 16) != 0;
  }
  std::vector<at::Tensor> wire_t;
  for (auto& t : s->tensors) {
    // The receiver's copy kernel walks at most kMaxPullDims dims: stage a
    // contiguous copy (on this stream, before the ready event) when the
    // view's own dims do not merge down that far.
    bool ok = t.dim() <= kWireDims && !(peer_other_gpu && narrow_rows(t));
    for (int k = 0; ok && k < t.dim(); ++k) ok = t.stride(k) >= 0;
    if (ok) {
      std::vector<std::int64_t> sz(t.sizes().begin(), t.sizes().end());
      std::vector<std::int64_t> sd(t.strides().begin(), t.strides().end());
      auto d = dims_of(sz.data(), sd.data(), t.dim());
      std::vector<Dim> merged;
      ok = refine(d, d, merged) && merged.size() <= static_cast<std::size_t>(kMaxPullDims);
    }
    if (ok) {
      wire_t.push_back(t);
    } else {
      st->staged.push_back(t.contiguous());
      wire_t.push_back(st->staged.back());
      st_staged_++;
    }
  }
  // a receiver in another process maps the sender's memory: memory that CUDA
  // IPC cannot export travels through an exportable pool buffer instead
  if (!st->local) {
    for (auto& t : wire_t) {
      at::Tensor e = export_or_stage(t, c);
      if (!e.is_same(t)) {
        st->staged.push_back(e);
        t = e;
      }
    }
  }
  {
    // A batch shares one ready event, recorded by its first message: it may
    // precede the copies just staged for this one, so a send that staged
    // anything records its own event behind them.
    std::lock_guard<SpinMutex> lk(batch_mu_);
    st->ready = ready_event_for(c, st->stream, st->staged.empty() ? batch_depth_ : 0, batch_event_);
  }

  blob.assign(sizeof(DrtsWire) + wire_t.size() * sizeof(SegWire), 0);
  auto* w = reinterpret_cast<DrtsWire*>(blob.data());
  w->magic = kWireMagic;
  w->nseg = static_cast<std::uint32_t>(wire_t.size());
  w->pid = static_cast<std::int32_t>(::getpid());
  w->device = dev;
  std::memcpy(w->uuid, c->uuid, 16);
  if (!st->local) {
    st->value = c->next_value.fetch_add(1) + 1;
    st->slot = st->value % kSlots;
    w->slot = st->slot;
    w->value = st->value;
    w->mbox_id = c->mbox_id;
    w->mbox_base = c->mbox_base;
    w->mbox_handle = c->mbox_handle;
    const auto* ph = eng_->peer_header(dst);
    bool known = ph->cuda_uuid_valid.load(std::memory_order_acquire) != 0;
    bool same = known && std::memcmp(ph->cuda_uuid, c->uuid, 16) == 0;
    st->device_wait = known && !same;
    (st->device_wait ? st_sends_device_ : st_sends_host_)++;
  }
  w->sender_waits_on_device = st->device_wait ? 1u : 0u;
  auto* segs = reinterpret_cast<SegWire*>(blob.data() + sizeof(DrtsWire));
  for (std::size_t i = 0; i < wire_t.size(); ++i) {
    const at::Tensor& t = wire_t[i];
    SegWire& sw = segs[i];
    sw.elem = static_cast<std::uint32_t>(t.element_size());
    sw.ndim = static_cast<std::int32_t>(t.dim());
    for (int k = 0; k < t.dim(); ++k) {
      sw.sizes[k] = t.size(k);
      sw.strides[k] = t.stride(k);
    }
    if (t.numel() == 0) continue;
    const char* p = static_cast<const char*>(t.data_ptr());
    if (st->local) {
      CUpointer_attribute attrs[2] = {CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, CU_POINTER_ATTRIBUTE_RANGE_SIZE};
      CUdeviceptr start = 0;
      std::size_t sz = 0;
      void* data[2] = {&start, &sz};
      cu_check(cuPointerGetAttributes(2, attrs, data, reinterpret_cast<CUdeviceptr>(p)),
               "cuPointerGetAttributes");
      sw.base = static_cast<std::uint64_t>(start);
      sw.alloc_size = sz;
      sw.offset = reinterpret_cast<std::uint64_t>(p) - sw.base;
    } else {
      ipc_export(p, &sw.buffer_id, &sw.base, &sw.alloc_size, &sw.handle);
      sw.offset = reinterpret_cast<std::uint64_t>(p) - sw.base;
    }
  }
  s->dev = st;
  *gate = !st->local;
  *complete_on_post = st->device_wait;
  if (st->local) {
    std::lock_guard<std::mutex> lk(local_mu_);
    local_sends_[s->id] = s;
  }
}

bool CudaTransport::send_gate_open(const ReqPtr& s) {
  auto st = state<SendState>(s);
  if (!st || st->local) return true;
  cudaError_t e = cudaEventQuery(st->ready->ev);
  if (e == cudaSuccess) return true;
  if (e == cudaErrorNotReady) return false;
  cudaGetLastError();
  std::lock_guard<SpinMutex> lk(pend_mu_);
  dev_error_ = std::string("commux: CUDA error while waiting for send data: ") + cudaGetErrorString(e);
  return true;
}

void CudaTransport::prepare_recv(const ReqPtr& r) {
  const int dev = r->tensors[0].device().index();
  for (auto& t : r->tensors)
    TORCH_CHECK(t.device().index() == dev, "commux recv: a coalesced CUDA message spans devices");
  DevCtx* c = ctx(dev);
  publish_uuid(c);
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
  auto st = std::make_shared<RecvState>();
  st->device = dev;
  st->stream = current_stream(dev);
  {
    std::lock_guard<SpinMutex> lk(batch_mu_);
    st->ready = ready_event_for(c, st->stream, batch_depth_, batch_event_);
  }
  r->dev = st;
}

void CudaTransport::build_descs(const ReqPtr& r, const char* blob, std::size_t len, bool local,
                                PendingPull& pp) {
  auto* w = reinterpret_cast<const DrtsWire*>(blob);
  if (len < sizeof(DrtsWire) || w->magic != kWireMagic ||
      len < sizeof(DrtsWire) + w->nseg * sizeof(SegWire))
    throw std::runtime_error("commux: malformed device message descriptor");
  auto* segs = reinterpret_cast<const SegWire*>(blob + sizeof(DrtsWire));
  auto rs = state<RecvState>(r);
  DevCtx* c = pp.ctx;
  std::uint64_t* done = nullptr;
  std::uint64_t done_val = 0;
  if (!local) {
    auto* mb = static_cast<std::uint64_t*>(ipc_open(pp.src, w->mbox_id, 0, 0, w->mbox_handle, c));
    done = mb + w->slot;
    done_val = w->value;
  }
  std::uint64_t sbytes = 0;
  for (std::uint32_t i = 0; i < w->nseg; ++i)
    sbytes += static_cast<std::uint64_t>(numel_wire(segs[i])) * segs[i].elem;
  if (sbytes > r->total)
    throw std::runtime_error("commux recv: message of " + std::to_string(sbytes) +
                             " bytes does not fit the " + std::to_string(r->total) + "-byte buffer");

  auto src_base = [&](const SegWire& sw) -> const char* {
    if (numel_wire(sw) == 0) return nullptr;
    if (local) return reinterpret_cast<const char*>(sw.base);
    return static_cast<const char*>(ipc_open(pp.src, sw.buffer_id, sw.base, sw.alloc_size, sw.handle, c));
  };
  auto src_ptr = [&](const SegWire& sw) -> const char* {
    const char* b = src_base(sw);
    return b == nullptr ? nullptr : b + sw.offset;
  };

  std::vector<PullDesc> out;
  // every descriptor appended since `from` must stay inside its buffers
  auto validate = [&](std::size_t from, const SegWire& sw, const at::Tensor& dst) {
    auto lo = reinterpret_cast<std::uintptr_t>(src_base(sw));
    auto dlo = reinterpret_cast<std::uintptr_t>(dst.storage().data());
    for (std::size_t k = from; k < out.size(); ++k)
      check_desc(out[k], lo, lo + sw.alloc_size, dlo, dlo + dst.storage().nbytes());
  };
  bool paired = w->nseg == r->tensors.size();
  for (std::uint32_t i = 0; paired && i < w->nseg; ++i)
    paired = numel_wire(segs[i]) == r->tensors[i].numel() &&
             segs[i].elem == static_cast<std::uint32_t>(r->tensors[i].element_size());
  if (paired) {
    for (std::uint32_t i = 0; i < w->nseg; ++i) {
      const SegWire& sw = segs[i];
      at::Tensor dt = r->tensors[i];
      if (dt.numel() == 0) continue;
      const char* sp = src_ptr(sw);
      char* dp = static_cast<char*>(dt.data_ptr());
      auto a = dims_of(sw.sizes, sw.strides, sw.ndim);
      std::vector<std::int64_t> dsz(dt.sizes().begin(), dt.sizes().end());
      std::vector<std::int64_t> dst(dt.strides().begin(), dt.strides().end());
      auto b = dims_of(dsz.data(), dst.data(), static_cast<int>(dsz.size()));
      std::vector<Dim> dims;
      bool ok = refine(a, b, dims) && dims.size() <= static_cast<std::size_t>(kMaxPullDims);
      const std::size_t from = out.size();
      if (ok) {
        emit_descs(sp, dp, dims, sw.elem, out);
        validate(from, sw, dt);
        continue;
      }
      // No common <=4-dim walk: land in a contiguous temp laid out like the
      // source, then scatter with a torch copy on the same stream.
      std::vector<std::int64_t> ssz(sw.sizes, sw.sizes + sw.ndim);
      at::Tensor tmp = at::empty(ssz, dt.options());
      std::vector<std::int64_t> tstr(tmp.strides().begin(), tmp.strides().end());
      auto tb = dims_of(ssz.data(), tstr.data(), sw.ndim);
      if (!refine(a, tb, dims) || dims.size() > static_cast<std::size_t>(kMaxPullDims))
        throw std::runtime_error("commux: the sender's tensor layout has more than 4 "
                                 "non-mergeable dimensions; send a contiguous tensor");
      emit_descs(sp, static_cast<char*>(tmp.data_ptr()), dims, sw.elem, out);
      validate(from, sw, tmp);
      rs->unpack.push_back({tmp, dt});
    }
  } else {
    // Byte-stream semantics (different tensor counts or element types): both
    // sides must be contiguous; the bytes are concatenated in order.
    std::vector<std::pair<const char*, std::uint64_t>> src_ranges;
    std::vector<const SegWire*> src_segs;
    for (std::uint32_t i = 0; i < w->nseg; ++i) {
      if (!contiguous_wire(segs[i]))
        throw std::runtime_error("commux recv: sender and receiver tensors differ in count or "
                                 "dtype, which needs contiguous tensors on both sides");
      std::uint64_t nb = static_cast<std::uint64_t>(numel_wire(segs[i])) * segs[i].elem;
      if (nb) {
        src_ranges.push_back({src_ptr(segs[i]), nb});
        src_segs.push_back(&segs[i]);
      }
    }
    std::size_t si = 0;
    std::size_t di = 0;
    std::uint64_t doff = 0;
    for (auto& sr : src_ranges) {
      std::uint64_t soff = 0;
      while (soff < sr.second) {
        while (di < r->tensors.size() &&
               doff >= static_cast<std::uint64_t>(r->tensors[di].numel()) * r->tensors[di].element_size()) {
          ++di;
          doff = 0;
        }
        TORCH_CHECK(di < r->tensors.size(), "commux recv: receive buffers too small");
        at::Tensor& dt = r->tensors[di];
        TORCH_CHECK(dt.is_contiguous(), "commux recv: byte-stream receive needs contiguous tensors");
        std::uint64_t dcap = static_cast<std::uint64_t>(dt.numel()) * dt.element_size() - doff;
        std::uint64_t n = std::min(dcap, sr.second - soff);
        std::vector<Dim> dims{{static_cast<std::int64_t>(n), 1, 1}};
        const std::size_t from = out.size();
        emit_descs(sr.first + soff, static_cast<char*>(dt.data_ptr()) + doff, dims, 1, out);
        validate(from, *src_segs[si], dt);
        soff += n;
        doff += n;
      }
      ++si;
    }
  }
  if (out.empty()) {
    PullDesc d{};
    d.ndim = 1;
    d.unit = 1;
    d.units = 0;
    d.nchunks = 1;
    out.push_back(d);
  }
  std::uint32_t chunks = 0;
  for (auto& d : out) {
    d.done = done;
    d.done_val = done_val;
    chunks += d.nchunks;
    st_pull_bytes_ += static_cast<std::int64_t>(d.units) * d.unit;
  }
  pp.descs = std::move(out);
  pp.msg_chunks = chunks;
}

void CudaTransport::on_match(const ReqPtr& r, int src, std::uint64_t send_id, const char* blob,
                             std::size_t len) {
  auto rs = state<RecvState>(r);
  const bool local = src == eng_->rank();
  DevCtx* c = ctx(rs->device);
  ReqPtr s;
  if (local) {
    std::lock_guard<std::mutex> lk(local_mu_);
    auto it = local_sends_.find(send_id);
    if (it != local_sends_.end()) {
      s = it->second;
      local_sends_.erase(it);
    }
  }
  auto* w = reinterpret_cast<const DrtsWire*>(blob);
  if (!local && len >= sizeof(DrtsWire) && w->sender_waits_on_device &&
      std::memcmp(w->uuid, c->uuid, 16) == 0) {
    eng_->send_fin(src, send_id, -3);
    eng_->fail(r, "commux: rank " + std::to_string(src) +
                      " sends from the GPU this receive lives on while it expected another "
                      "GPU; drive CUDA p2p from one device per rank");
    return;
  }
  PendingPull pp;
  pp.r = r;
  pp.src = src;
  pp.send_id = send_id;
  pp.ctx = c;
  pp.sender_waits = !local && len >= sizeof(DrtsWire) && w->sender_waits_on_device != 0;
  try {
    build_descs(r, blob, len, local, pp);
  } catch (const std::exception& e) {
    if (!local) eng_->send_fin(src, send_id, -4);
    if (s) eng_->fail(s, e.what());
    eng_->fail(r, e.what());
    return;
  }
  st_pulls_++;
  if (!local && len >= sizeof(DrtsWire))
    (std::memcmp(w->uuid, c->uuid, 16) == 0 ? st_pulls_same_gpu_ : st_pulls_peer_gpu_)++;
  if (!local) {
    {
      std::lock_guard<SpinMutex> lk(pend_mu_);
      pending_.push_back(std::move(pp));
      inflight_.fetch_add(1);
    }
    eng_->wake_progress();
    return;
  }
  TORCH_CHECK(s, "commux: internal error, self-send state missing");
  auto ss = state<SendState>(s);
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c->dev));
  cudaStream_t cur = current_stream(c->dev);
  if (ss->stream != cur) CMX_CUDA(cudaStreamWaitEvent(cur, ss->ready->ev, 0));
  if (rs->stream != cur) CMX_CUDA(cudaStreamWaitEvent(cur, rs->ready->ev, 0));
  pp.descs.shrink_to_fit();
  {
    std::lock_guard<SpinMutex> lk(batch_mu_);
    if (batch_depth_ > 0) {
      // launched together with the rest of the window at end_batch
      batch_local_.push_back({std::move(pp), cur});
      batch_local_sends_.push_back(s);
      return;
    }
  }
  std::vector<PendingPull> one;
  one.push_back(std::move(pp));
  launch_batch(c, one, cur);
  ss->local_done = rs->done;
  eng_->complete(s);
}

void CudaTransport::launch_batch(DevCtx* c, std::vector<PendingPull>& pulls, cudaStream_t stream) {
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c->dev));
  std::uint32_t* counters = c->scratch(stream);
  std::uint32_t nmsg = static_cast<std::uint32_t>(pulls.size());
  std::uint32_t next = c->take_slots(stream, nmsg);
  PullBatch b{};
  b.counters = counters;
  b.status = c->status_d;
  const int ctas = pull_ctas(c);
  auto flush = [&]() {
    if (b.n == 0) return;
    int launched = 0;
    CMX_CUDA(launch_pull(b, ctas, 256, stream, &launched));
    kernel_launches += launched;
    b.n = 0;
    b.total_chunks = 0;
  };
  for (auto& p : pulls) {
    std::uint32_t slot = next++ % kCounterSlots;
    for (auto& d : p.descs) {
      if (b.n == static_cast<std::uint32_t>(kMaxBatch)) flush();
      d.chunk0 = b.total_chunks;
      d.counter_idx = slot;
      d.msg_chunks = p.msg_chunks;
      b.d[b.n++] = d;
      b.total_chunks += d.nchunks;
    }
  }
  flush();
  // receives that could not be walked directly land in a temp: scatter now
  bool any_unpack = false;
  for (auto& p : pulls) any_unpack |= !state<RecvState>(p.r)->unpack.empty();
  if (any_unpack) {
    c10::cuda::CUDAStreamGuard sg(c10::cuda::getStreamFromExternal(stream, static_cast<c10::DeviceIndex>(c->dev)));
    for (auto& p : pulls)
      for (auto& tv : state<RecvState>(p.r)->unpack) tv.second.copy_(tv.first.view(tv.second.sizes()));
  }
  auto done = c->event();
  CMX_CUDA(cudaEventRecord(done->ev, stream));
  // No recordStream on the receive tensors: the request (and its tensors)
  // stays referenced until the done event completed (progress thread), and a
  // caller that waited has its stream ordered after that event.
  for (auto& p : pulls) {
    auto rs = state<RecvState>(p.r);
    rs->done = done;
    eng_->complete(p.r);
  }
}

bool CudaTransport::poll() {
  // inflight_ counts the pulls waiting in pending_ plus those in flights_:
  // when it is zero there is nothing to do, and the progress thread, which
  // calls this on every turn of its loop, stays off pend_mu_ (posting threads
  // take it for every device message and every device_error() check)
  if (inflight_.load(std::memory_order_acquire) == 0) return false;
  bool busy = false;
  std::vector<PendingPull> ready;
  {
    std::lock_guard<SpinMutex> lk(pend_mu_);
    for (auto it = pending_.begin(); it != pending_.end();) {
      auto rs = state<RecvState>(it->r);
      cudaError_t e = cudaEventQuery(rs->ready->ev);
      if (e == cudaSuccess) {
        ready.push_back(std::move(*it));
        it = pending_.erase(it);
      } else {
        if (e != cudaErrorNotReady) {
          cudaGetLastError();
          dev_error_ = std::string("commux: CUDA error on a receive's stream: ") + cudaGetErrorString(e);
        }
        ++it;
      }
    }
  }
  if (!ready.empty()) {
    busy = true;
    std::map<DevCtx*, std::vector<PendingPull>> by_ctx;
    for (auto& p : ready) by_ctx[p.ctx].push_back(std::move(p));
    for (auto& kv : by_ctx) {
      Flight f;
      std::vector<std::pair<int, std::uint64_t>> launched;
      for (auto& p : kv.second) {
        f.fins.push_back({p.src, p.send_id});
        if (p.sender_waits) launched.push_back({p.src, p.send_id});
        f.reqs.push_back(p.r);
      }
      f.pulls = static_cast<int>(kv.second.size());
      launch_batch(kv.first, kv.second, kv.first->comm);
      f.done = state<RecvState>(f.reqs.front())->done;
      flights_.push_back(std::move(f));
      // the copies are enqueued: their senders may now wait on the device
      for (auto& x : launched) eng_->send_fin(x.first, x.second, proto::kFinLaunched);
    }
  }
  while (!flights_.empty()) {
    Flight& f = flights_.front();
    cudaError_t e = cudaEventQuery(f.done->ev);
    if (e == cudaErrorNotReady) break;
    if (e != cudaSuccess) {
      cudaGetLastError();
      std::lock_guard<SpinMutex> lk(pend_mu_);
      dev_error_ = std::string("commux: CUDA error in a pull: ") + cudaGetErrorString(e);
    }
    for (auto& fin : f.fins) {
      eng_->send_fin(fin.first, fin.second, e == cudaSuccess ? 0 : -5);
      st_fins_++;
    }
    inflight_.fetch_sub(f.pulls);  // == f.fins.size()
    flights_.pop_front();
    busy = true;
  }
  return busy;
}

namespace {

std::string fin_error(std::int64_t status) {
  const char* why = status == -3   ? "the receiver shares this GPU but the send expected a peer GPU"
                    : status == -4 ? "the receiver could not describe the copy (layout/size mismatch)"
                    : status == -5 ? "the receiver's copy kernel failed"
                                   : "the receiver rejected the message";
  return std::string("commux send: ") + why;
}

}  // namespace

void CudaTransport::on_fin(const ReqPtr& s, std::int64_t status) {
  auto st = state<SendState>(s);
  if (status == proto::kFinLaunched) {
    if (st) st->launched.store(true, std::memory_order_release);
    return;
  }
  if (st) {
    if (status != 0) st->fin_status.store(status, std::memory_order_relaxed);
    st->fin.store(true, std::memory_order_release);
  }
  if (status != 0) {
    eng_->fail(s, fin_error(status));
    return;
  }
  if (st && !st->device_wait) eng_->complete(s);
}

// Blocks the calling thread until the receiver of a device_wait send has
// enqueued its copy (or failed, or the group aborted), bounded by the group
// timeout. A wait kernel launched before that point would keep this GPU
// busy on a copy that is not enqueued yet; a CUDA call of the receiver that
// waits for its own GPU to go idle (mapping or unmapping peer memory) could
// then wait, through the peers' spinning kernels, on this very call.
void CudaTransport::wait_pull_launched(SendState& st) {
  if (st.launched.load(std::memory_order_acquire) || st.fin.load(std::memory_order_acquire)) return;
  const auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  while (!st.launched.load(std::memory_order_acquire) && !st.fin.load(std::memory_order_acquire)) {
    if (eng_->aborted()) throw std::runtime_error("commux send: the group was aborted");
    if (++spins < 2000) {
      std::this_thread::yield();
      continue;
    }
    if (std::chrono::steady_clock::now() - t0 > eng_->timeout())
      throw std::runtime_error("commux send: the receiver did not start the copy within " +
                               std::to_string(eng_->timeout().count()) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

void CudaTransport::wait_sends_on_stream(const std::vector<ReqPtr>& sends) {
  // group the device-side waits per device into one-warp launches
  std::map<int, std::vector<std::shared_ptr<SendState>>> by_dev;
  for (auto& s : sends) {
    auto st = state<SendState>(s);
    wait_pull_launched(*st);
    if (st->fin.load(std::memory_order_acquire)) {  // consumed already, or failed
      const std::int64_t e = st->fin_status.load(std::memory_order_relaxed);
      if (e != 0) throw std::runtime_error(fin_error(e));
      continue;
    }
    by_dev[st->device].push_back(st);
  }
  for (auto& kv : by_dev) {
    DevCtx* c = ctx(kv.first);
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c->dev));
    cudaStream_t cur = current_stream(c->dev);
    WaitBatch b;
    std::memset(&b, 0, sizeof(b));
    b.timeout_ns = timeout_ns_;
    b.status = c->status_d;
    for (auto& st : kv.second) {
      if (b.n == static_cast<std::uint32_t>(kMaxWaitFlags)) {
        CMX_CUDA(launch_wait(b, cur));
        kernel_launches++;
        st_wait_kernels_++;
        b.n = 0;
      }
      b.flag[b.n] = c->mbox + st->slot;
      b.val[b.n] = st->value;
      ++b.n;
    }
    if (b.n) {
      CMX_CUDA(launch_wait(b, cur));
      kernel_launches++;
      st_wait_kernels_++;
    }
  }
}

void CudaTransport::stream_wait(const ReqPtr& r) { stream_wait_all({r}); }

void CudaTransport::stream_wait_all(const std::vector<ReqPtr>& rs) {
  // One stream wait per distinct event: the messages of one batch share the
  // event of their launch.
  std::vector<ReqPtr> dev_sends;
  std::vector<std::pair<int, cudaEvent_t>> events;
  auto add = [&](int dev, const EventPtr& e) {
    if (!e) return;
    for (auto& x : events)
      if (x.second == e->ev) return;
    events.push_back({dev, e->ev});
  };
  for (auto& r : rs) {
    if (!r->dev || r->state.load() != kDone) continue;
    if (r->kind == ReqKind::Recv) {
      auto st = state<RecvState>(r);
      add(st->device, st->done);
    } else {
      auto st = state<SendState>(r);
      if (st->local)
        add(st->device, st->local_done);
      else if (st->device_wait)
        dev_sends.push_back(r);
    }
  }
  for (auto& e : events) {
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(e.first));
    CMX_CUDA(cudaStreamWaitEvent(current_stream(e.first), e.second, 0));
  }
  if (!dev_sends.empty()) wait_sends_on_stream(dev_sends);
}

bool CudaTransport::query(const ReqPtr& r) {
  if (!r->dev) return true;
  if (r->kind == ReqKind::Recv) {
    auto st = state<RecvState>(r);
    return st->done && cudaEventQuery(st->done->ev) == cudaSuccess;
  }
  auto st = state<SendState>(r);
  if (st->local) return st->local_done && cudaEventQuery(st->local_done->ev) == cudaSuccess;
  return st->fin.load(std::memory_order_acquire);
}

std::string CudaTransport::device_error() {
  {
    std::lock_guard<SpinMutex> lk(pend_mu_);
    if (!dev_error_.empty()) return dev_error_;
  }
  std::lock_guard<std::mutex> lk(ctx_mu_);
  for (auto& kv : ctx_) {
    volatile unsigned long long* st = kv.second->status_h;
    unsigned long long code = st[0];
    if (code == kStatusOk) continue;
    std::ostringstream os;
    if (code == kStatusWaitTimeout)
      os << "commux: a device-side wait on GPU " << kv.first << " gave up after "
         << timeout_ns_ / 1000000 << " ms (flag 0x" << std::hex << st[1] << std::dec
         << " wanted " << st[2] << ", saw " << st[3] << "); the peer never completed its side";
    else if (code == kStatusBadDescriptor)
      os << "commux: a copy on GPU " << kv.first << " left its declared bounds (source 0x" << std::hex
         << st[1] << std::dec << ", byte offsets " << static_cast<long long>(st[2]) << " / "
         << static_cast<long long>(st[3]) << "); the unit was skipped";
    else if (code == kStatusCollTimeout)
      os << "commux: a device collective on GPU " << kv.first << " timed out waiting for rank "
         << st[1] << " (barrier epoch " << st[2] << ")";
    else
      os << "commux: device error code " << code << " on GPU " << kv.first;
    return os.str();
  }
  return "";
}

int CudaTransport::inflight() { return inflight_.load(); }

void CudaTransport::begin_batch() {
  std::lock_guard<SpinMutex> lk(batch_mu_);
  ++batch_depth_;
}

void CudaTransport::end_batch() {
  std::vector<std::pair<PendingPull, cudaStream_t>> todo;
  std::vector<ReqPtr> sends;
  {
    std::lock_guard<SpinMutex> lk(batch_mu_);
    if (batch_depth_ == 0 || --batch_depth_ > 0) return;
    todo.swap(batch_local_);
    sends.swap(batch_local_sends_);
    batch_event_.clear();
  }
  if (todo.empty()) return;
  std::map<std::pair<DevCtx*, cudaStream_t>, std::vector<PendingPull>> groups;
  std::map<std::pair<DevCtx*, cudaStream_t>, std::vector<ReqPtr>> group_sends;
  for (std::size_t i = 0; i < todo.size(); ++i) {
    auto key = std::make_pair(todo[i].first.ctx, todo[i].second);
    groups[key].push_back(std::move(todo[i].first));
    group_sends[key].push_back(sends[i]);
  }
  for (auto& kv : groups) {
    launch_batch(kv.first.first, kv.second, kv.first.second);
    EventPtr done = state<RecvState>(kv.second.front().r)->done;
    for (auto& s : group_sends[kv.first]) {
      state<SendState>(s)->local_done = done;
      eng_->complete(s);
    }
  }
}

std::vector<std::pair<std::string, std::int64_t>> CudaTransport::stats() {
  std::vector<std::pair<std::string, std::int64_t>> v = {
      {"cuda_pulls", st_pulls_.load()},
      {"cuda_pull_bytes", st_pull_bytes_.load()},
      {"cuda_kernel_launches", kernel_launches.load()},
      {"cuda_wait_kernels", st_wait_kernels_.load()},
      {"cuda_fins", st_fins_.load()},
      {"cuda_ipc_opens", st_ipc_opens_.load()},
      {"cuda_ipc_closes", st_ipc_closes_.load()},
      {"cuda_export_staged", st_export_staged_.load()},
      {"cuda_ipc_exports", st_ipc_exports_.load()},
      {"cuda_staged_sends", st_staged_.load()},
      {"cuda_sends_device_flag", st_sends_device_.load()},
      {"cuda_sends_host_fin", st_sends_host_.load()},
      {"cuda_pulls_peer_gpu", st_pulls_peer_gpu_.load()},
      {"cuda_pulls_same_gpu", st_pulls_same_gpu_.load()},
      {"cuda_plan_device_msgs", plan_device_msgs.load()},
      {"cuda_plan_shared_msgs", plan_shared_msgs.load()},
      {"cuda_plan_starts", plan_starts.load()},
  };
  if (coll_)
    for (auto& kv : coll_->stats()) v.push_back(kv);
  return v;
}

}  // namespace cuda
}  // namespace commux

extern "C" commux::DeviceTransport* commux_create_device_transport(commux::Engine* e) {
  return new commux::cuda::CudaTransport(e);
}
