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
#include <sstream>

#include "coll.hpp"
#include "commux/process_group_ucx.hpp"

namespace commux {
namespace cuda {

namespace {

constexpr std::uint32_t kWireMagic = 0x54524443u;
constexpr int kWireDims = 8;
constexpr std::uint64_t kSlots = 1ull << 16;  // consumed-flag slots per device
constexpr std::uint64_t kMaxUnitsPerDesc = 1ull << 30;

// One tensor of a device message, as the sender describes it.
struct SegWire {
  std::uint64_t buffer_id;  // allocation id in the sender process (0: local)
  std::uint64_t base;       // allocation base address in the sender process
  std::uint64_t alloc_size;
  std::uint64_t offset;     // first element, bytes from base
  cudaIpcMemHandle_t handle;
  std::uint32_t elem;
  std::int32_t ndim;
  std::int64_t sizes[kWireDims];
  std::int64_t strides[kWireDims];  // elements
};

struct DrtsWire {
  std::uint32_t magic;
  std::uint32_t nseg;
  std::int32_t pid;
  std::int32_t device;
  unsigned char uuid[16];
  std::uint32_t sender_waits_on_device;
  std::uint32_t pad;
  std::uint64_t mbox_id;
  std::uint64_t mbox_base;
  cudaIpcMemHandle_t mbox_handle;
  std::uint64_t slot;
  std::uint64_t value;
};

cudaStream_t current_stream(int dev) {
  return c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream();
}

void cu_check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* s = nullptr;
  cuGetErrorString(r, &s);
  throw std::runtime_error(std::string("commux CUDA driver error in ") + what + ": " +
                           (s ? s : "unknown"));
}

template <typename T>
std::shared_ptr<T> state(const ReqPtr& r) {
  return std::static_pointer_cast<T>(r->dev);
}

// A tensor dimension as (size, src stride, dst stride), strides in elements
// or bytes depending on the stage.
struct Dim {
  std::int64_t size, ss, ds;
};

// Refine two shapes with equal element counts into one common shape (split
// dims where they differ) so a single index walks both. Returns false when no
// common refinement exists (e.g. sizes 6 and 4 facing each other).
bool refine(const std::vector<std::pair<std::int64_t, std::int64_t>>& a,
            const std::vector<std::pair<std::int64_t, std::int64_t>>& b, std::vector<Dim>& out) {
  out.clear();
  int i = static_cast<int>(a.size()) - 1, j = static_cast<int>(b.size()) - 1;
  if (i < 0 || j < 0) return false;
  std::int64_t ra = a[i].first, rb = b[j].first, sa = a[i].second, sb = b[j].second;
  while (i >= 0 && j >= 0) {
    std::int64_t m = std::min(ra, rb);
    if (m <= 0 || ra % m || rb % m) return false;
    out.push_back({m, sa, sb});
    if (ra == m) {
      if (--i >= 0) {
        ra = a[i].first;
        sa = a[i].second;
      }
    } else {
      ra /= m;
      sa *= m;
    }
    if (rb == m) {
      if (--j >= 0) {
        rb = b[j].first;
        sb = b[j].second;
      }
    } else {
      rb /= m;
      sb *= m;
    }
  }
  if (i >= 0 || j >= 0) return false;
  std::reverse(out.begin(), out.end());
  // merge dims that are contiguous in both
  std::vector<Dim> m;
  for (auto& d : out) {
    if (!m.empty() && m.back().ss == d.size * d.ss && m.back().ds == d.size * d.ds) {
      m.back().size *= d.size;
      m.back().ss = d.ss;
      m.back().ds = d.ds;
    } else {
      m.push_back(d);
    }
  }
  out.swap(m);
  return true;
}

std::vector<std::pair<std::int64_t, std::int64_t>> dims_of(const std::int64_t* sizes,
                                                           const std::int64_t* strides, int nd) {
  std::vector<std::pair<std::int64_t, std::int64_t>> v;
  for (int k = 0; k < nd; ++k)
    if (sizes[k] != 1) v.push_back({sizes[k], strides[k]});
  if (v.empty()) v.push_back({1, 1});
  return v;
}

// Turn common dims (element strides) into pull descriptors with the widest
// vector unit the alignment allows; appends to `out`.
void emit_descs(const char* sp, char* dp, std::vector<Dim> dims, std::int64_t elem,
                std::vector<PullDesc>& out) {
  // element strides -> byte strides
  for (auto& d : dims) {
    d.ss *= elem;
    d.ds *= elem;
  }
  std::int64_t unit = elem;
  Dim& in = dims.back();
  if (in.ss == elem && in.ds == elem) {
    std::int64_t inner_bytes = in.size * elem;
    for (std::int64_t u : {16, 8, 4, 2, 1}) {
      bool ok = inner_bytes % u == 0 && reinterpret_cast<std::uintptr_t>(sp) % u == 0 &&
                reinterpret_cast<std::uintptr_t>(dp) % u == 0;
      for (std::size_t k = 0; ok && k + 1 < dims.size(); ++k)
        ok = dims[k].ss % u == 0 && dims[k].ds % u == 0;
      if (ok) {
        unit = u;
        break;
      }
    }
    in.size = inner_bytes / unit;
    in.ss = unit;
    in.ds = unit;
    // a row of exactly one unit (e.g. a 16-byte x-face row): the row dim
    // adds nothing but a division per unit
    if (in.size == 1 && dims.size() > 1) dims.pop_back();
  } else if (!(elem == 1 || elem == 2 || elem == 4 || elem == 8 || elem == 16)) {
    throw std::runtime_error("commux: unsupported element size for a strided device copy");
  }
  if (dims.size() > static_cast<std::size_t>(kMaxPullDims))
    throw std::runtime_error("layout");
  // split along the outermost dim so every descriptor has < 2^30 units
  std::int64_t per0 = 1;
  for (std::size_t k = 1; k < dims.size(); ++k) per0 *= dims[k].size;
  if (per0 > static_cast<std::int64_t>(kMaxUnitsPerDesc))
    throw std::runtime_error("commux: device message row too large");
  std::int64_t step0 = std::max<std::int64_t>(1, static_cast<std::int64_t>(kMaxUnitsPerDesc) / per0);
  for (std::int64_t s0 = 0; s0 < dims[0].size; s0 += step0) {
    std::int64_t n0 = std::min(step0, dims[0].size - s0);
    PullDesc d{};
    d.src = sp + s0 * dims[0].ss;
    d.dst = dp + s0 * dims[0].ds;
    d.ndim = static_cast<std::uint32_t>(dims.size());
    d.unit = static_cast<std::uint32_t>(unit);
    const int off = kMaxPullDims - static_cast<int>(dims.size());
    for (int k = 0; k < kMaxPullDims; ++k) {
      d.div[k] = FastDiv(1);
      d.sst[k] = 0;
      d.dstr[k] = 0;
    }
    std::int64_t units = 1;
    for (std::size_t k = 0; k < dims.size(); ++k) {
      std::int64_t sz = k == 0 ? n0 : dims[k].size;
      d.div[off + k] = FastDiv(static_cast<std::uint32_t>(sz));
      d.sst[off + k] = dims[k].ss;
      d.dstr[off + k] = dims[k].ds;
      units *= sz;
    }
    d.units = static_cast<std::uint32_t>(units);
    d.nchunks = static_cast<std::uint32_t>(std::max<std::int64_t>(1, (units + kChunkUnits - 1) / kChunkUnits));
    // the kernel's common walk holds strides in 32 bits
    constexpr std::int64_t lim = std::int64_t{1} << 31;
    for (int k = 0; k < kMaxPullDims; ++k)
      if (d.sst[k] >= lim || d.sst[k] <= -lim || d.dstr[k] >= lim || d.dstr[k] <= -lim) d.wide = 1;
    out.push_back(d);
  }
}

// Host-side bounds check of every descriptor before launch: the bytes a
// descriptor touches must lie inside the source allocation (the IPC mapping)
// and the destination storage. A layout bug then raises here instead of
// reaching the GPU as an out-of-bounds access. The bounds-check build also
// hands the same limits to the kernel, which checks every unit it copies.
void check_desc(PullDesc& d, std::uintptr_t src_lo, std::uintptr_t src_hi,
                std::uintptr_t dst_lo, std::uintptr_t dst_hi) {
  if (d.units == 0) return;
  std::int64_t s_min = 0, s_max = 0, d_min = 0, d_max = 0;
  for (int k = 0; k < kMaxPullDims; ++k) {
    std::int64_t ext = static_cast<std::int64_t>(d.div[k].d) - 1;
    std::int64_t a = ext * d.sst[k], b = ext * d.dstr[k];
    (a < 0 ? s_min : s_max) += a;
    (b < 0 ? d_min : d_max) += b;
  }
  auto sp = reinterpret_cast<std::intptr_t>(d.src), dp = reinterpret_cast<std::intptr_t>(d.dst);
  bool ok = sp + s_min >= static_cast<std::intptr_t>(src_lo) &&
            sp + s_max + static_cast<std::intptr_t>(d.unit) <= static_cast<std::intptr_t>(src_hi) &&
            dp + d_min >= static_cast<std::intptr_t>(dst_lo) &&
            dp + d_max + static_cast<std::intptr_t>(d.unit) <= static_cast<std::intptr_t>(dst_hi);
  if (!ok)
    throw std::runtime_error("commux: internal error, a copy descriptor leaves its buffers "
                             "(layout bug caught before launch)");
#if defined(COMMUX_DEVICE_CHECKS)
  d.src_lo = static_cast<std::intptr_t>(src_lo) - sp;
  d.src_hi = static_cast<std::intptr_t>(src_hi) - sp;
  d.dst_lo = static_cast<std::intptr_t>(dst_lo) - dp;
  d.dst_hi = static_cast<std::intptr_t>(dst_hi) - dp;
#endif
}

bool contiguous_wire(const SegWire& s) {
  std::int64_t expect = 1;
  for (int k = s.ndim - 1; k >= 0; --k) {
    if (s.sizes[k] != 1 && s.strides[k] != expect) return false;
    expect *= s.sizes[k];
  }
  return true;
}

std::int64_t numel_wire(const SegWire& s) {
  std::int64_t n = 1;
  for (int k = 0; k < s.ndim; ++k) n *= s.sizes[k];
  return n;
}

// Narrow rows (a halo x-face: 16-byte runs at a row pitch) cross NVLink far
// below its bandwidth when a peer reads them one by one; such a send is
// packed into a contiguous staging buffer on its own GPU first, and the
// receiver reads that buffer.
constexpr std::int64_t kPackRunBytes = 512;

bool narrow_rows(const at::Tensor& t) {
  if (t.numel() == 0 || t.dim() > kWireDims) return false;
  std::vector<std::int64_t> sz(t.sizes().begin(), t.sizes().end()), sd(t.strides().begin(), t.strides().end());
  auto d = dims_of(sz.data(), sd.data(), t.dim());
  std::vector<Dim> m;
  if (!refine(d, d, m) || m.empty()) return false;
  const Dim& in = m.back();
  const std::int64_t run = (in.ss == 1 ? in.size : 1) * static_cast<std::int64_t>(t.element_size());
  return run < kPackRunBytes;
}

}  // namespace

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
    std::lock_guard<std::mutex> lk(pend_mu_);
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
  std::lock_guard<std::mutex> lk(ipc_mu_);
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
  std::lock_guard<std::mutex> lk(ipc_mu_);
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
  std::lock_guard<std::mutex> lk(ipc_mu_);
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
    std::lock_guard<std::mutex> lk(batch_mu_);
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
  std::lock_guard<std::mutex> lk(pend_mu_);
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
    std::lock_guard<std::mutex> lk(batch_mu_);
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
  try {
    build_descs(r, blob, len, local, pp);
  } catch (const std::exception& e) {
    if (!local) eng_->send_fin(src, send_id, -4);
    if (s) eng_->fail(s, e.what());
    eng_->fail(r, e.what());
    return;
  }
  st_pulls_++;
  if (!local) {
    {
      std::lock_guard<std::mutex> lk(pend_mu_);
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
    std::lock_guard<std::mutex> lk(batch_mu_);
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
  bool busy = false;
  std::vector<PendingPull> ready;
  {
    std::lock_guard<std::mutex> lk(pend_mu_);
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
      for (auto& p : kv.second) {
        f.fins.push_back({p.src, p.send_id});
        f.reqs.push_back(p.r);
      }
      launch_batch(kv.first, kv.second, kv.first->comm);
      f.done = state<RecvState>(f.reqs.front())->done;
      flights_.push_back(std::move(f));
    }
  }
  while (!flights_.empty()) {
    Flight& f = flights_.front();
    cudaError_t e = cudaEventQuery(f.done->ev);
    if (e == cudaErrorNotReady) break;
    if (e != cudaSuccess) {
      cudaGetLastError();
      std::lock_guard<std::mutex> lk(pend_mu_);
      dev_error_ = std::string("commux: CUDA error in a pull: ") + cudaGetErrorString(e);
    }
    for (auto& fin : f.fins) {
      eng_->send_fin(fin.first, fin.second, e == cudaSuccess ? 0 : -5);
      st_fins_++;
    }
    inflight_.fetch_sub(static_cast<int>(f.fins.size()));
    flights_.pop_front();
    busy = true;
  }
  return busy;
}

void CudaTransport::on_fin(const ReqPtr& s, std::int64_t status) {
  auto st = state<SendState>(s);
  if (st) st->fin.store(true, std::memory_order_release);
  if (status != 0) {
    const char* why = status == -3   ? "the receiver shares this GPU but the send expected a peer GPU"
                      : status == -4 ? "the receiver could not describe the copy (layout/size mismatch)"
                      : status == -5 ? "the receiver's copy kernel failed"
                                     : "the receiver rejected the message";
    eng_->fail(s, std::string("commux send: ") + why);
    return;
  }
  if (st && !st->device_wait) eng_->complete(s);
}

void CudaTransport::wait_sends_on_stream(const std::vector<ReqPtr>& sends) {
  // group the device-side waits per device into one-warp launches
  std::map<int, std::vector<std::shared_ptr<SendState>>> by_dev;
  for (auto& s : sends) {
    auto st = state<SendState>(s);
    if (st->fin.load(std::memory_order_acquire)) continue;  // consumed already
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
    std::lock_guard<std::mutex> lk(pend_mu_);
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
  std::lock_guard<std::mutex> lk(batch_mu_);
  ++batch_depth_;
}

void CudaTransport::end_batch() {
  std::vector<std::pair<PendingPull, cudaStream_t>> todo;
  std::vector<ReqPtr> sends;
  {
    std::lock_guard<std::mutex> lk(batch_mu_);
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
  };
  if (coll_)
    for (auto& kv : coll_->stats()) v.push_back(kv);
  return v;
}

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
    cudaGetLastError();
  }
  std::vector<Msg> sends, recvs;

  // Builds the launches every start() replays: (1) pack + "ready" signals of
  // the sends to other GPUs (without packing, the signals are stored by the
  // first pull launch at entry instead), (2) the pulls of every receive, (3)
  // the wait for the receivers' "consumed" flags, ending with the epoch bump.
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
    if (merge) {
      pull.insert(pull.begin(), packs.begin(), packs.end());
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
    // device state: [epoch u64, starts at 1][counters u32 x kCounterSlots]
    const std::size_t state_bytes = 64 + kCounterSlots * sizeof(std::uint32_t);
    state_ = at::empty({static_cast<std::int64_t>(state_bytes)},
                       at::TensorOptions().dtype(at::kByte).device(at::kCUDA, c_->dev));
    epoch_d_ = reinterpret_cast<std::uint64_t*>(state_.data_ptr());
    counters_d_ = reinterpret_cast<std::uint32_t*>(static_cast<char*>(state_.data_ptr()) + 64);
    std::vector<char> init(state_bytes, 0);
    const std::uint64_t one = 1;
    std::memcpy(init.data(), &one, sizeof(one));
    CMX_CUDA(cudaMemcpy(state_.data_ptr(), init.data(), state_bytes, cudaMemcpyHostToDevice));
    pre_ = batches(pre);
    pulls_ = batches(pull);
    if (!ready_only.empty()) {
      TORCH_CHECK(ready_only.size() <= static_cast<std::size_t>(kMaxEntrySignals), "commux plan: more than ",
                  kMaxEntrySignals, " unpacked sends to other GPUs");
      PullBatch& first = pre_.empty() ? *pulls_[0] : *pre_[0];
      first.nsig = static_cast<std::uint32_t>(ready_only.size());
      for (std::size_t k = 0; k < ready_only.size(); ++k) first.sig[k] = ready_only[k];
    }
    std::memset(&wait_, 0, sizeof(wait_));
    wait_.timeout_ns = tr_->device_timeout_ns();
    wait_.status = c_->status_d;
    wait_.epoch = epoch_d_;
    wait_.bump = epoch_d_;  // the wait launch also advances the epoch
    for (auto& m : sends)
      if (m.mode == PlanMode::Device) {
        TORCH_CHECK(wait_.n < static_cast<std::uint32_t>(kMaxWaitFlags), "commux plan: more than ",
                    kMaxWaitFlags, " sends to other GPUs");
        wait_.flag[wait_.n++] = m.consumed_local;
      }
    // COMMUX_PLAN_TRACE: span of every launch of a start (earliest CTA start,
    // latest CTA end), printed after each start (which then synchronises)
    if (env_int("COMMUX_PLAN_TRACE", 0) != 0) {
      const std::size_t n = pre_.size() + pulls_.size() + 1;
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
      wait_.trace = d + 2 * k;
      trace_n_ = n;
    }
  }

  void start() override {
    ++starts_;
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(c_->dev));
    cudaStream_t cur = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(c_->dev)).stream();
    // messages to/from a rank on this same GPU go through the host-gated path
    std::vector<ReqPtr> shared;
    if (n_shared_) {
      tr_->begin_batch();
      try {
        for (auto& m : recvs)
          if (m.mode == PlanMode::Shared)
            shared.push_back(eng_->post_recv({m.t}, m.peer, make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), 0, false)));
        for (auto& m : sends)
          if (m.mode == PlanMode::Shared)
            shared.push_back(eng_->post_send({m.t}, m.peer, make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), 0, false)));
      } catch (...) {
        tr_->end_batch();
        throw;
      }
      tr_->end_batch();
    }
    if (!exec_) capture();
    last_stream_ = cur;
    if (trace_h_ != nullptr)
      for (std::size_t k = 0; k < trace_n_; ++k) {
        trace_h_[2 * k] = ~0ull;
        trace_h_[2 * k + 1] = 0;
      }
    CMX_CUDA(cudaGraphLaunch(exec_, cur));
    tr_->kernel_launches += nodes_;
    if (trace_h_ != nullptr) report_trace(cur);
    if (!shared.empty()) {
      for (auto& r : shared) eng_->wait(r, std::chrono::milliseconds(0));
      tr_->stream_wait_all(shared);
    }
    std::string e = tr_->device_error();
    if (!e.empty()) C10_THROW_ERROR(DistBackendError, e);
  }

  std::vector<std::pair<std::string, std::int64_t>> info() override {
    std::int64_t loc = 0, dev = 0, packed = 0;
    for (auto* v : {&sends, &recvs})
      for (auto& m : *v) (m.mode == PlanMode::Local ? loc : dev) += m.mode != PlanMode::Shared;
    for (auto& m : sends) packed += (m.mode == PlanMode::Device && !m.pack.empty()) ? 1 : 0;
    return {{"local", loc},      {"device", dev},       {"shared", n_shared_}, {"packed_sends", packed},
            {"graph_nodes", nodes_}, {"starts", static_cast<std::int64_t>(starts_)}};
  }

  std::int64_t n_shared_ = 0;

 private:
  void report_trace(cudaStream_t cur) {
    CMX_CUDA(cudaStreamSynchronize(cur));
    unsigned long long t0 = ~0ull;
    for (std::size_t k = 0; k < trace_n_; ++k) t0 = std::min(t0, trace_h_[2 * k]);
    std::string line;
    char buf[96];
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
    span("wait");
    std::fprintf(stderr, "[commux plan trace rank %d] start %llu, us from the first CTA:%s\n", eng_->rank(),
                 static_cast<unsigned long long>(starts_), line.c_str());
  }

  // Messages -> parameter blocks of at most kMaxBatch descriptors, one unit
  // class each; every message counts into its own counter slot (the plan's
  // launches run one after another and each message returns its counter to
  // zero, so the slots are reused by the next start).
  std::vector<std::unique_ptr<PullBatch>> batches(const std::vector<std::vector<PullDesc>>& msgs) {
    std::map<int, std::vector<PullDesc>> by_cls;
    std::uint32_t slot = 0;
    for (auto& m : msgs) {
      if (m.empty()) continue;
      const int cls = pull_unit_class(m[0]);
      std::uint32_t chunks = 0;
      for (auto& d : m) {
        TORCH_CHECK(pull_unit_class(d) == cls, "commux plan: a message mixes unit classes");
        chunks += d.nchunks;
      }
      TORCH_CHECK(slot < kCounterSlots - 1, "commux plan: too many messages");
      auto& v = by_cls[cls];
      for (auto d : m) {
        d.counter_idx = slot;
        d.msg_chunks = chunks;
        v.push_back(d);
      }
      ++slot;
    }
    std::vector<std::unique_ptr<PullBatch>> out;
    for (auto& kv : by_cls) {
      std::size_t i = 0;
      while (i < kv.second.size()) {
        auto b = std::make_unique<PullBatch>();
        b->n = 0;
        b->total_chunks = 0;
        b->counters = counters_d_;
        b->status = c_->status_d;
        b->timeout_ns = tr_->device_timeout_ns();
        b->epoch = epoch_d_;
        b->nsig = 0;
        while (i < kv.second.size() && b->n < static_cast<std::uint32_t>(kMaxBatch)) {
          PullDesc d = kv.second[i++];
          d.chunk0 = b->total_chunks;
          b->total_chunks += d.nchunks;
          b->d[b->n++] = d;
        }
        out.push_back(std::move(b));
      }
    }
    return out;
  }

  void capture() {
    cudaStream_t cs = nullptr;
    CMX_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    // a launch whose CTAs wait on peers keeps every CTA resident at once, so
    // a CTA never waits while another CTA of the launch that still has pack
    // work waits for an SM; launches without waits keep the wider grid
    bool waits = false;
    for (auto& m : recvs) waits |= m.mode == PlanMode::Device;
    const int ctas = waits ? std::min(tr_->pull_ctas(c_), 4 * c_->sm_count) : tr_->pull_ctas(c_);
    nodes_ = 0;
    CMX_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    for (auto* ls : {&pre_, &pulls_})
      for (auto& b : *ls) {
        int launched = 0;
        if (e == cudaSuccess) e = launch_pull(*b, ctas, 256, cs, &launched);
        nodes_ += launched;
      }
    // waits (if any), then the epoch bump; a plan whose every message stays
    // on this GPU has no flags, so no epoch to advance and no launch here
    bool flags = wait_.n > 0;
    for (auto& m : recvs) flags |= m.mode == PlanMode::Device;
    if (e == cudaSuccess && flags) {
      e = launch_wait(wait_, cs);
      ++nodes_;
    }
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
  std::uint32_t* counters_d_ = nullptr;
  std::vector<std::unique_ptr<PullBatch>> pre_, pulls_;
  WaitBatch wait_{};
  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t exec_ = nullptr;
  std::int64_t nodes_ = 0;
  unsigned long long* trace_h_ = nullptr;  // COMMUX_PLAN_TRACE (host-mapped)
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
      reply_recvs.push_back({plan->sends.size(),
                             eng_->post_recv({rb}, m.peer, make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), kPlanReplySub, true)),
                             rb});
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
      desc_recvs.push_back({plan->recvs.size(),
                            eng_->post_recv({db}, m.peer, make_ucp_tag(0, static_cast<std::uint32_t>(m.tag), kPlanSub, true)),
                            db});
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
  plan->finalize();
  return plan;
}

}  // namespace cuda
}  // namespace commux

extern "C" commux::DeviceTransport* commux_create_device_transport(commux::Engine* e) {
  return new commux::cuda::CudaTransport(e);
}
