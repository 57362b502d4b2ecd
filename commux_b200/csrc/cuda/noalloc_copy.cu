// commux_strided_copy_noalloc: a strided copy through the pull kernel whose
// scratch (the per-descriptor completion counters the kernel counts into) is a
// file-scope device array instead of the per-stream cudaMalloc'd counters the
// p2p transport uses. The host side builds the descriptors on the stack and
// checks both views against their allocations with driver queries, so a call
// allocates neither device nor host memory. The interface, its limits and its
// concurrency rules are documented in commux/noalloc.h.

#include <cuda.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "commux/noalloc.h"
#include "cuda_common.hpp"

namespace commux {
namespace cuda {
namespace {

constexpr int kNoAllocDescs = 64;              // counters = copy descriptors per call
constexpr int kNoAllocMaxInDims = 8;
constexpr int kNoAllocMaxDevices = 64;
constexpr std::int64_t kNoAllocUnitsPerDesc = std::int64_t{1} << 30;
constexpr std::int64_t kNoAllocMaxExtent = std::int64_t{1} << 40;  // sizes and strides, elements
constexpr std::size_t kNoAllocCounterBytes = kNoAllocDescs * sizeof(std::uint32_t);
constexpr std::size_t kNoAllocDoneOffset = 512;  // u64 completion flags, one per descriptor
constexpr std::size_t kNoAllocBytes = 1024;
static_assert(kNoAllocCounterBytes + 32 <= kNoAllocDoneOffset, "scratch layout");
static_assert(kNoAllocDoneOffset + kNoAllocDescs * sizeof(std::uint64_t) <= kNoAllocBytes, "scratch layout");
static_assert(kNoAllocDescs <= kMaxBatch, "one launch holds every descriptor");

// The scratch: [0, 256) the per-descriptor counters the kernel's warps count
// their slices into (u32 x 64), [256, 288) the kernel's status word (only
// written by ready-flag waits, which this path never has), [512, 1024) the
// per-descriptor completion flags the last warp of a descriptor stores
// (u64 x 64). All of it is zeroed on the caller's stream before each launch.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

struct DevSetup {
  unsigned char* scratch = nullptr;
  int sms = 0;
};
DevSetup g_setup[kNoAllocMaxDevices];
std::mutex g_setup_mu;

int fail(char* err, std::size_t len, int code, const char* fmt, ...) {
  if (err != nullptr && len > 0) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(err, len, fmt, ap);
    va_end(ap);
  }
  return code;
}

struct NDim {
  std::int64_t size, ss, ds;  // elements, then bytes
};

using Wide = __int128;  // extents of hostile sizes x strides cannot overflow

// Byte extent [lo, hi) of a view relative to its pointer.
void span(const NDim* d, int n, bool src, std::int64_t unit, Wide& lo, Wide& hi) {
  lo = 0;
  hi = unit;
  for (int k = 0; k < n; ++k) {
    const Wide e = static_cast<Wide>(d[k].size - 1) * (src ? d[k].ss : d[k].ds);
    (e < 0 ? lo : hi) += e;
  }
}

int check_range(const void* p, Wide lo, Wide hi, int dev, const char* which, char* err,
                std::size_t len) {
  CUpointer_attribute attrs[3] = {CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, CU_POINTER_ATTRIBUTE_RANGE_SIZE,
                                  CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL};
  CUdeviceptr start = 0;
  std::size_t size = 0;
  int ordinal = -1;
  void* data[3] = {&start, &size, &ordinal};
  if (cuPointerGetAttributes(3, attrs, data, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS || start == 0)
    return fail(err, len, CMX_NOALLOC_ERANGE, "commux_strided_copy_noalloc: %s %p is not device memory", which, p);
  if (ordinal != dev)
    return fail(err, len, CMX_NOALLOC_ERANGE,
                "commux_strided_copy_noalloc: %s is on device %d, the current device is %d", which, ordinal, dev);
  const auto a = static_cast<Wide>(reinterpret_cast<std::uintptr_t>(p));
  const auto s = static_cast<Wide>(start);
  if (a + lo < s || a + hi > s + static_cast<Wide>(size))
    return fail(err, len, CMX_NOALLOC_ERANGE,
                "commux_strided_copy_noalloc: the %s view [%lld, %lld) bytes around %p leaves its "
                "allocation of %zu bytes",
                which, static_cast<long long>(lo), static_cast<long long>(hi), p, size);
  return CMX_NOALLOC_OK;
}

}  // namespace
}  // namespace cuda
}  // namespace commux

extern "C" int commux_strided_copy_noalloc(void* dst, const int64_t* dst_strides, const void* src,
                                           const int64_t* src_strides, const int64_t* sizes, int ndim,
                                           int elem_bytes, void* stream, char* err, size_t err_len) {
  using namespace commux::cuda;
  if (err != nullptr && err_len > 0) err[0] = '\0';
  if (dst == nullptr || src == nullptr || sizes == nullptr || dst_strides == nullptr ||
      src_strides == nullptr || ndim < 0 || ndim > kNoAllocMaxInDims)
    return fail(err, err_len, CMX_NOALLOC_EINVAL,
                "commux_strided_copy_noalloc: null pointer or ndim outside [0, %d]", kNoAllocMaxInDims);
  const std::int64_t elem = elem_bytes;
  if (!(elem == 1 || elem == 2 || elem == 4 || elem == 8 || elem == 16))
    return fail(err, err_len, CMX_NOALLOC_EINVAL,
                "commux_strided_copy_noalloc: elem_bytes must be 1, 2, 4, 8 or 16 (got %d)", elem_bytes);
  if (reinterpret_cast<std::uintptr_t>(src) % elem || reinterpret_cast<std::uintptr_t>(dst) % elem)
    return fail(err, err_len, CMX_NOALLOC_EINVAL,
                "commux_strided_copy_noalloc: src and dst must be aligned to elem_bytes");

  // dims: drop size-1 dims, then merge neighbours contiguous in both views
  NDim d[kNoAllocMaxInDims];
  int n = 0;
  for (int k = 0; k < ndim; ++k) {
    if (sizes[k] < 0)
      return fail(err, err_len, CMX_NOALLOC_EINVAL, "commux_strided_copy_noalloc: negative size");
    if (sizes[k] == 0) return CMX_NOALLOC_OK;  // nothing to copy
    if (sizes[k] == 1) continue;
    if (sizes[k] > kNoAllocMaxExtent || src_strides[k] > kNoAllocMaxExtent || src_strides[k] < -kNoAllocMaxExtent ||
        dst_strides[k] > kNoAllocMaxExtent || dst_strides[k] < -kNoAllocMaxExtent)
      return fail(err, err_len, CMX_NOALLOC_ETOOBIG,
                  "commux_strided_copy_noalloc: too large, a size or stride exceeds 2^40 elements");
    NDim cur{sizes[k], src_strides[k], dst_strides[k]};
    if (n > 0 && static_cast<Wide>(d[n - 1].ss) == static_cast<Wide>(cur.size) * cur.ss &&
        static_cast<Wide>(d[n - 1].ds) == static_cast<Wide>(cur.size) * cur.ds) {
      if (d[n - 1].size > kNoAllocMaxExtent / cur.size)
        return fail(err, err_len, CMX_NOALLOC_ETOOBIG, "commux_strided_copy_noalloc: view too large");
      d[n - 1] = NDim{d[n - 1].size * cur.size, cur.ss, cur.ds};
    } else {
      d[n++] = cur;
    }
  }
  if (n == 0) d[n++] = NDim{1, 1, 1};
  for (int k = 0; k < n; ++k) {
    d[k].ss *= elem;
    d[k].ds *= elem;
  }
  // widest vector unit: the innermost dim, when contiguous in both, becomes
  // a run of 16/8/4/2/1-byte units
  std::int64_t unit = elem;
  NDim& in = d[n - 1];
  if (in.ss == elem && in.ds == elem) {
    const std::int64_t inner = in.size * elem;
    for (std::int64_t u : {16, 8, 4, 2, 1}) {
      bool ok = inner % u == 0 && reinterpret_cast<std::uintptr_t>(src) % u == 0 &&
                reinterpret_cast<std::uintptr_t>(dst) % u == 0;
      for (int k = 0; ok && k + 1 < n; ++k) ok = d[k].ss % u == 0 && d[k].ds % u == 0;
      if (ok) {
        unit = u;
        break;
      }
    }
    in = NDim{inner / unit, unit, unit};
    if (in.size == 1 && n > 1) --n;
  }
  if (n > kMaxPullDims)
    return fail(err, err_len, CMX_NOALLOC_ELAYOUT,
                "commux_strided_copy_noalloc: %d dims remain after merging, at most %d are supported", n,
                kMaxPullDims);
  std::int64_t per0 = 1;
  for (int k = 1; k < n; ++k) {
    if (d[k].size > kNoAllocUnitsPerDesc / per0)
      return fail(err, err_len, CMX_NOALLOC_ETOOBIG,
                  "commux_strided_copy_noalloc: too large, the dims inside the outermost one hold more "
                  "than 2^30 units of %lld bytes",
                  static_cast<long long>(unit));
    per0 *= d[k].size;
  }
  const std::int64_t step0 = kNoAllocUnitsPerDesc / per0;
  const std::int64_t ndesc = (d[0].size + step0 - 1) / step0;
  if (ndesc > kNoAllocDescs)
    return fail(err, err_len, CMX_NOALLOC_ETOOBIG,
                "commux_strided_copy_noalloc: too large, the copy needs %lld descriptors and the static "
                "scratch has counters for %d (at most %lld units of %lld bytes)",
                static_cast<long long>(ndesc), kNoAllocDescs,
                static_cast<long long>(kNoAllocDescs * kNoAllocUnitsPerDesc), static_cast<long long>(unit));

  // set-up, once per device: the scratch array's address on this device
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: cudaGetDevice: %s",
                cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(err, err_len, CMX_NOALLOC_EINVAL, "commux_strided_copy_noalloc: device %d out of range", dev);
  DevSetup su;
  {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (g_setup[dev].scratch == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr)
        return fail(err, err_len, CMX_NOALLOC_ECUDA,
                    "commux_strided_copy_noalloc: set-up failed, cudaGetSymbolAddress: %s",
                    cudaGetErrorString(e));
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess || sms <= 0)
        return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: set-up failed: %s",
                    cudaGetErrorString(e));
      g_setup[dev].sms = sms;
      g_setup[dev].scratch = static_cast<unsigned char*>(p);
    }
    su = g_setup[dev];
  }
  // the primary context is current on this thread (driver queries below)
  e = cudaSetDevice(dev);
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: cudaSetDevice: %s",
                cudaGetErrorString(e));

  // both views inside their allocations on this device
  NDim rows[kMaxPullDims];
  for (int k = 0; k < n; ++k) rows[k] = d[k];
  Wide lo = 0, hi = 0;
  span(rows, n, true, unit, lo, hi);
  int rc = check_range(src, lo, hi, dev, "src", err, err_len);
  if (rc != CMX_NOALLOC_OK) return rc;
  span(rows, n, false, unit, lo, hi);
  rc = check_range(dst, lo, hi, dev, "dst", err, err_len);
  if (rc != CMX_NOALLOC_OK) return rc;

  // descriptors, one per slab of step0 outer rows, each its own message
  PullBatch b;
  b.n = 0;
  b.epoch = nullptr;
  b.trace = nullptr;
  b.trace_count = nullptr;
  b.nsig = 0;
  b.counters = reinterpret_cast<std::uint32_t*>(su.scratch);
  b.status = reinterpret_cast<unsigned long long*>(su.scratch + kNoAllocCounterBytes);
  b.timeout_ns = 0;
  std::uint32_t chunks = 0;
  const int off = kMaxPullDims - n;
  for (std::int64_t s0 = 0, i = 0; s0 < d[0].size; s0 += step0, ++i) {
    const std::int64_t n0 = d[0].size - s0 < step0 ? d[0].size - s0 : step0;
    PullDesc& x = b.d[i];
    x = PullDesc{};
    x.src = static_cast<const char*>(src) + s0 * d[0].ss;
    x.dst = static_cast<char*>(dst) + s0 * d[0].ds;
    x.ndim = static_cast<std::uint32_t>(n);
    x.unit = static_cast<std::uint32_t>(unit);
    std::int64_t units = 1;
    for (int k = 0; k < n; ++k) {
      const std::int64_t sz = k == 0 ? n0 : d[k].size;
      x.div[off + k] = FastDiv(static_cast<std::uint32_t>(sz));
      x.sst[off + k] = d[k].ss;
      x.dstr[off + k] = d[k].ds;
      units *= sz;
    }
    x.units = static_cast<std::uint32_t>(units);
    for (int k = 0; k < kMaxPullDims; ++k) {
      constexpr std::int64_t lim = std::int64_t{1} << 31;
      if (x.sst[k] >= lim || x.sst[k] <= -lim || x.dstr[k] >= lim || x.dstr[k] <= -lim) x.wide = 1;
    }
    x.nchunks = static_cast<std::uint32_t>((units + kChunkUnits - 1) / kChunkUnits);
    x.chunk0 = chunks;
    x.msg_chunks = x.nchunks;
    x.counter_idx = static_cast<std::uint32_t>(i);
    x.done = reinterpret_cast<std::uint64_t*>(su.scratch + kNoAllocDoneOffset) + i;
    x.done_val = 1;
    chunks += x.nchunks;
    b.n = static_cast<std::uint32_t>(i + 1);
  }
  b.total_chunks = chunks;

  auto s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(su.scratch, 0, kNoAllocBytes, s);  // counters and flags start at zero
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: cudaMemsetAsync: %s",
                cudaGetErrorString(e));
  e = launch_pull(b, su.sms * 8, 256, s);
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: launch: %s",
                cudaGetErrorString(e));
  return CMX_NOALLOC_OK;
}
