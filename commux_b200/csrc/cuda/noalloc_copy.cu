// commux_strided_copy_noalloc: a strided copy through the pull kernel whose
// scratch (the per-descriptor completion counters the kernel counts into) is a
// file-scope device array instead of the per-stream cudaMalloc'd counters the
// p2p transport uses. The host side plans the descriptors on the stack
// (noalloc_plan.hpp) and checks both views against their allocations with
// driver queries, so a call allocates neither device nor host memory. The
// interface, its limits and its concurrency rules are documented in
// commux/noalloc.h.

#include <cuda.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "commux/noalloc.h"
#include "cuda_common.hpp"
#include "noalloc_plan.hpp"

namespace commux {
namespace cuda {
namespace {

using noalloc::fail;
using noalloc::NDim;
using noalloc::Wide;

constexpr int kNoAllocMaxDevices = 64;
constexpr std::size_t kNoAllocCounterBytes = noalloc::kDescs * sizeof(std::uint32_t);
constexpr std::size_t kNoAllocDoneOffset = 512;  // u64 completion flags, one per descriptor
constexpr std::size_t kNoAllocBytes = 1024;
static_assert(kNoAllocCounterBytes + 32 <= kNoAllocDoneOffset, "scratch layout");
static_assert(kNoAllocDoneOffset + noalloc::kDescs * sizeof(std::uint64_t) <= kNoAllocBytes, "scratch layout");
static_assert(noalloc::kDescs <= kMaxBatch, "one launch holds every descriptor");

// The scratch: [0, 256) the per-descriptor counters the kernel's warps count
// their slices into (u32 x 64), [256, 288) the kernel's status word (only
// written by ready-flag waits, which this path never has), [512, 1024) the
// per-descriptor completion flags the last warp of a descriptor stores
// (u64 x 64). All of it is zeroed on the caller's stream before each launch.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Zeroes the scratch (one CTA of 256 threads, a 32-bit word each). Device
// code names the array directly; host code only ever passes its address.
__global__ void noalloc_clear_kernel() {
  reinterpret_cast<std::uint32_t*>(g_noalloc_scratch)[threadIdx.x] = 0u;
}
static_assert(kNoAllocBytes == 256 * sizeof(std::uint32_t), "one word per thread");

struct DevSetup {
  unsigned char* scratch = nullptr;
  CUcontext ctx = nullptr;  // the primary context the address belongs to
  int sms = 0;
};
DevSetup g_setup[kNoAllocMaxDevices];
std::mutex g_setup_mu;

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

// The per-device set-up, under g_setup_mu: the scratch array's address in the
// device's primary context, the SM count, and every kernel a call can launch
// loaded now (CUDA loads kernels lazily on first use by default, and loading
// one may allocate device memory; after this, no later call does).
int setup(int dev, DevSetup& su, char* err, std::size_t err_len) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: set-up failed, cudaGetSymbolAddress: %s",
                cudaGetErrorString(e));
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess && sms <= 0) e = cudaErrorInvalidDevice;
  if (e == cudaSuccess) e = preload_pull_kernels();
  cudaFuncAttributes fa;
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, noalloc_clear_kernel);
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: set-up failed: %s",
                cudaGetErrorString(e));
  CUcontext ctx = nullptr;
  if (cuCtxGetCurrent(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: set-up failed: no current context");
  su.scratch = static_cast<unsigned char*>(p);
  su.ctx = ctx;
  su.sms = sms;
  return CMX_NOALLOC_OK;
}

// True when `cur` is the primary context of `dev` (the context the CUDA
// runtime, and so the scratch address, belongs to).
bool is_primary(CUcontext cur, int dev) {
  CUdevice d = 0;
  if (cuDeviceGet(&d, dev) != CUDA_SUCCESS) return false;
  unsigned int flags = 0;
  int active = 0;
  if (cuDevicePrimaryCtxGetState(d, &flags, &active) != CUDA_SUCCESS || !active) return false;
  CUcontext primary = nullptr;
  if (cuDevicePrimaryCtxRetain(&primary, d) != CUDA_SUCCESS) return false;  // active: no new context
  cuDevicePrimaryCtxRelease(d);
  return primary == cur;
}

}  // namespace
}  // namespace cuda
}  // namespace commux

extern "C" int commux_strided_copy_noalloc(void* dst, const int64_t* dst_strides, const void* src,
                                           const int64_t* src_strides, const int64_t* sizes, int ndim,
                                           int elem_bytes, void* stream, char* err, size_t err_len) {
  using namespace commux::cuda;
  if (err != nullptr && err_len > 0) err[0] = '\0';
  PullBatch b;  // on the stack (about 25 KB): no allocation
  noalloc::Plan plan;
  int rc = noalloc::plan_copy(dst, dst_strides, src, src_strides, sizes, ndim, elem_bytes, nullptr, b.d, plan, err,
                              err_len);
  if (rc != CMX_NOALLOC_OK || plan.ndesc == 0) return rc;

  // set-up, once per device (again if the device's primary context changed)
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: cudaGetDevice: %s",
                cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(err, err_len, CMX_NOALLOC_EINVAL, "commux_strided_copy_noalloc: device %d out of range", dev);
  CUcontext cur = nullptr;
  if (cuCtxGetCurrent(&cur) != CUDA_SUCCESS)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: cuCtxGetCurrent failed");
  DevSetup su;
  {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (g_setup[dev].scratch == nullptr || cur != g_setup[dev].ctx) {
      // a context other than the device's primary one is current: the
      // scratch address would belong to the wrong context
      if (cur != nullptr && !is_primary(cur, dev))
        return fail(err, err_len, CMX_NOALLOC_EINVAL,
                    "commux_strided_copy_noalloc: the current context is not the primary context of device %d; "
                    "make the primary context current (cuCtxSetCurrent) before the call",
                    dev);
      rc = setup(dev, g_setup[dev], err, err_len);
      if (rc != CMX_NOALLOC_OK) return rc;
    }
    su = g_setup[dev];
  }

  // both views inside their allocations on this device
  Wide lo = 0, hi = 0;
  noalloc::span(plan.dims, plan.n, true, plan.unit, lo, hi);
  rc = check_range(src, lo, hi, dev, "src", err, err_len);
  if (rc != CMX_NOALLOC_OK) return rc;
  noalloc::span(plan.dims, plan.n, false, plan.unit, lo, hi);
  rc = check_range(dst, lo, hi, dev, "dst", err, err_len);
  if (rc != CMX_NOALLOC_OK) return rc;

  b.n = plan.ndesc;
  b.total_chunks = plan.chunks;
  b.epoch = nullptr;
  b.trace = nullptr;
  b.trace_count = nullptr;
  b.cta_trace = nullptr;
  b.nsig = 0;
  b.bump = nullptr;
  b.cta_done = nullptr;
  b.nfin = 0;
  b.counters = reinterpret_cast<std::uint32_t*>(su.scratch);
  b.status = reinterpret_cast<unsigned long long*>(su.scratch + kNoAllocCounterBytes);
  b.timeout_ns = 0;
  auto* done = reinterpret_cast<std::uint64_t*>(su.scratch + kNoAllocDoneOffset);
  for (std::uint32_t i = 0; i < b.n; ++i) b.d[i].done = done + i;

  auto s = static_cast<cudaStream_t>(stream);
  noalloc_clear_kernel<<<1, 256, 0, s>>>();  // counters and flags start at zero
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: clear: %s", cudaGetErrorString(e));
  e = launch_pull(b, su.sms * 8, 256, s);
  if (e != cudaSuccess)
    return fail(err, err_len, CMX_NOALLOC_ECUDA, "commux_strided_copy_noalloc: launch: %s",
                cudaGetErrorString(e));
  return CMX_NOALLOC_OK;
}
