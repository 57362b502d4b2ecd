// Self-test of the bounds-check build (cmake -DCOMMUX_DEVICE_CHECKS=ON, or
// `python -m commux_b200.build --device-checks`).
//
// In that build every pull descriptor carries the byte limits the host-side
// check derived from the source allocation and the destination storage, and
// the pull kernel tests each unit against them before touching memory: a unit
// outside its limits is skipped and the first violation is written to the
// status word (kStatusBadDescriptor, the source address and both offsets),
// which the host turns into an error. A kernel index bug then shows up as a
// reported status instead of a wild access, and no wait or trap is involved.
//
// The self-test exercises exactly that path without any access outside real
// memory: it allocates buffers twice the size of the copy and declares limits
// narrower than the copy, so the units the kernel must refuse still lie inside
// the allocations. Cases: a copy inside its limits (status stays clear, all
// bytes copied), a source limit cut in half (status set, the first half
// copied, the second half untouched), a destination limit that excludes the
// first kilobyte, and the same source cut on the 64-bit-stride walk.
//
// The production build exports the same symbols: the self-test then returns
// 1 (not a bounds-check build) and commux_device_checks_enabled() returns 0.

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include "cuda_common.hpp"

namespace {

[[maybe_unused]] constexpr int kDisabled = 1;  // production build
#if defined(COMMUX_DEVICE_CHECKS)
constexpr int kOk = 0;
constexpr int kCuda = 2;   // a CUDA call failed
constexpr int kWrong = 3;  // the check did not behave as specified
#endif

int fail(char* err, std::size_t len, int code, const char* fmt, ...) {
  if (err != nullptr && len > 0) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(err, len, fmt, ap);
    va_end(ap);
  }
  return code;
}

}  // namespace

extern "C" int commux_device_checks_enabled(void) {
#if defined(COMMUX_DEVICE_CHECKS)
  return 1;
#else
  return 0;
#endif
}

extern "C" int commux_device_check_selftest(void* stream_ptr, char* err, std::size_t err_len) {
#if !defined(COMMUX_DEVICE_CHECKS)
  (void)stream_ptr;
  return fail(err, err_len, kDisabled, "library built without COMMUX_DEVICE_CHECKS");
#else
  using namespace commux::cuda;
  auto stream = static_cast<cudaStream_t>(stream_ptr);
  constexpr std::int64_t kCopy = 4096;   // bytes the descriptor walks
  constexpr std::int64_t kAlloc = 8192;  // bytes behind each pointer
  constexpr std::uint32_t kUnit = 16;

  char* src = nullptr;
  char* dst = nullptr;
  std::uint32_t* counters = nullptr;
  unsigned long long* status_h = nullptr;
  unsigned long long* status_d = nullptr;
  auto cleanup = [&] {
    if (src) cudaFree(src);
    if (dst) cudaFree(dst);
    if (counters) cudaFree(counters);
    if (status_h) cudaFreeHost(status_h);
  };
#define CMX_ST(call)                                                                        \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) {                                                                \
      cleanup();                                                                            \
      return fail(err, err_len, kCuda, "%s: %s", #call, cudaGetErrorString(e_));            \
    }                                                                                       \
  } while (0)
  CMX_ST(cudaMalloc(&src, kAlloc));
  CMX_ST(cudaMalloc(&dst, kAlloc));
  CMX_ST(cudaMalloc(&counters, kCounterSlots * sizeof(std::uint32_t)));
  CMX_ST(cudaMemsetAsync(counters, 0, kCounterSlots * sizeof(std::uint32_t), stream));
  CMX_ST(cudaHostAlloc(reinterpret_cast<void**>(&status_h), 64, cudaHostAllocMapped));
  CMX_ST(cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_d), status_h, 0));

  std::vector<unsigned char> pattern(kAlloc), got(kAlloc);
  for (std::int64_t i = 0; i < kAlloc; ++i) pattern[i] = static_cast<unsigned char>((i * 131 + 7) & 0xff);
  CMX_ST(cudaMemcpyAsync(src, pattern.data(), kAlloc, cudaMemcpyHostToDevice, stream));

  auto batch = std::make_unique<PullBatch>();  // ~29 KB: off the stack
  struct Case {
    const char* name;
    std::uint32_t wide;
    std::int64_t src_lo, src_hi, dst_lo, dst_hi;
    std::int64_t copied_lo, copied_hi;  // destination bytes expected to hold the source
    bool violation;
  };
  const Case cases[] = {
      {"inside its limits", 0, 0, kCopy, 0, kCopy, 0, kCopy, false},
      {"source limit at half", 0, 0, kCopy / 2, 0, kCopy, 0, kCopy / 2, true},
      {"destination limit from 1 KiB", 0, 0, kCopy, 1024, kCopy, 1024, kCopy, true},
      {"source limit at half, 64-bit walk", 1, 0, kCopy / 2, 0, kCopy, 0, kCopy / 2, true},
  };
  for (const Case& k : cases) {
    std::memset(status_h, 0, 64);
    CMX_ST(cudaMemsetAsync(dst, 0, kAlloc, stream));
    PullBatch& b = *batch;
    b = PullBatch{};
    b.n = 1;
    b.total_chunks = 1;
    b.counters = counters;
    b.status = status_d;
    b.timeout_ns = 1000000000ull;
    PullDesc& d = b.d[0];
    d.src = src;
    d.dst = dst;
    for (int i = 0; i < kMaxPullDims; ++i) d.div[i] = FastDiv(1);
    d.div[kMaxPullDims - 1] = FastDiv(static_cast<std::uint32_t>(kCopy / kUnit));
    d.sst[kMaxPullDims - 1] = kUnit;
    d.dstr[kMaxPullDims - 1] = kUnit;
    d.ndim = 1;
    d.unit = kUnit;
    d.units = static_cast<std::uint32_t>(kCopy / kUnit);
    d.chunk0 = 0;
    d.nchunks = 1;
    d.msg_chunks = 1;
    d.wide = k.wide;
    d.src_lo = k.src_lo;
    d.src_hi = k.src_hi;
    d.dst_lo = k.dst_lo;
    d.dst_hi = k.dst_hi;
    CMX_ST(launch_pull(b, 1, 256, stream));
    CMX_ST(cudaMemcpyAsync(got.data(), dst, kAlloc, cudaMemcpyDeviceToHost, stream));
    CMX_ST(cudaStreamSynchronize(stream));
    const unsigned long long code = status_h[0];
    if (k.violation != (code == kStatusBadDescriptor) || (!k.violation && code != kStatusOk)) {
      cleanup();
      return fail(err, err_len, kWrong, "case '%s': status %llu, expected %s", k.name, code,
                  k.violation ? "a bounds violation" : "none");
    }
    for (std::int64_t i = 0; i < kAlloc; ++i) {
      const bool copied = i >= k.copied_lo && i < k.copied_hi;
      const unsigned char want = copied ? pattern[i] : 0;
      if (got[i] != want) {
        cleanup();
        return fail(err, err_len, kWrong, "case '%s': destination byte %lld is %u, expected %u", k.name,
                    static_cast<long long>(i), got[i], want);
      }
    }
  }
#undef CMX_ST
  cleanup();
  return fail(err, err_len, kOk, "ok");
#endif
}
