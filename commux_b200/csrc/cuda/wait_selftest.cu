// Self-test of the bounded device waits, the GPU half of failure detection.
//
// Every device-side wait of the transport (the one-warp wait kernel on a
// sender's stream, the pull kernel's wait for a plan's "ready" flag, the
// collectives' flag rounds) spins on %globaltimer with a limit. Past the
// limit it records kStatusWaitTimeout in the host-mapped status word, with
// the flag's address, the value it wanted and the value it saw, and returns:
// no trap, no endless loop, and the context stays usable. The host turns the
// status into an error (CudaTransport::device_error).
//
// The self-test makes such waits run out on purpose, on flags that nothing
// sets, with a short limit:
//   1. the wait kernel on a flag left at 0 (wants 1): status, flag address,
//      wanted and seen values, and a duration at least the limit;
//   2. the same flag set to 1 afterwards: the wait completes, status clear
//      (the context survived);
//   3. a pull whose "ready" flag stays 0: status set, the destination
//      untouched, the completion flag not stored, the message's scratch
//      counter back at zero;
//   4. the same pull once the flag is set: the copy lands, the completion
//      flag is stored.
// Returns 0 on success, 2 when a CUDA call failed, 3 when a check failed,
// with a message in `err`.

#include <cuda_runtime.h>

#include <chrono>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include "cuda_common.hpp"

namespace {

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

extern "C" int commux_device_wait_selftest(void* stream_ptr, unsigned timeout_ms, char* err, std::size_t err_len) {
  using namespace commux::cuda;
  auto stream = static_cast<cudaStream_t>(stream_ptr);
  constexpr int kCuda = 2, kWrong = 3;
  constexpr std::size_t kBytes = 4096;
  const std::uint64_t timeout_ns = static_cast<std::uint64_t>(timeout_ms) * 1000000ull;

  std::uint64_t* flags = nullptr;  // [0] wait flag, [1] ready flag, [2] done flag
  char* src = nullptr;
  char* dst = nullptr;
  std::uint32_t* counters = nullptr;
  unsigned long long* status_h = nullptr;
  unsigned long long* status_d = nullptr;
  auto cleanup = [&] {
    if (flags) cudaFree(flags);
    if (src) cudaFree(src);
    if (dst) cudaFree(dst);
    if (counters) cudaFree(counters);
    if (status_h) cudaFreeHost(status_h);
  };
#define CMX_WT(call)                                                              \
  do {                                                                            \
    cudaError_t e_ = (call);                                                      \
    if (e_ != cudaSuccess) {                                                      \
      cleanup();                                                                  \
      return fail(err, err_len, kCuda, "%s: %s", #call, cudaGetErrorString(e_)); \
    }                                                                             \
  } while (0)
#define CMX_EXPECT(cond, ...)                          \
  do {                                                 \
    if (!(cond)) {                                     \
      cleanup();                                       \
      return fail(err, err_len, kWrong, __VA_ARGS__);  \
    }                                                  \
  } while (0)

  CMX_WT(cudaMalloc(&flags, 3 * sizeof(std::uint64_t)));
  CMX_WT(cudaMalloc(&src, kBytes));
  CMX_WT(cudaMalloc(&dst, kBytes));
  CMX_WT(cudaMalloc(&counters, kCounterSlots * sizeof(std::uint32_t)));
  CMX_WT(cudaHostAlloc(reinterpret_cast<void**>(&status_h), 64, cudaHostAllocMapped));
  CMX_WT(cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_d), status_h, 0));
  CMX_WT(cudaMemsetAsync(flags, 0, 3 * sizeof(std::uint64_t), stream));
  CMX_WT(cudaMemsetAsync(counters, 0, kCounterSlots * sizeof(std::uint32_t), stream));
  CMX_WT(cudaMemsetAsync(src, 0x5a, kBytes, stream));
  CMX_WT(cudaMemsetAsync(dst, 0, kBytes, stream));
  CMX_WT(cudaStreamSynchronize(stream));
  const std::uint64_t one = 1;

  // 1. the wait kernel gives up on a flag nothing sets
  std::memset(status_h, 0, 64);
  WaitBatch w;
  std::memset(&w, 0, sizeof(w));
  w.n = 1;
  w.timeout_ns = timeout_ns;
  w.status = status_d;
  w.flag[0] = flags;
  w.val[0] = 1;
  const auto t0 = std::chrono::steady_clock::now();
  CMX_WT(launch_wait(w, stream));
  CMX_WT(cudaStreamSynchronize(stream));
  const double ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  CMX_EXPECT(status_h[0] == kStatusWaitTimeout, "wait kernel: status %llu, expected a timeout", status_h[0]);
  CMX_EXPECT(status_h[1] == reinterpret_cast<unsigned long long>(flags) && status_h[2] == 1 && status_h[3] == 0,
             "wait kernel: recorded flag 0x%llx wanted %llu saw %llu", status_h[1], status_h[2], status_h[3]);
  CMX_EXPECT(ms >= 0.9 * timeout_ms, "wait kernel gave up after %.1f ms, before its %u ms limit", ms, timeout_ms);

  // 2. the context is still usable: the same wait completes once the flag is set
  std::memset(status_h, 0, 64);
  CMX_WT(cudaMemcpyAsync(flags, &one, sizeof(one), cudaMemcpyHostToDevice, stream));
  CMX_WT(launch_wait(w, stream));
  CMX_WT(cudaStreamSynchronize(stream));
  CMX_EXPECT(status_h[0] == kStatusOk, "wait kernel on a set flag: status %llu", status_h[0]);

  // 3. a pull whose "ready" flag stays unset copies nothing and stores no completion
  auto batch = std::make_unique<PullBatch>();  // ~25 KB: off the stack
  auto make_pull = [&](PullBatch& b) {
    b = PullBatch{};
    b.n = 1;
    b.total_chunks = 1;
    b.counters = counters;
    b.status = status_d;
    b.timeout_ns = timeout_ns;
    PullDesc& d = b.d[0];
    d.src = src;
    d.dst = dst;
    for (int i = 0; i < kMaxPullDims; ++i) d.div[i] = FastDiv(1);
    d.div[kMaxPullDims - 1] = FastDiv(static_cast<std::uint32_t>(kBytes / 16));
    d.sst[kMaxPullDims - 1] = 16;
    d.dstr[kMaxPullDims - 1] = 16;
    d.ndim = 1;
    d.unit = 16;
    d.units = static_cast<std::uint32_t>(kBytes / 16);
    d.nchunks = 1;
    d.msg_chunks = 1;
    d.counter_idx = 0;
    d.done = flags + 2;
    d.done_val = 1;
    d.ready = flags + 1;
    d.ready_val = 1;
  };
  std::memset(status_h, 0, 64);
  make_pull(*batch);
  CMX_WT(launch_pull(*batch, 1, 256, stream));
  std::vector<unsigned char> got(kBytes);
  std::uint64_t done = 0;
  std::uint32_t counter = 0;
  CMX_WT(cudaMemcpyAsync(got.data(), dst, kBytes, cudaMemcpyDeviceToHost, stream));
  CMX_WT(cudaMemcpyAsync(&done, flags + 2, sizeof(done), cudaMemcpyDeviceToHost, stream));
  CMX_WT(cudaMemcpyAsync(&counter, counters, sizeof(counter), cudaMemcpyDeviceToHost, stream));
  CMX_WT(cudaStreamSynchronize(stream));
  CMX_EXPECT(status_h[0] == kStatusWaitTimeout && status_h[1] == reinterpret_cast<unsigned long long>(flags + 1),
             "pull ready wait: status %llu flag 0x%llx", status_h[0], status_h[1]);
  bool untouched = true;
  for (unsigned char b : got) untouched = untouched && b == 0;
  CMX_EXPECT(untouched, "pull ready wait: the destination was written after the wait gave up");
  CMX_EXPECT(done == 0, "pull ready wait: the completion flag was stored after the wait gave up");
  CMX_EXPECT(counter == 0, "pull ready wait: the message counter was left at 0x%x", counter);

  // 4. the same pull after the flag is set: the copy lands
  std::memset(status_h, 0, 64);
  CMX_WT(cudaMemcpyAsync(flags + 1, &one, sizeof(one), cudaMemcpyHostToDevice, stream));
  CMX_WT(launch_pull(*batch, 1, 256, stream));
  CMX_WT(cudaMemcpyAsync(got.data(), dst, kBytes, cudaMemcpyDeviceToHost, stream));
  CMX_WT(cudaMemcpyAsync(&done, flags + 2, sizeof(done), cudaMemcpyDeviceToHost, stream));
  CMX_WT(cudaStreamSynchronize(stream));
  CMX_EXPECT(status_h[0] == kStatusOk, "pull after the flag was set: status %llu", status_h[0]);
  bool copied = true;
  for (unsigned char b : got) copied = copied && b == 0x5a;
  CMX_EXPECT(copied, "pull after the flag was set: the destination does not hold the source");
  CMX_EXPECT(done == 1, "pull after the flag was set: completion flag %llu", static_cast<unsigned long long>(done));
#undef CMX_EXPECT
#undef CMX_WT
  cleanup();
  return fail(err, err_len, 0, "ok");
}
