#pragma once

// Structures shared by the host side of the CUDA transport and its sm_100a
// kernels.

#include <cuda_runtime.h>

#include <cstdint>

namespace commux {
namespace cuda {

constexpr int kMaxPullDims = 4;      // dims of a pull descriptor after merging
constexpr int kMaxBatch = 128;       // descriptors per pull launch (by value)
constexpr int kMaxWaitFlags = 128;   // flags per wait launch (one thread each)
constexpr std::uint32_t kCounterSlots = 1024;  // per-stream message counters
constexpr std::uint32_t kChunkUnits = 1024;  // units per CTA work item (16 KB of 16 B units)
constexpr int kMaxEntrySignals = 64;  // flags a pull launch stores at entry

// 32-bit division by an invariant divisor through a multiply-high and a shift
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, round-up variant). Valid for n < 2^31.
struct FastDiv {
  std::uint32_t d = 1, mul = 0, shr = 0;
  FastDiv() = default;
  explicit FastDiv(std::uint32_t div) : d(div) {
    if (div <= 1) {
      mul = 0;
      shr = 0;
      return;
    }
    std::uint32_t l = 0;
    while ((1ull << l) < div) ++l;  // l = ceil(log2 div)
    std::uint64_t p = 31 + l;
    mul = static_cast<std::uint32_t>(((1ull << p) + div - 1) / div);
    shr = static_cast<std::uint32_t>(p - 32);
  }
#if defined(__CUDACC__)
  __device__ __forceinline__ std::uint32_t div(std::uint32_t n) const {
    return d == 1 ? n : (__umulhi(n, mul) >> shr);
  }
#endif
};

// One strided copy: units of `unit` bytes, dims outermost first.
struct PullDesc {
  const char* src;
  char* dst;
  std::int64_t sst[kMaxPullDims];   // src stride per dim, bytes
  std::int64_t dstr[kMaxPullDims];  // dst stride per dim, bytes
  FastDiv div[kMaxPullDims];        // divisors = sizes per dim
  std::uint32_t ndim;
  std::uint32_t unit;               // 16, 8, 4, 2 or 1 bytes
  std::uint32_t units;              // total units (< 2^31)
  std::uint32_t chunk0;             // first chunk index of this descriptor
  std::uint32_t nchunks;            // chunks of this descriptor
  std::uint32_t msg_chunks;         // chunks of its whole message
  std::uint32_t counter_idx;        // per-message completion counter (scratch)
  std::uint32_t wide;               // 1: some |stride| >= 2^31 bytes (64-bit walk)
  std::uint64_t* done;              // flag to set once copied (may be remote)
  std::uint64_t done_val;
  // persistent plans: the copy may start once *ready >= ready_val (a flag in
  // this GPU's memory that the sender's stream sets); nullptr: no wait
  const std::uint64_t* ready;
  std::uint64_t ready_val;
  // interleaved group: ilv > 1 descriptors [ilv_first, ilv_first + ilv) with
  // equal chunk0 and nchunks take their chunks round robin (see find_desc);
  // ilv <= 1: a descriptor of its own
  std::uint32_t ilv;
  std::uint32_t ilv_first;
#if defined(COMMUX_DEVICE_CHECKS)
  // bounds-check build: the byte offsets from src / dst that the copy may
  // touch, [lo, hi). A unit outside them is skipped and reported in the
  // status word (kStatusBadDescriptor) instead of being accessed. lo == hi
  // == 0 (a value-initialised descriptor): no limit declared.
  std::int64_t src_lo, src_hi, dst_lo, dst_hi;
#endif
};

struct PullBatch {
  std::uint32_t n;
  std::uint32_t total_chunks;
  std::uint32_t* counters;          // per-stream scratch, zero between launches
  unsigned long long* status;       // host-mapped status word (4 x u64)
  std::uint64_t timeout_ns;         // bound of the ready-flag waits
  // persistent plans: the ready/done value of every flagged descriptor is
  // *epoch (device memory, advanced once per start by the plan's last launch),
  // so a plan's launches never change and replay as one CUDA graph
  const std::uint64_t* epoch;
  // COMMUX_PLAN_TRACE: [0] = start of CTA 0, [1] = end of the last CTA
  // (%globaltimer, ns; host-mapped); trace_count (device memory) finds the
  // last CTA. nullptr otherwise
  unsigned long long* trace;
  unsigned int* trace_count;
  // COMMUX_PLAN_TRACE=2: per CTA, 4 words (host-mapped): first and last
  // %globaltimer stamp of the CTA, ns its thread 0 spent waiting on ready
  // flags, chunks it copied that had a ready flag. nullptr otherwise
  unsigned long long* cta_trace;
  // flags stored (release, system scope) by the first CTA at kernel entry,
  // value *epoch: the "data ready" signals of a plan whose sends need no
  // packing ride on its pull launch instead of a launch of their own
  std::uint32_t nsig;
  std::uint64_t* sig[kMaxEntrySignals];
  // persistent plans, last launch of a start: the CTA that finishes last
  // (counted in *cta_done, device memory, zero between launches) waits,
  // bounded, until every fin[i] reaches *epoch -- the receivers' "consumed"
  // flags of this rank's sends -- and then advances *bump (the epoch).
  // bump == nullptr: nothing of the kind.
  std::uint64_t* bump;
  unsigned int* cta_done;
  std::uint32_t nfin;
  const std::uint64_t* fin[kMaxWaitFlags];
  PullDesc d[kMaxBatch];
};
// passed by value as a __grid_constant__ kernel parameter (limit 32764 bytes)
static_assert(sizeof(PullBatch) <= 32764, "PullBatch exceeds the kernel parameter space");

// Flags a wait kernel polls (all in this GPU's own memory, written remotely).
struct WaitBatch {
  std::uint32_t n;
  std::uint64_t timeout_ns;
  unsigned long long* status;
  const std::uint64_t* epoch;  // non-null: every val is *epoch
  const std::uint64_t* flag[kMaxWaitFlags];
  std::uint64_t val[kMaxWaitFlags];
};

// Device error codes written to the status word.
enum : unsigned long long {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,     // a flag wait gave up
  kStatusBadDescriptor = 2,   // bounds check failed (COMMUX_DEVICE_CHECKS)
  kStatusCollTimeout = 3,     // collective barrier gave up
};

// Launchers (p2p_kernels.cu).
// Launches the pull kernel(s) for a batch; adds the number of launches to
// *launches when given (one per unit class present in the batch).
cudaError_t launch_pull(const PullBatch& b, int max_ctas, int threads, cudaStream_t s,
                        int* launches = nullptr);
// Unit class of a descriptor: one kernel instantiation per class (16, 8, 4,
// 2, 1 byte units; 0 = wide strides).
inline int pull_unit_class(const PullDesc& d) { return d.wide ? 0 : static_cast<int>(d.unit); }
cudaError_t launch_wait(const WaitBatch& b, cudaStream_t s);
// Launches the pull kernel on a batch already in device memory (`dev`, a
// copy of `host`, whose descriptors share one unit class); each CTA stages
// the batch into shared memory first.
cudaError_t launch_pull_staged(const PullBatch& host, const PullBatch* dev, int max_ctas, cudaStream_t s);

// Loads every pull-kernel build into the current context (see p2p_kernels.cu).
cudaError_t preload_pull_kernels();

}  // namespace cuda
}  // namespace commux
