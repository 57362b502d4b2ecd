// Tagged p2p data movement on sm_100a.
//
// pull_kernel: one launch moves a batch of matched messages. Each descriptor
// is a strided copy from the sender's buffer (mapped into this GPU through
// CUDA IPC, so the loads cross NVLink; or local for self-sends) into the
// receiver's buffer, both with arbitrary strides: the halo face/edge/corner
// gather on the sender side and the ghost-region scatter on the receiver side
// happen inside this one copy, with no pack/unpack buffers. The reference
// moves bytes inside UCX's cuda_ipc transport after `.contiguous()` copies and
// a host stream sync (reference: src/process_group_ucx.cpp:581-591, :490).
//
// Work split: each descriptor is cut into chunks of kChunkUnits units; CTAs
// stride over the global chunk list. The warp that finishes the last slice of
// a message stores the message's completion flag with release semantics at
// system scope (the sender polls it from its own stream), after which it
// zeroes the message's counter so the scratch is clean for the next launch on
// that stream.

#include <cstddef>

#include "cuda_common.hpp"
#include "device_utils.cuh"

namespace commux {
namespace cuda {

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// Byte offsets of unit u in the source and destination (dims outermost
// first, divisors in d.div, sizes of unused outer dims 1). S is the stride
// type: 32-bit when every stride of the descriptor fits (d.wide == 0), which
// keeps the unrolled copy loop inside 64 registers; 64-bit otherwise.
template <typename S>
__device__ __forceinline__ void unit_offsets(const PullDesc& d, std::uint32_t u, std::int64_t& so,
                                             std::int64_t& dof) {
  so = 0;
  dof = 0;
  std::uint32_t rem = u;
#pragma unroll
  for (int i = kMaxPullDims - 1; i >= 1; --i) {
    const std::uint32_t q = d.div[i].div(rem);
    const std::uint32_t r = rem - q * d.div[i].d;
    so += static_cast<std::int64_t>(r) * static_cast<S>(d.sst[i]);
    dof += static_cast<std::int64_t>(r) * static_cast<S>(d.dstr[i]);
    rem = q;
  }
  so += static_cast<std::int64_t>(rem) * static_cast<S>(d.sst[0]);
  dof += static_cast<std::int64_t>(rem) * static_cast<S>(d.dstr[0]);
}

// Bounds-check build: true when the `bytes` bytes at byte offsets `so`
// (source) and `dof` (destination) lie inside the descriptor's declared
// limits; otherwise records the first violation (source address, offsets) in
// the status word and the caller skips the unit. Always true in the
// production build.
__device__ __forceinline__ bool unit_ok(const PullDesc& d, std::int64_t so, std::int64_t dof,
                                        std::int64_t bytes, unsigned long long* status) {
#if defined(COMMUX_DEVICE_CHECKS)
  const bool s_ok = (d.src_lo == 0 && d.src_hi == 0) || (so >= d.src_lo && so + bytes <= d.src_hi);
  const bool d_ok = (d.dst_lo == 0 && d.dst_hi == 0) || (dof >= d.dst_lo && dof + bytes <= d.dst_hi);
  if (s_ok && d_ok) return true;
  report_status(status, kStatusBadDescriptor, reinterpret_cast<unsigned long long>(d.src),
                static_cast<unsigned long long>(so), static_cast<unsigned long long>(dof));
  return false;
#else
  (void)d;
  (void)so;
  (void)dof;
  (void)bytes;
  (void)status;
  return true;
#endif
}

// One warp copies units [u0, u1): lane l takes u0 + l, u0 + l + 32, ...,
// kUnroll loads in flight before the stores. A unit is (row, column) of the
// innermost dim; a lane re-derives the row's offsets over the outer dims only
// when its row changes, so most units cost one division.
template <int U>
__device__ __forceinline__ void copy_units(const PullDesc& d, std::uint32_t u0, std::uint32_t u1,
                                           unsigned long long* status) {
  using V = typename VecT<U>::T;
  constexpr std::uint32_t step = 32;
  constexpr int in = kMaxPullDims - 1;
  const char* __restrict__ src = d.src;
  char* __restrict__ dst = d.dst;
  const std::int32_t css = static_cast<std::int32_t>(d.sst[in]);
  const std::int32_t cds = static_cast<std::int32_t>(d.dstr[in]);
  const FastDiv rdiv = d.div[in];  // in registers: the descriptor may live in global memory
  std::uint32_t crow = 0xffffffffu;
  std::int64_t rso = 0, rdo = 0;
  for (std::uint32_t base = u0 + (threadIdx.x & 31u); base < u1; base += step * kUnroll) {
    V v[kUnroll];
    std::int64_t dofs[kUnroll];
    std::uint32_t skip = 0;
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const std::uint32_t u = base + k * step;
      if (u < u1) {
        const std::uint32_t row = rdiv.div(u);
        const std::uint32_t col = u - row * rdiv.d;
        if (row != crow) {
          crow = row;
          std::uint32_t rem = row;
          rso = 0;
          rdo = 0;
#pragma unroll
          for (int i = in - 1; i >= 1; --i) {
            const std::uint32_t q = d.div[i].div(rem);
            const std::uint32_t r = rem - q * d.div[i].d;
            rso += static_cast<std::int64_t>(r) * static_cast<std::int32_t>(d.sst[i]);
            rdo += static_cast<std::int64_t>(r) * static_cast<std::int32_t>(d.dstr[i]);
            rem = q;
          }
          rso += static_cast<std::int64_t>(rem) * static_cast<std::int32_t>(d.sst[0]);
          rdo += static_cast<std::int64_t>(rem) * static_cast<std::int32_t>(d.dstr[0]);
        }
        dofs[k] = rdo + static_cast<std::int64_t>(col) * cds;
        const std::int64_t so = rso + static_cast<std::int64_t>(col) * css;
        if (unit_ok(d, so, dofs[k], U, status))
          v[k] = *reinterpret_cast<const V*>(src + so);
        else
          skip |= 1u << k;  // bounds-check build only: no load, no store
      }
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const std::uint32_t u = base + k * step;
      if (u < u1 && (skip & (1u << k)) == 0u) *reinterpret_cast<V*>(dst + dofs[k]) = v[k];
    }
  }
}

template <int U>
__device__ __forceinline__ void copy_one(const char* s, char* d) {
  using V = typename VecT<U>::T;
  *reinterpret_cast<V*>(d) = *reinterpret_cast<const V*>(s);
}

// Descriptors with a stride of 2 GiB or more: one unit at a time, 64-bit
// strides (layouts this wide are rare; kept out of line so the common loop
// keeps its registers).
__device__ __noinline__ void copy_units_wide(const PullDesc& d, std::uint32_t u0, std::uint32_t u1,
                                             unsigned long long* status) {
  for (std::uint32_t u = u0 + (threadIdx.x & 31u); u < u1; u += 32) {
    std::int64_t so, dof;
    unit_offsets<std::int64_t>(d, u, so, dof);
    if (!unit_ok(d, so, dof, d.unit, status)) continue;
    switch (d.unit) {
      case 16:
        copy_one<16>(d.src + so, d.dst + dof);
        break;
      case 8:
        copy_one<8>(d.src + so, d.dst + dof);
        break;
      case 4:
        copy_one<4>(d.src + so, d.dst + dof);
        break;
      case 2:
        copy_one<2>(d.src + so, d.dst + dof);
        break;
      default:
        copy_one<1>(d.src + so, d.dst + dof);
        break;
    }
  }
}

// Bounded wait for a persistent plan's ready flag (thread 0 of the CTA).
// Gives up after the timeout, or at once if another wait already failed.
__device__ __forceinline__ bool wait_ready(const std::uint64_t* ready, std::uint64_t want,
                                          unsigned long long* status, std::uint64_t timeout_ns) {
  if (ld_acquire_sys(ready) >= want) return true;
  const std::uint64_t t0 = globaltimer_ns();
  std::uint32_t spins = 0;
  while (ld_acquire_sys(ready) < want) {
    if ((++spins & 63u) == 0u) {
      if (*reinterpret_cast<volatile unsigned long long*>(status) != 0ull) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_status(status, kStatusWaitTimeout, reinterpret_cast<unsigned long long>(ready), want,
                      ld_acquire_sys(ready));
        return false;
      }
    }
    __nanosleep(64);
  }
  return true;
}

// The batch a launch works from: its kernel parameter block (pull_kernel;
// read through the constant cache), or a copy in shared memory that each CTA
// stages from device memory at its start (pull_kernel_staged, persistent
// plans). The epoch of a plan's launch comes from device memory.
struct InlineSrc {
  const PullBatch& b;
  __device__ std::uint32_t n() const { return b.n; }
  __device__ std::uint32_t total() const { return b.total_chunks; }
  __device__ const PullDesc& desc(std::uint32_t i) const { return b.d[i]; }
  __device__ std::uint32_t* counters() const { return b.counters; }
  __device__ unsigned long long* status() const { return b.status; }
  __device__ std::uint64_t timeout_ns() const { return b.timeout_ns; }
  __device__ std::uint64_t epoch() const { return b.epoch ? *b.epoch : 0; }
  __device__ unsigned long long* cta_trace() const { return b.cta_trace; }
  __device__ void trace_start() const {
    if (b.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) b.trace[0] = globaltimer_ns();
  }
  __device__ void trace_end() const {
    if (b.trace == nullptr) return;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(b.trace_count, 1u) == gridDim.x - 1) {  // the last CTA of the launch
        b.trace[1] = globaltimer_ns();
        *b.trace_count = 0u;
      }
    }
  }
  // The data these signals announce was written by earlier work on this
  // stream; the release store at system scope orders it before the flag for
  // a peer that acquires the flag, so no separate fence precedes it.
  __device__ void entry_signals(std::uint64_t epoch) const {
    if (blockIdx.x == 0 && threadIdx.x < b.nsig) st_release_sys(b.sig[threadIdx.x], epoch);
  }
  // The last CTA to finish waits for the receivers' "consumed" flags and
  // advances the epoch: every other CTA has read the epoch already (at its
  // start) and has finished, so the next start sees the new value.
  __device__ void finish(std::uint64_t epoch) const {
    if (b.bump == nullptr) return;
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      last = atomicAdd(b.cta_done, 1u) == gridDim.x - 1 ? 1 : 0;
    }
    __syncthreads();
    if (!last) return;
    for (std::uint32_t i = threadIdx.x; i < b.nfin; i += blockDim.x) {
      const std::uint64_t t0 = globaltimer_ns();
      std::uint32_t spins = 0;
      while (ld_acquire_sys(b.fin[i]) < epoch) {
        if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > b.timeout_ns) {
          report_status(b.status, kStatusWaitTimeout, reinterpret_cast<unsigned long long>(b.fin[i]), epoch,
                        ld_acquire_sys(b.fin[i]));
          break;
        }
        __nanosleep(128);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      *b.cta_done = 0u;
      *b.bump = epoch + 1;
    }
  }
};

// Descriptor owning global chunk c and the chunk's index inside it. The
// descriptors are sorted by chunk0 (the first has chunk0 == 0); the binary
// search finds the last one whose chunk0 <= c. An interleaved group (ilv > 1:
// descriptors [ilv_first, ilv_first + ilv), all with the same chunk0 and
// chunk count) takes its chunks round robin, chunk k of each member in turn,
// so row k of every member is copied at about the same time.
template <class S>
__device__ __forceinline__ std::uint32_t find_desc(const S& s, std::uint32_t c, std::uint32_t& local) {
  std::uint32_t lo = 0, hi = s.n();  // answer in [lo, hi)
  while (hi - lo > 1) {
    const std::uint32_t mid = (lo + hi) >> 1;
    if (s.desc(mid).chunk0 <= c)
      lo = mid;
    else
      hi = mid;
  }
  const PullDesc& h = s.desc(lo);
  const std::uint32_t off = c - h.chunk0;
  if (h.ilv > 1) {
    local = off / h.ilv;
    return h.ilv_first + off % h.ilv;
  }
  local = off;
  return lo;
}

// Each chunk is split into one contiguous slice per warp; every warp counts
// its own slice into the message's counter (target: chunks x warps), so the
// CTA needs no barrier except where a plan's ready flag must be awaited.
// Messages without a completion flag (copies ordered by the stream alone)
// skip the counting and its fence. A descriptor of zero units is a pure
// signal: its message's flag is stored once the launch reaches it.
template <int U, class S>
__device__ __forceinline__ void pull_body(const S& s) {
  __shared__ int skip;
  constexpr std::uint32_t kWarps = kThreads / 32;
  constexpr std::uint32_t kFailBit = 0x80000000u;
  const std::uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const std::uint64_t epoch = s.epoch();
  s.trace_start();
  // COMMUX_PLAN_TRACE=2 tallies of this CTA (thread 0), in shared memory so
  // they hold no registers across the copy loop
  __shared__ unsigned long long t_begin, waited, flagged;
  if (threadIdx.x == 0) {
    t_begin = s.cta_trace() != nullptr ? globaltimer_ns() : 0;
    waited = 0;
    flagged = 0;
  }
  s.entry_signals(epoch);
  for (std::uint32_t c = blockIdx.x; c < s.total(); c += gridDim.x) {
    std::uint32_t local = 0;
    const PullDesc& d = s.desc(find_desc(s, c, local));
    const std::uint32_t u0 = local * kChunkUnits;
    bool failed = false;
    if (d.ready != nullptr) {  // persistent plan: wait for the sender's data
      if (threadIdx.x == 0) {
        const bool tr = s.cta_trace() != nullptr;
        const std::uint64_t w0 = tr ? globaltimer_ns() : 0;
        skip = wait_ready(d.ready, epoch ? epoch : d.ready_val, s.status(), s.timeout_ns()) ? 0 : 1;
        if (tr) {
          waited += globaltimer_ns() - w0;
          ++flagged;
        }
      }
      __syncthreads();
      failed = skip != 0;
      __syncthreads();  // every thread read `skip` before it is rewritten
    }
    // a failed wait copies nothing but still counts, so the scratch counter
    // returns to zero; the message's completion flag is then not stored
    const std::uint32_t end = failed ? u0 : min(u0 + kChunkUnits, d.units);
    const std::uint32_t per = (end - u0 + kWarps - 1) / kWarps;
    const std::uint32_t wlo = min(end, u0 + warp * per), whi = min(end, wlo + per);
    if constexpr (U == 0)
      copy_units_wide(d, wlo, whi, s.status());
    else
      copy_units<U>(d, wlo, whi, s.status());
    std::uint64_t* done = d.done;
    if (done == nullptr) continue;
    __syncwarp();  // every load of this warp's slice has returned
    if (lane == 0) {
      std::uint32_t* counter = s.counters() + d.counter_idx;
      fence_acq_rel_gpu();  // with the relaxed add below: a release of the slice
      if (failed) atomicOr(counter, kFailBit);
      std::uint32_t prev = atomicAdd(counter, 1u);
      if ((prev & ~kFailBit) + 1 == d.msg_chunks * kWarps) {
        const bool any_failed = failed || (prev & kFailBit) != 0u;
        *counter = 0u;
        if (!any_failed) {
          // acquire the other warps' slices (their release fences and adds
          // are GPU-local), then publish all of them to the peer: the store's
          // release at system scope is cumulative over what this thread has
          // acquired
          fence_acq_rel_gpu();
          st_release_sys(done, epoch ? epoch : d.done_val);
        }
      }
    }
  }
  s.trace_end();
  if (s.cta_trace() != nullptr && threadIdx.x == 0) {
    unsigned long long* r = s.cta_trace() + 4ull * blockIdx.x;
    r[0] = t_begin;
    r[1] = globaltimer_ns();
    r[2] = waited;
    r[3] = flagged;
  }
  s.finish(epoch);
}

// One instantiation per unit size U (U == 0: the 64-bit-stride walk for wide
// layouts): a single kernel holding every unit's copy loop needs more than
// 80 registers, one loop alone fits the 64 that four CTAs per SM allow.
template <int U>
__global__ void __launch_bounds__(kThreads, 4) pull_kernel(const __grid_constant__ PullBatch b) {
  pull_body<U>(InlineSrc{b});
}

// The same copy for a batch in device memory (persistent plans): each CTA
// first copies the batch header and its n descriptors (at most about 28 KB)
// into shared memory, then works only from there. A plan's descriptor table
// (26 descriptors for a halo, up to 128) does not fit the per-SM constant
// cache, so from the parameter block every chunk's descriptor search and
// field reads were a chain of cache misses: CTAs of the 1-GPU halo spent
// about 7 us per 16 KB chunk.
template <int U>
__global__ void __launch_bounds__(kThreads, 4) pull_kernel_staged(const PullBatch* __restrict__ g) {
  extern __shared__ __align__(16) unsigned char staged[];
  const std::size_t bytes = offsetof(PullBatch, d) + static_cast<std::size_t>(g->n) * sizeof(PullDesc);
  const uint2* from = reinterpret_cast<const uint2*>(g);
  uint2* to = reinterpret_cast<uint2*>(staged);
  for (std::size_t k = threadIdx.x; k < bytes / sizeof(uint2); k += blockDim.x) to[k] = from[k];
  __syncthreads();
  pull_body<U>(InlineSrc{*reinterpret_cast<const PullBatch*>(staged)});
}
static_assert(offsetof(PullBatch, d) % sizeof(uint2) == 0 && sizeof(PullDesc) % sizeof(uint2) == 0,
              "the batch is staged in 8-byte words");

// One warp: lane i waits until *flag[i] >= val[i], giving up after the
// timeout (status word set, kernel returns; never traps).
__global__ void wait_kernel(const __grid_constant__ WaitBatch b) {
  const std::uint32_t i = threadIdx.x;
  if (i >= b.n) return;
  const std::uint64_t want = b.epoch ? *b.epoch : b.val[i];
  const std::uint64_t t0 = globaltimer_ns();
  std::uint32_t spins = 0;
  while (ld_acquire_sys(b.flag[i]) < want) {
    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > b.timeout_ns) {
      report_status(b.status, kStatusWaitTimeout, reinterpret_cast<unsigned long long>(b.flag[i]),
                    want, ld_acquire_sys(b.flag[i]));
      return;
    }
    __nanosleep(128);
  }
}

}  // namespace

namespace {

cudaError_t launch_class(int cls, const PullBatch& b, int max_ctas, cudaStream_t s) {
  const int grid =
      static_cast<int>(b.total_chunks < static_cast<std::uint32_t>(max_ctas) ? b.total_chunks : max_ctas);
  switch (cls) {
    case 16:
      pull_kernel<16><<<grid, kThreads, 0, s>>>(b);
      break;
    case 8:
      pull_kernel<8><<<grid, kThreads, 0, s>>>(b);
      break;
    case 4:
      pull_kernel<4><<<grid, kThreads, 0, s>>>(b);
      break;
    case 2:
      pull_kernel<2><<<grid, kThreads, 0, s>>>(b);
      break;
    case 1:
      pull_kernel<1><<<grid, kThreads, 0, s>>>(b);
      break;
    default:
      pull_kernel<0><<<grid, kThreads, 0, s>>>(b);
      break;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pull_staged(const PullBatch& host, const PullBatch* dev, int max_ctas, cudaStream_t s) {
  if (host.n == 0 || host.total_chunks == 0) return cudaSuccess;
  const int cls = pull_unit_class(host.d[0]);
  for (std::uint32_t i = 1; i < host.n; ++i)
    if (pull_unit_class(host.d[i]) != cls) return cudaErrorInvalidValue;
  const int grid =
      static_cast<int>(host.total_chunks < static_cast<std::uint32_t>(max_ctas) ? host.total_chunks : max_ctas);
  const std::size_t smem = offsetof(PullBatch, d) + static_cast<std::size_t>(host.n) * sizeof(PullDesc);
  switch (cls) {
    case 16:
      pull_kernel_staged<16><<<grid, kThreads, smem, s>>>(dev);
      break;
    case 8:
      pull_kernel_staged<8><<<grid, kThreads, smem, s>>>(dev);
      break;
    case 4:
      pull_kernel_staged<4><<<grid, kThreads, smem, s>>>(dev);
      break;
    case 2:
      pull_kernel_staged<2><<<grid, kThreads, smem, s>>>(dev);
      break;
    case 1:
      pull_kernel_staged<1><<<grid, kThreads, smem, s>>>(dev);
      break;
    default:
      pull_kernel_staged<0><<<grid, kThreads, smem, s>>>(dev);
      break;
  }
  return cudaGetLastError();
}

// A batch whose descriptors share one unit class is one launch; a mixed batch
// becomes one launch per class, in order on the stream (completion counters
// count warps across all of them, so a message may span launches).
cudaError_t launch_pull(const PullBatch& b, int max_ctas, int threads, cudaStream_t s, int* launches) {
  (void)threads;
  if (b.n == 0 || b.total_chunks == 0) return cudaSuccess;
  const int first = pull_unit_class(b.d[0]);
  bool same = true;
  for (std::uint32_t i = 1; same && i < b.n; ++i) same = pull_unit_class(b.d[i]) == first;
  if (same) {
    if (launches != nullptr) ++*launches;
    return launch_class(first, b, max_ctas, s);
  }
  static thread_local PullBatch sub;  // 25 KB: off the stack, reused
  sub.counters = b.counters;
  sub.status = b.status;
  sub.timeout_ns = b.timeout_ns;
  sub.epoch = b.epoch;
  sub.trace = b.trace;
  sub.trace_count = b.trace_count;
  sub.cta_trace = nullptr;
  sub.nsig = 0;  // entry signals go with the first class launched
  sub.bump = nullptr;  // the end-of-start wait goes with the last one
  int last_cls = -1;
  for (int cls : {16, 8, 4, 2, 1, 0})
    for (std::uint32_t i = 0; i < b.n && last_cls != cls; ++i)
      if (pull_unit_class(b.d[i]) == cls && b.d[i].nchunks > 0) last_cls = cls;
  bool first_launch = true;
  for (int cls : {16, 8, 4, 2, 1, 0}) {
    sub.n = 0;
    sub.total_chunks = 0;
    for (std::uint32_t i = 0; i < b.n; ++i) {
      if (pull_unit_class(b.d[i]) != cls) continue;
      PullDesc x = b.d[i];
      x.chunk0 = sub.total_chunks;
      sub.total_chunks += x.nchunks;
      sub.d[sub.n++] = x;
    }
    if (sub.n == 0 || sub.total_chunks == 0) continue;
    if (first_launch) {
      sub.nsig = b.nsig;
      for (std::uint32_t k = 0; k < b.nsig; ++k) sub.sig[k] = b.sig[k];
      first_launch = false;
    } else {
      sub.nsig = 0;
    }
    if (cls == last_cls) {
      sub.bump = b.bump;
      sub.cta_done = b.cta_done;
      sub.nfin = b.nfin;
      for (std::uint32_t k = 0; k < b.nfin; ++k) sub.fin[k] = b.fin[k];
    }
    if (launches != nullptr) ++*launches;
    cudaError_t e = launch_class(cls, sub, max_ctas, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Loads every build of the pull kernel into the current context now, instead
// of at its first launch (CUDA's default lazy loading; a load may allocate
// device memory).
cudaError_t preload_pull_kernels() {
  cudaFuncAttributes a;
  for (cudaError_t e : {cudaFuncGetAttributes(&a, pull_kernel<16>), cudaFuncGetAttributes(&a, pull_kernel<8>),
                        cudaFuncGetAttributes(&a, pull_kernel<4>), cudaFuncGetAttributes(&a, pull_kernel<2>),
                        cudaFuncGetAttributes(&a, pull_kernel<1>), cudaFuncGetAttributes(&a, pull_kernel<0>)})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

cudaError_t launch_wait(const WaitBatch& b, cudaStream_t s) {
  if (b.n == 0) return cudaSuccess;
  wait_kernel<<<1, kMaxWaitFlags, 0, s>>>(b);
  return cudaGetLastError();
}

}  // namespace cuda
}  // namespace commux
