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
// stride over the global chunk list. The CTA that finishes the last chunk of
// a descriptor stores the descriptor's completion flag with release
// semantics at system scope (the sender polls it from its own stream), after
// which it zeroes the descriptor's counter so the scratch is clean for the
// next launch on that stream.

#include "cuda_common.hpp"
#include "device_utils.cuh"

namespace commux {
namespace cuda {

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ void unit_offsets(const PullDesc& d, std::uint32_t u, std::int64_t& so,
                                             std::int64_t& dof) {
  if (d.ndim == 1) {
    so = static_cast<std::int64_t>(u) * d.sst[kMaxPullDims - 1];
    dof = static_cast<std::int64_t>(u) * d.dstr[kMaxPullDims - 1];
    return;
  }
  so = 0;
  dof = 0;
  std::uint32_t rem = u;
#pragma unroll
  for (int i = kMaxPullDims - 1; i >= 1; --i) {
    std::uint32_t q = d.div[i].div(rem);
    std::uint32_t r = rem - q * d.div[i].d;
    so += static_cast<std::int64_t>(r) * d.sst[i];
    dof += static_cast<std::int64_t>(r) * d.dstr[i];
    rem = q;
  }
  so += static_cast<std::int64_t>(rem) * d.sst[0];
  dof += static_cast<std::int64_t>(rem) * d.dstr[0];
}

// One warp copies units [u0, u1): lane l takes u0 + l, u0 + l + 32, ...,
// kUnroll loads in flight before the stores.
template <int U>
__device__ __forceinline__ void copy_units(const PullDesc& d, std::uint32_t u0, std::uint32_t u1) {
  using V = typename VecT<U>::T;
  constexpr std::uint32_t step = 32;
  for (std::uint32_t base = u0 + (threadIdx.x & 31u); base < u1; base += step * kUnroll) {
    V v[kUnroll];
    std::int64_t dofs[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      std::uint32_t u = base + k * step;
      if (u < u1) {
        std::int64_t so;
        unit_offsets(d, u, so, dofs[k]);
        v[k] = *reinterpret_cast<const V*>(d.src + so);
      }
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      std::uint32_t u = base + k * step;
      if (u < u1) *reinterpret_cast<V*>(d.dst + dofs[k]) = v[k];
    }
  }
}

// Bounded wait for a persistent plan's ready flag (thread 0 of the CTA).
// Gives up after the timeout, or at once if another wait already failed.
__device__ __forceinline__ bool wait_ready(const PullDesc& d, const PullBatch& b) {
  if (ld_acquire_sys(d.ready) >= d.ready_val) return true;
  const std::uint64_t t0 = globaltimer_ns();
  std::uint32_t spins = 0;
  while (ld_acquire_sys(d.ready) < d.ready_val) {
    if ((++spins & 63u) == 0u) {
      if (*reinterpret_cast<volatile unsigned long long*>(b.status) != 0ull) return false;
      if (globaltimer_ns() - t0 > b.timeout_ns) {
        report_status(b.status, kStatusWaitTimeout, reinterpret_cast<unsigned long long>(d.ready),
                      d.ready_val, ld_acquire_sys(d.ready));
        return false;
      }
    }
    __nanosleep(64);
  }
  return true;
}

// Each chunk is split into one contiguous slice per warp; every warp counts
// its own slice into the message's counter (target: chunks x warps), so the
// CTA needs no barrier except where a plan's ready flag must be awaited.
__global__ void __launch_bounds__(kThreads, 4) pull_kernel(const __grid_constant__ PullBatch b) {
  __shared__ int skip;
  constexpr std::uint32_t kWarps = kThreads / 32;
  constexpr std::uint32_t kFailBit = 0x80000000u;
  const std::uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  for (std::uint32_t c = blockIdx.x; c < b.total_chunks; c += gridDim.x) {
    std::uint32_t di = 0;
    while (di + 1 < b.n && c >= b.d[di + 1].chunk0) ++di;
    const PullDesc& d = b.d[di];
    const std::uint32_t u0 = (c - d.chunk0) * kChunkUnits;
    bool failed = false;
    if (d.ready != nullptr) {  // persistent plan: wait for the sender's data
      if (threadIdx.x == 0) skip = wait_ready(d, b) ? 0 : 1;
      __syncthreads();
      failed = skip != 0;
      __syncthreads();  // every thread read `skip` before it is rewritten
    }
    // a failed wait copies nothing but still counts, so the scratch counter
    // returns to zero; the message's completion flag is then not stored
    const std::uint32_t end = failed ? u0 : min(u0 + kChunkUnits, d.units);
    const std::uint32_t per = (end - u0 + kWarps - 1) / kWarps;
    const std::uint32_t wlo = min(end, u0 + warp * per), whi = min(end, wlo + per);
    switch (d.unit) {
      case 16:
        copy_units<16>(d, wlo, whi);
        break;
      case 8:
        copy_units<8>(d, wlo, whi);
        break;
      case 4:
        copy_units<4>(d, wlo, whi);
        break;
      case 2:
        copy_units<2>(d, wlo, whi);
        break;
      default:
        copy_units<1>(d, wlo, whi);
        break;
    }
    __syncwarp();  // every load of this warp's slice has returned
    if (lane == 0) {
      __threadfence();
      if (failed) atomicOr(&b.counters[d.counter_idx], kFailBit);
      std::uint32_t prev = atomicAdd(&b.counters[d.counter_idx], 1u);
      if ((prev & ~kFailBit) + 1 == d.msg_chunks * kWarps) {
        const bool any_failed = failed || (prev & kFailBit) != 0u;
        b.counters[d.counter_idx] = 0u;
        if (d.done != nullptr && !any_failed) {
          fence_acq_rel_sys();
          st_release_sys(d.done, d.done_val);
        }
      }
    }
  }
}

// Store each flag with release semantics at system scope (after everything
// the stream did before): "data ready" signals of persistent plans.
__global__ void signal_many_kernel(const __grid_constant__ SignalBatch b) {
  const std::uint32_t i = threadIdx.x;
  if (i >= b.n) return;
  fence_acq_rel_sys();
  st_release_sys(b.flag[i], b.val[i]);
}

// One warp: lane i waits until *flag[i] >= val[i], giving up after the
// timeout (status word set, kernel returns; never traps).
__global__ void wait_kernel(const __grid_constant__ WaitBatch b) {
  const std::uint32_t i = threadIdx.x;
  if (i >= b.n) return;
  const std::uint64_t t0 = globaltimer_ns();
  std::uint32_t spins = 0;
  while (ld_acquire_sys(b.flag[i]) < b.val[i]) {
    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > b.timeout_ns) {
      report_status(b.status, kStatusWaitTimeout, reinterpret_cast<unsigned long long>(b.flag[i]),
                    b.val[i], ld_acquire_sys(b.flag[i]));
      return;
    }
    __nanosleep(128);
  }
}

__global__ void signal_kernel(std::uint64_t* flag, std::uint64_t val) {
  fence_acq_rel_sys();
  st_release_sys(flag, val);
}

}  // namespace

cudaError_t launch_pull(const PullBatch& b, int max_ctas, int threads, cudaStream_t s) {
  if (b.n == 0 || b.total_chunks == 0) return cudaSuccess;
  int grid = static_cast<int>(b.total_chunks < static_cast<std::uint32_t>(max_ctas) ? b.total_chunks : max_ctas);
  (void)threads;
  pull_kernel<<<grid, kThreads, 0, s>>>(b);
  return cudaGetLastError();
}

cudaError_t launch_wait(const WaitBatch& b, cudaStream_t s) {
  if (b.n == 0) return cudaSuccess;
  wait_kernel<<<1, kMaxWaitFlags, 0, s>>>(b);
  return cudaGetLastError();
}

cudaError_t launch_signal_many(const SignalBatch& b, cudaStream_t s) {
  if (b.n == 0) return cudaSuccess;
  signal_many_kernel<<<1, kMaxSignal, 0, s>>>(b);
  return cudaGetLastError();
}

cudaError_t launch_signal(std::uint64_t* flag, std::uint64_t val, cudaStream_t s) {
  signal_kernel<<<1, 1, 0, s>>>(flag, val);
  return cudaGetLastError();
}

}  // namespace cuda
}  // namespace commux
