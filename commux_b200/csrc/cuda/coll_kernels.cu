// Device collectives on sm_100a over symmetric CUDA-IPC workspaces.
//
// Every rank owns one workspace (flags + regions A and B) mapped into every
// peer. All data crosses NVLink as plain 16-byte stores into a peer's
// workspace (posted writes: a CTA never stalls on a remote round trip); every
// reduction then reads local HBM. Synchronisation is per CTA: CTA b of each
// rank exchanges flags only with CTA b of the others, so there is no grid-wide
// barrier and ranks pipeline freely. Flags are monotonically increasing
// sequence numbers (epoch << 20 | chunk), stored with release and polled with
// acquire at system scope; every wait gives up after a timeout, records the
// failure in a host-mapped status word and returns (no trap, no endless spin).
//
// Reuse rules: a call with epoch e only touches half (e & 1) of A and B, and
// every call contains an all-to-all flag round, so a peer has finished call
// e-2 before call e writes into the same half (see coll_args.hpp). Inside a
// call, each chunk has two flag rounds, so chunk c+1 never overwrites what a
// peer still reads from chunk c.
//
// The reduction folds ranks in rank order 0..P-1 with fp32 accumulation for
// bf16/fp16, so all ranks hold bit-identical results that the CPU fold of the
// host backend reproduces exactly. (The reference reduces with ATen ops along
// a binomial tree of whole-tensor messages, reference:
// src/process_group_ucx.cpp:214-232, :734-792.)
//
// Kernels:
//   oneshot  (small allreduce/reduce): push my data into slot[me] of every
//            rank's A, one flag round, fold the P slots locally.
//   twoshot  (large allreduce/reduce/reduce_scatter), chunk by chunk, the
//            phases of a chunk in sequence within each CTA: push segment s of
//            the chunk into slot[me] of rank s's A (reduce-scatter by
//            writes), flag round, rank s folds its segment (its own part read
//            from its input) and pushes it into slot[s] of B on every rank
//            that needs it, flag round, copy out. (A software pipeline over
//            half-size, double-buffered chunks, which folded chunk c-1 while
//            chunk c crossed NVLink, measured 14 % slower at 1 GiB on 2 GPUs:
//            its flag stores still waited for every store to land, and NVLink
//            idled during the flag waits.)
//   gather   (allgather/broadcast at 2 ranks), chunked: push my block into
//            slot[me] of every rank's B (broadcast: the root's block into
//            slot 0), flag round, copy out, flag round.
//   bcast    (broadcast from 3 ranks): scatter from the root + allgather
//            among the ranks, pipelined over double-buffered chunks (see
//            bcast_kernel).
//   chain    (opt-in, COMMUX_CHAIN_RANKS: broadcast and large reduce): the
//            chunks of the message flow along a chain of the ranks, so
//            every link carries the message once (see chain_kernel).
//   barrier  one CTA: a system-scope fence (everything this rank's stream
//            wrote before the barrier, local or into a peer's memory, is
//            visible system-wide), a flag to every rank, a bounded wait for
//            every rank's flag.
//   nvls     (large allreduce of f32/f16/bf16), pipelined over double-
//            buffered chunks by two warp groups (see "warp groups" below):
//            copy my data into my NVLS buffer, flag round, multimem.ld_reduce
//            my segment through the multicast mapping (NVSwitch sums every
//            rank's copy) and multimem.st the result back (the switch writes
//            it into every rank's copy), flag round, copy out. Each rank's NVLink carries
//            about 1x the message each way instead of 2(P-1)/P x.
//            The switch's reduction order is its own: results are identical
//            on every rank but, for f16/bf16 with P > 2, may differ in the
//            last bit from the rank-order fold.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "coll_args.hpp"
#include "cuda_common.hpp"
#include "device_utils.cuh"

namespace commux {
namespace cuda {

namespace {

constexpr int kCollThreads = 512;

template <typename T>
struct AccT {
  using type = T;
};
template <>
struct AccT<__half> {
  using type = float;
};
template <>
struct AccT<__nv_bfloat16> {
  using type = float;
};

template <typename A, typename T>
__device__ __forceinline__ A to_acc(T v) {
  return static_cast<A>(v);
}
template <>
__device__ __forceinline__ float to_acc<float, __half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_acc<float, __nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T, typename A>
__device__ __forceinline__ T from_acc(A v) {
  return static_cast<T>(v);
}
template <>
__device__ __forceinline__ __half from_acc<__half, float>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16, float>(float v) {
  return __float2bfloat16_rn(v);
}

template <int OP, typename A>
__device__ __forceinline__ A combine(A a, A b) {
  if constexpr (OP == kOpSum || OP == kOpAvg) {
    return a + b;
  } else if constexpr (OP == kOpProd) {
    return a * b;
  } else if constexpr (OP == kOpMin) {
    return b < a ? b : a;
  } else {
    return b > a ? b : a;
  }
}

// ---- flag rounds -------------------------------------------------------------

__device__ __forceinline__ std::uint64_t* flag_at(std::uint64_t* base, int phase, int src, int b) {
  return base + (static_cast<std::size_t>(phase) * kMaxCollRanks + src) * kMaxCollCtas + b;
}

// After all threads' stores, thread p stores the flag into rank p's area
// (every rank when `only` < 0, else only rank `only`). The barrier orders the
// CTA's stores before thread p's flag store, whose release at system scope is
// cumulative over them, so no separate fence precedes it.
__device__ __forceinline__ void signal(const CollArgs& a, int phase, std::uint64_t seq, int only = -1) {
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.P && (only < 0 || p == only)) st_release_sys(flag_at(a.flags[p], phase, a.me, blockIdx.x), seq);
}

// Thread p waits for rank p's flag (every rank when `only` < 0). Returns false
// after recording a status if a wait timed out.
__device__ __forceinline__ bool await(const CollArgs& a, int phase, std::uint64_t seq, int only = -1) {
  __shared__ int timed_out;
  if (threadIdx.x == 0) timed_out = 0;
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.P && (only < 0 || p == only)) {
    const std::uint64_t* f = flag_at(a.flags[a.me], phase, p, blockIdx.x);
    const std::uint64_t t0 = globaltimer_ns();
    std::uint32_t spins = 0;
    while (ld_acquire_sys(f) < seq) {
      if ((++spins & 31u) == 0u && globaltimer_ns() - t0 > a.timeout_ns) {
        report_status(a.status, kStatusCollTimeout, static_cast<unsigned long long>(p), seq >> 20,
                      ld_acquire_sys(f));
        atomicExch(&timed_out, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return timed_out == 0;
}

// ---- packed copies and folds -----------------------------------------------

template <typename T>
struct Packs {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0;
}

// dst[i] = src[i], i in [lo, hi); lo is a multiple of the pack size.
template <typename T>
__device__ __forceinline__ void copy_range(T* dst, const T* src, std::int64_t lo, std::int64_t hi) {
  constexpr int N = Packs<T>::N;
  if (lo >= hi) return;
  std::int64_t full_hi = (aligned16(dst + lo) && aligned16(src + lo)) ? lo + ((hi - lo) / N) * N : lo;
  constexpr int U = 4;  // packs in flight per thread
  const std::int64_t step = static_cast<std::int64_t>(blockDim.x) * N;
  std::int64_t i = lo + static_cast<std::int64_t>(threadIdx.x) * N;
  for (; i + (U - 1) * step < full_hi; i += U * step) {
    uint4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k) v[k] = *reinterpret_cast<const uint4*>(src + i + k * step);
#pragma unroll
    for (int k = 0; k < U; ++k) *reinterpret_cast<uint4*>(dst + i + k * step) = v[k];
  }
  for (; i < full_hi; i += step) *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
  for (std::int64_t j = full_hi + threadIdx.x; j < hi; j += blockDim.x) dst[j] = src[j];
}

// out[i] = fold over p of base[p*stride + i], i in [lo, hi).
template <typename T, int OP>
__device__ __forceinline__ void fold_range(T* out, const T* base, std::int64_t stride, int P,
                                           std::int64_t lo, std::int64_t hi) {
  using A = typename AccT<T>::type;
  constexpr int N = Packs<T>::N;
  if (lo >= hi) return;
  const bool vec = aligned16(out + lo) && aligned16(base + lo) && (stride % N) == 0;
  std::int64_t full_hi = vec ? lo + ((hi - lo) / N) * N : lo;
  for (std::int64_t i = lo + static_cast<std::int64_t>(threadIdx.x) * N; i < full_hi;
       i += static_cast<std::int64_t>(blockDim.x) * N) {
    A acc[N];
    {
      uint4 raw = *reinterpret_cast<const uint4*>(base + i);
      const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int k = 0; k < N; ++k) acc[k] = to_acc<A>(v[k]);
    }
    for (int p = 1; p < P; ++p) {
      uint4 raw = *reinterpret_cast<const uint4*>(base + p * stride + i);
      const T* v = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int k = 0; k < N; ++k) acc[k] = combine<OP>(acc[k], to_acc<A>(v[k]));
    }
    uint4 outraw;
    T* o = reinterpret_cast<T*>(&outraw);
#pragma unroll
    for (int k = 0; k < N; ++k) {
      A r = acc[k];
      if constexpr (OP == kOpAvg) r = r / static_cast<A>(P);
      o[k] = from_acc<T>(r);
    }
    *reinterpret_cast<uint4*>(out + i) = outraw;
  }
  for (std::int64_t i = full_hi + threadIdx.x; i < hi; i += blockDim.x) {
    A acc = to_acc<A>(base[i]);
    for (int p = 1; p < P; ++p) acc = combine<OP>(acc, to_acc<A>(base[p * stride + i]));
    if constexpr (OP == kOpAvg) acc = acc / static_cast<A>(P);
    out[i] = from_acc<T>(acc);
  }
}

// Piece k of `parts` of [0, n), cut on pack boundaries.
template <typename T>
__device__ __forceinline__ void piece(std::int64_t n, int parts, int k, std::int64_t& lo,
                                      std::int64_t& hi) {
  constexpr int N = Packs<T>::N;
  std::int64_t packs = (n + N - 1) / N;
  std::int64_t per = (packs + parts - 1) / parts;
  lo = min(n, static_cast<std::int64_t>(k) * per * N);
  hi = min(n, lo + per * N);
}

template <typename T>
__device__ __forceinline__ T* region_a(const CollArgs& a, int p) {
  return reinterpret_cast<T*>(a.data[p] + a.half_off);
}
template <typename T>
__device__ __forceinline__ T* region_b(const CollArgs& a, int p) {
  return reinterpret_cast<T*>(a.data[p] + a.region_bytes + a.half_off);
}
template <typename T>
__device__ __forceinline__ std::int64_t slot_elems(const CollArgs& a, int nslots) {
  constexpr int N = Packs<T>::N;
  std::int64_t e = (a.region_bytes / 2) / static_cast<std::int64_t>(sizeof(T)) / nslots;
  return (e / N) * N;
}

// ---- oneshot -------------------------------------------------------------------

template <typename T, int OP>
__global__ void __launch_bounds__(kCollThreads, 2) oneshot_kernel(const __grid_constant__ CollArgs a) {
  const T* in = static_cast<const T*>(a.in);
  T* out = static_cast<T*>(a.out);
  std::int64_t lo, hi;
  piece<T>(a.n, gridDim.x, blockIdx.x, lo, hi);
  const std::int64_t slot = slot_elems<T>(a, a.P);
  for (int q = 0; q < a.P; ++q) {
    const int p = (a.me + q) % a.P;  // stagger destinations across ranks
    copy_range(region_a<T>(a, p) + a.me * slot, in, lo, hi);
  }
  const std::uint64_t seq = a.seq_base + 1;
  signal(a, 0, seq);
  if (!await(a, 0, seq)) return;
  if (a.mode == kModeReduce && a.me != a.root) return;
  fold_range<T, OP>(out, region_a<T>(a, a.me), slot, a.P, lo, hi);
}

// ---- warp groups -------------------------------------------------------------
//
// nvls_kernel splits each CTA into two warp groups: the "link" group moves
// data across NVLink (multimem operations through the multicast mapping), the
// "local" group copies within this GPU's HBM. Chunk c+1 is copied in while
// chunk c is reduced through the switch and chunk c-1 copied out. Each group syncs
// only on its own named barrier; the groups meet through flags (global, for
// every rank, including this one) and through a shared-memory counter polled
// with a bounded wait, never through a barrier they must both reach, so a
// group that gives up on a timeout cannot leave the other one stuck.

struct Grp {
  int id;    // named barrier (1 or 2)
  int base;  // first thread
  int n;     // threads
  __device__ int tid() const { return static_cast<int>(threadIdx.x) - base; }
  __device__ void sync() const { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
};

// Shared state of the two groups of one CTA.
struct PipeShared {
  int fail[2];        // per group: a wait of that group gave up (written before its barrier)
  int decision[2];    // per group: outcome of a cross-group wait (thread 0 -> group)
  volatile long long folded;  // local group: chunks whose fold is complete
};

__device__ __forceinline__ void gsignal(const CollArgs& a, const Grp& g, int phase, std::uint64_t seq) {
  g.sync();  // every store of the group precedes the flag
  const int p = g.tid();
  if (p < a.P) {
    // a full fence, unlike signal(): the group's stores include multimem.st
    // through the multicast object
    fence_acq_rel_sys();
    st_release_sys(flag_at(a.flags[p], phase, a.me, blockIdx.x), seq);
  }
}

// Thread p of the group waits for rank p's flag; false (the same on every
// thread of the group) if any of those waits gave up, now or earlier.
__device__ __forceinline__ bool gawait(const CollArgs& a, const Grp& g, PipeShared& sh, int gi, int phase,
                                       std::uint64_t seq) {
  const int p = g.tid();
  if (p < a.P) {
    const std::uint64_t* f = flag_at(a.flags[a.me], phase, p, blockIdx.x);
    const std::uint64_t t0 = globaltimer_ns();
    std::uint32_t spins = 0;
    while (ld_acquire_sys(f) < seq) {
      if ((++spins & 31u) == 0u && globaltimer_ns() - t0 > a.timeout_ns) {
        report_status(a.status, kStatusCollTimeout, static_cast<unsigned long long>(p), seq >> 20,
                      ld_acquire_sys(f));
        sh.fail[gi] = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  g.sync();
  return sh.fail[gi] == 0;
}

// dst[i] = src[i] for i in [lo, hi), by the threads of one group, four
// 16-byte packs in flight per thread.
template <typename T>
__device__ __forceinline__ void gcopy(const Grp& g, T* dst, const T* src, std::int64_t lo, std::int64_t hi) {
  constexpr int N = Packs<T>::N;
  constexpr int U = 4;
  if (lo >= hi) return;
  const std::int64_t t = g.tid(), nt = g.n, step = nt * N;
  std::int64_t full_hi = (aligned16(dst + lo) && aligned16(src + lo)) ? lo + ((hi - lo) / N) * N : lo;
  std::int64_t i = lo + t * N;
  for (; i + (U - 1) * step < full_hi; i += U * step) {
    uint4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k) v[k] = *reinterpret_cast<const uint4*>(src + i + k * step);
#pragma unroll
    for (int k = 0; k < U; ++k) *reinterpret_cast<uint4*>(dst + i + k * step) = v[k];
  }
  for (; i < full_hi; i += step) *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
  for (std::int64_t j = full_hi + t; j < hi; j += nt) dst[j] = src[j];
}

// out[i] = fold over p of (p == me ? own[i] : base[p*stride + i]), rank order.
template <typename T, int OP>
__device__ __forceinline__ void gfold(const Grp& g, T* out, const T* base, std::int64_t stride, int P, int me,
                                      const T* own, std::int64_t lo, std::int64_t hi) {
  using A = typename AccT<T>::type;
  constexpr int N = Packs<T>::N;
  if (lo >= hi) return;
  const std::int64_t t = g.tid(), nt = g.n;
  const bool vec = aligned16(out + lo) && aligned16(base + lo) && aligned16(own + lo) && (stride % N) == 0;
  std::int64_t full_hi = vec ? lo + ((hi - lo) / N) * N : lo;
  constexpr int U = 2;  // packs in flight per thread
  const std::int64_t step = nt * N;
  std::int64_t i0 = lo + t * N;
  for (; i0 < full_hi; i0 += U * step) {
    A acc[U][N];
    for (int p = 0; p < P; ++p) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const std::int64_t i = i0 + u * step;
        if (i < full_hi) raw[u] = *reinterpret_cast<const uint4*>(p == me ? own + i : base + p * stride + i);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T* v = reinterpret_cast<const T*>(&raw[u]);
        if (p == 0) {
#pragma unroll
          for (int k = 0; k < N; ++k) acc[u][k] = to_acc<A>(v[k]);
        } else {
#pragma unroll
          for (int k = 0; k < N; ++k) acc[u][k] = combine<OP>(acc[u][k], to_acc<A>(v[k]));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const std::int64_t i = i0 + u * step;
      if (i >= full_hi) break;
      uint4 outraw;
      T* o = reinterpret_cast<T*>(&outraw);
#pragma unroll
      for (int k = 0; k < N; ++k) {
        A r = acc[u][k];
        if constexpr (OP == kOpAvg) r = r / static_cast<A>(P);
        o[k] = from_acc<T>(r);
      }
      *reinterpret_cast<uint4*>(out + i) = outraw;
    }
  }
  for (std::int64_t i = full_hi + t; i < hi; i += nt) {
    A acc = to_acc<A>(me == 0 ? own[i] : base[i]);
    for (int p = 1; p < P; ++p) acc = combine<OP>(acc, to_acc<A>(p == me ? own[i] : base[p * stride + i]));
    if constexpr (OP == kOpAvg) acc = acc / static_cast<A>(P);
    out[i] = from_acc<T>(acc);
  }
}

// Elements per chunk of one segment: a few chunks to pipeline, none below
// 2 MiB (each flag round costs microseconds), within the slot the workspace
// quarter gives each rank.
template <typename T>
__device__ __forceinline__ std::int64_t pipe_chunk(std::int64_t seg, std::int64_t slot_cap) {
  constexpr int N = Packs<T>::N;
  std::int64_t c = (seg + 3) / 4;
  const std::int64_t lo = (2 << 20) / static_cast<std::int64_t>(sizeof(T));
  if (c < lo) c = lo;
  if (c > slot_cap) c = slot_cap;
  return (c + N - 1) / N * N > slot_cap ? slot_cap : (c + N - 1) / N * N;
}

// ---- twoshot (phases in sequence per CTA) -------------------------------------------------------------------

// Phase stamp of CTA 0 (COMMUX_COLL_TRACE): point k of chunk c.
__device__ __forceinline__ void stamp(const CollArgs& a, std::int64_t c, int k) {
  if (a.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && c < kTraceChunks)
    a.trace[c * kTracePoints + k] = globaltimer_ns();
}

template <typename T, int OP>
__global__ void __launch_bounds__(kCollThreads, 2) twoshot_kernel(const __grid_constant__ CollArgs a) {
  constexpr int N = Packs<T>::N;
  const T* in = static_cast<const T*>(a.in);
  T* out = static_cast<T*>(a.out);
  const int P = a.P;
  const bool rs = a.mode == kModeReduceScatter;
  const std::int64_t seg_cap = slot_elems<T>(a, P);
  const std::int64_t total = rs ? a.n * P : a.n;
  // segment s of the tensor: [s*seg, s*seg + seg) (reduce_scatter: block s)
  const std::int64_t seg = rs ? a.n : (((total + P - 1) / P + N - 1) / N) * N;
  const std::int64_t nchunks = (seg + seg_cap - 1) / seg_cap;
  T* a_me = region_a<T>(a, a.me);
  T* b_me = region_b<T>(a, a.me);
  for (std::int64_t c = 0; c < nchunks; ++c) {
    const std::int64_t s0 = c * seg_cap;
    const std::int64_t slen = min(seg_cap, seg - s0);
    std::int64_t lo, hi;
    piece<T>(slen, gridDim.x, blockIdx.x, lo, hi);
    const std::uint64_t seq = a.seq_base + static_cast<std::uint64_t>(c) + 1;
    stamp(a, c, 0);
    // phase 0: my part of segment s -> slot[me] of rank s's A (my own
    // segment's part stays in `in` and is read from there by the fold)
    for (int q = 1; q < P; ++q) {
      const int s = (a.me + q) % P;
      const std::int64_t g = static_cast<std::int64_t>(s) * seg + s0;
      const std::int64_t ghi = rs ? g + hi : min(g + hi, total);
      copy_range(region_a<T>(a, s) + a.me * seg_cap - g, in, g + lo, ghi);
    }
    stamp(a, c, 1);
    signal(a, 0, seq);
    stamp(a, c, 2);
    if (!await(a, 0, seq)) return;
    stamp(a, c, 3);
    // fold my segment: reduce_scatter and allreduce write it straight into
    // `out` (allreduce then pushes it from there), reduce into my B slot
    const std::int64_t mine = static_cast<std::int64_t>(a.me) * seg + s0;
    const std::int64_t mhi = rs ? hi : min(hi, total - mine);
    const bool to_out = rs || a.mode == kModeAllreduce || a.me == a.root;
    T* folded = to_out ? (rs ? out + s0 : out + mine) : b_me + a.me * seg_cap;
    gfold<T, OP>(Grp{0, 0, static_cast<int>(blockDim.x)}, folded, a_me, seg_cap, P, a.me, in + mine, lo, mhi);
    stamp(a, c, 4);
    if (!rs) {
      __syncthreads();
      // phase 1: my folded segment -> slot[me] of B on every rank that needs it
      for (int q = 1; q < P; ++q) {
        const int p = (a.me + q) % P;
        if (a.mode == kModeReduce && p != a.root) continue;
        copy_range(region_b<T>(a, p) + a.me * seg_cap, folded, lo, mhi);
      }
    }
    stamp(a, c, 5);
    signal(a, 1, seq);
    if (!await(a, 1, seq)) return;
    stamp(a, c, 6);
    if (rs || (a.mode == kModeReduce && a.me != a.root)) continue;
    for (int p = 0; p < P; ++p) {
      if (p == a.me) continue;  // folded in place above
      const std::int64_t g = static_cast<std::int64_t>(p) * seg + s0;
      const std::int64_t phi = min(hi, total - g);
      copy_range(out + g, b_me + p * seg_cap - 0, lo, phi);
    }
    stamp(a, c, 7);
  }
}

// ---- barrier ---------------------------------------------------------------------

constexpr int kBarrierPhase = 2;

__global__ void barrier_kernel(const __grid_constant__ CollArgs a) {
  const std::uint64_t seq = a.seq_base + 1;
  // the writes of the kernels before this one on the stream (and any into
  // peers' memory) are performed system-wide before the flags go out
  fence_acq_rel_sys();
  signal(a, kBarrierPhase, seq);
  await(a, kBarrierPhase, seq);
}

// ---- gather (allgather / broadcast) ------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kCollThreads, 2) gather_kernel(const __grid_constant__ CollArgs a) {
  const T* in = static_cast<const T*>(a.in);
  T* out = static_cast<T*>(a.out);
  const int P = a.P;
  const bool bcast = a.mode == kModeBroadcast;
  const std::int64_t slot = slot_elems<T>(a, bcast ? 1 : P);
  const std::int64_t nchunks = (a.n + slot - 1) / slot;
  T* b_me = region_b<T>(a, a.me);
  for (std::int64_t c = 0; c < nchunks; ++c) {
    const std::int64_t c0 = c * slot;
    const std::int64_t clen = min(slot, a.n - c0);
    std::int64_t lo, hi;
    piece<T>(clen, gridDim.x, blockIdx.x, lo, hi);
    const std::uint64_t seq = a.seq_base + static_cast<std::uint64_t>(c) + 1;
    if (bcast) {
      if (a.me == a.root) {
        for (int q = 1; q < P; ++q) {
          const int p = (a.me + q) % P;
          copy_range(region_b<T>(a, p) - c0, in, c0 + lo, c0 + hi);
        }
        if (out != in) copy_range(out, in, c0 + lo, c0 + hi);
        signal(a, 0, seq);
      } else {
        if (!await(a, 0, seq, a.root)) return;
        copy_range(out, b_me - c0, c0 + lo, c0 + hi);
      }
    } else {
      for (int q = 1; q < P; ++q) {
        const int p = (a.me + q) % P;
        copy_range(region_b<T>(a, p) + a.me * slot - c0, in, c0 + lo, c0 + hi);
      }
      copy_range(out + static_cast<std::int64_t>(a.me) * a.n, in, c0 + lo, c0 + hi);
      signal(a, 0, seq);
      if (!await(a, 0, seq)) return;
      for (int q = 1; q < P; ++q) {
        const int p = (a.me + q) % P;
        copy_range(out + static_cast<std::int64_t>(p) * a.n, b_me + p * slot - c0, c0 + lo, c0 + hi);
      }
    }
    // everyone has consumed this chunk before anyone refills the slots
    signal(a, 1, seq);
    if (!await(a, 1, seq)) return;
  }
}

// ---- broadcast: scatter + allgather, pipelined over chunks ---------------------
//
// Chunk c of the message is P pieces of `cap` elements; piece k belongs to
// rank k. The root stores piece k into slot k of rank k's B quarter (c & 1)
// and its own piece into slot root of every rank's quarter; each other rank
// k forwards its piece to every rank but the root and itself, then copies
// all P pieces out. The root's link carries about 2(P-1)/P of the message
// (not P-1 times it), every other rank's about (P-2)/P. Flag phases: 0 =
// root's stores of chunk c landed, 1 = rank k's forward of chunk c landed,
// 2 = rank k copied chunk c out (its quarter may be refilled). A rank's
// iteration c forwards chunk c and copies chunk c-1 out before its flag
// stores, so the copy-out overlaps the forward's NVLink transfer.
template <typename T>
__global__ void __launch_bounds__(kCollThreads, 2) bcast_kernel(const __grid_constant__ CollArgs a) {
  const T* in = static_cast<const T*>(a.in);
  T* out = static_cast<T*>(a.out);
  const int P = a.P, root = a.root, me = a.me;
  const std::int64_t cap = slot_elems<T>(a, 2 * P);
  const std::int64_t chunk = cap * P;
  const std::int64_t nchunks = (a.n + chunk - 1) / chunk;
  auto quarter = [&](int p, std::int64_t c) { return region_b<T>(a, p) + (c & 1) * P * cap; };
  auto seq = [&](std::int64_t c) { return a.seq_base + static_cast<std::uint64_t>(c) + 1; };
  // element range [lo, hi) of this CTA's share of piece k of chunk c, as
  // offsets in the message; base = first element of the piece
  auto share = [&](std::int64_t c, int k, std::int64_t& base, std::int64_t& lo, std::int64_t& hi) {
    base = c * chunk + static_cast<std::int64_t>(k) * cap;
    const std::int64_t len = max(static_cast<std::int64_t>(0), min(cap, a.n - base));
    piece<T>(len, gridDim.x, blockIdx.x, lo, hi);
  };
  if (me == root) {
    for (std::int64_t c = 0; c < nchunks; ++c) {
      if (c >= 2 && !await(a, 2, seq(c - 2))) return;
      for (int q = 1; q < P; ++q) {
        const int p = (me + q) % P;
        std::int64_t base, lo, hi;
        share(c, p, base, lo, hi);  // p's own piece
        copy_range(quarter(p, c) + p * cap - base, in, base + lo, base + hi);
        share(c, root, base, lo, hi);  // the root's piece
        copy_range(quarter(p, c) + root * cap - base, in, base + lo, base + hi);
      }
      if (out != in) {
        std::int64_t lo, hi;
        piece<T>(min(chunk, a.n - c * chunk), gridDim.x, blockIdx.x, lo, hi);
        copy_range(out, in, c * chunk + lo, c * chunk + hi);
      }
      signal(a, 0, seq(c));
      // the root forwards and copies out nothing: its phases 1 and 2 of the
      // chunk hold at once (the others wait on every rank's flags)
      signal(a, 1, seq(c));
      signal(a, 2, seq(c));
    }
    // every rank has copied the last chunk out before the root leaves: a
    // later call cannot reach this call's half of the workspace while a peer
    // still reads it
    if (nchunks >= 1) await(a, 2, seq(nchunks - 1));
    return;
  }
  for (std::int64_t c = 0; c <= nchunks; ++c) {
    if (c < nchunks) {
      if (c >= 2 && !await(a, 2, seq(c - 2))) return;
      if (!await(a, 0, seq(c), root)) return;
      std::int64_t base, lo, hi;
      share(c, me, base, lo, hi);
      const T* mine = quarter(me, c) + me * cap - base;
      for (int q = 1; q < P; ++q) {
        const int p = (me + q) % P;
        if (p == root) continue;
        copy_range(quarter(p, c) + me * cap - base, mine, base + lo, base + hi);
      }
    }
    if (c >= 1) {
      const std::int64_t f = c - 1;
      if (!await(a, 1, seq(f))) return;
      for (int k = 0; k < P; ++k) {
        std::int64_t base, lo, hi;
        share(f, k, base, lo, hi);
        copy_range(out, quarter(me, f) + k * cap - base, base + lo, base + hi);
      }
    }
    if (c < nchunks) signal(a, 1, seq(c));
    if (c >= 1) signal(a, 2, seq(c - 1));
  }
}

// ---- chain: pipelined broadcast and reduce (opt-in) ---------------------------------
//
// Measured at 4 ranks (1 GiB fp32): broadcast 3556 us against 3200 us for
// scatter + allgather and 1630 us for NCCL; reduce 3730 us against 2637 us
// for two-shot. Every hop waits for its predecessor's per-chunk flag, which
// a CTA stores only after its posted stores have landed, so a link runs at
// about 300 GB/s. COMMUX_CHAIN_RANKS=<n> selects it from n ranks.
//
// The ranks form a chain, and chunks of the message flow along it, so every
// link carries the message once. In broadcast the chain starts at the root
// and each rank copies every chunk out. In reduce it ends at the root: each
// rank folds its own input into the partial result it received and passes it
// on (the fold order is the chain order, rank root+1 first; partial results
// travel in the message's type), and the root's fold writes the output.
// Each call's half of region B holds kChainSlots chunk slots per rank; chunk c
// goes to slot c % kChainSlots of the next rank. Flag phases, CTA b to CTA b:
// 0 = "slot holds chunk c" (to the next rank), 1 = "slot of chunk c is free
// again" (to the previous rank), 2 = the end-of-call round among all ranks
// (no rank starts a call that reuses this half while another still reads
// it). A rank waits on its predecessor's phase 0 and its successor's
// phase 1, so no wait cycle can form.
constexpr int kChainSlots = 4;

template <typename T, int OP>
__global__ void __launch_bounds__(kCollThreads, 2) chain_kernel(const __grid_constant__ CollArgs a) {
  using Acc = typename AccT<T>::type;
  constexpr int N = Packs<T>::N;
  const T* in = static_cast<const T*>(a.in);
  T* out = static_cast<T*>(a.out);
  const int P = a.P;
  const bool bcast = a.mode == kModeBroadcast;
  // chain position: broadcast starts at the root, reduce ends at it
  const int head = bcast ? a.root : (a.root + 1) % P;
  const int k = (a.me - head + P) % P;
  const int prev = (a.me + P - 1) % P, next = (a.me + 1) % P;
  const std::int64_t cap = (a.region_bytes / 2) / static_cast<std::int64_t>(sizeof(T)) / kChainSlots / N * N;
  const std::int64_t nchunks = (a.n + cap - 1) / cap;
  auto slot = [&](int p, std::int64_t c) { return region_b<T>(a, p) + (c % kChainSlots) * cap; };
  auto seq = [&](std::int64_t c) { return a.seq_base + static_cast<std::uint64_t>(c) + 1; };
  const std::uint64_t last = a.seq_base + static_cast<std::uint64_t>(nchunks) + 1;
  for (std::int64_t c = 0; c < nchunks; ++c) {
    const std::int64_t c0 = c * cap;
    std::int64_t lo, hi;
    piece<T>(min(cap, a.n - c0), gridDim.x, blockIdx.x, lo, hi);
    const bool first = k == 0, tail = k == P - 1;
    if (!first && !await(a, 0, seq(c), prev)) return;
    T* mine = slot(a.me, c) - c0;  // index the slot with message offsets
    if (!tail && c >= kChainSlots && !await(a, 1, seq(c - kChainSlots), next)) return;
    T* dst = tail ? nullptr : slot(next, c) - c0;
    if (bcast) {
      const T* src = first ? in : mine;
      if (!tail) copy_range(dst, src, c0 + lo, c0 + hi);
      if (!first || out != in) copy_range(out, src, c0 + lo, c0 + hi);
    } else if (first) {
      copy_range(dst, in, c0 + lo, c0 + hi);
    } else {
      // partial (from the previous rank) op my input -> the next rank, or
      // (at the root) -> the output; elementwise, fp32 accumulation
      T* to = tail ? out : dst;
      for (std::int64_t i = c0 + lo + static_cast<std::int64_t>(threadIdx.x); i < c0 + hi; i += blockDim.x) {
        Acc v = combine<OP>(to_acc<Acc>(mine[i]), to_acc<Acc>(in[i]));
        if constexpr (OP == kOpAvg)
          if (tail) v = v / static_cast<Acc>(P);
        to[i] = from_acc<T>(v);
      }
    }
    if (!tail) signal(a, 0, seq(c), next);
    if (!first) signal(a, 1, seq(c), prev);
  }
  signal(a, 2, last);
  await(a, 2, last);
}

// ---- nvls ----// ---- nvls ------------------------------------------------------------------------

__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

constexpr int kNvlsUnroll = 4;

// The switch-side reduction over every rank's copy of the 16-byte pack at
// multicast address p, then (AVG) the division by P.
template <typename T, int OP>
__device__ __forceinline__ uint4 nvls_load(const char* p, int P) {
  std::uint32_t r0, r1, r2, r3;
  if constexpr (std::is_same<T, float>::value) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    if constexpr (OP == kOpAvg) {
      const float pf = static_cast<float>(P);
      r0 = __float_as_uint(__uint_as_float(r0) / pf);
      r1 = __float_as_uint(__uint_as_float(r1) / pf);
      r2 = __float_as_uint(__uint_as_float(r2) / pf);
      r3 = __float_as_uint(__uint_as_float(r3) / pf);
    }
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if constexpr (OP == kOpSum || OP == kOpAvg)
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    else if constexpr (OP == kOpMin)
      asm volatile("multimem.ld_reduce.relaxed.sys.global.min.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    else
      asm volatile("multimem.ld_reduce.relaxed.sys.global.max.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    if constexpr (OP == kOpAvg) {
      const float pf = static_cast<float>(P);
      std::uint32_t* rr[4] = {&r0, &r1, &r2, &r3};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(rr[k]);
        float2 f = __bfloat1622float2(h);
        h = __floats2bfloat162_rn(f.x / pf, f.y / pf);
        *rr[k] = *reinterpret_cast<std::uint32_t*>(&h);
      }
    }
  } else {  // __half
    if constexpr (OP == kOpSum || OP == kOpAvg)
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    else if constexpr (OP == kOpMin)
      asm volatile("multimem.ld_reduce.relaxed.sys.global.min.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    else
      asm volatile("multimem.ld_reduce.relaxed.sys.global.max.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                   : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "l"(p) : "memory");
    if constexpr (OP == kOpAvg) {
      const float pf = static_cast<float>(P);
      std::uint32_t* rr[4] = {&r0, &r1, &r2, &r3};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __half2 h = *reinterpret_cast<__half2*>(rr[k]);
        float2 f = __half22float2(h);
        h = __floats2half2_rn(f.x / pf, f.y / pf);
        *rr[k] = *reinterpret_cast<std::uint32_t*>(&h);
      }
    }
  }
  return make_uint4(r0, r1, r2, r3);
}

// Store a pack through the multicast mapping (the switch writes it into every
// rank's copy); a store moves bits, so the f32 form serves every type.
__device__ __forceinline__ void nvls_store(char* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)), "f"(__uint_as_float(v.w))
               : "memory");
}

template <typename T, int OP>
__device__ __forceinline__ void nvls_pack(char* p, int P) {
  nvls_store(p, nvls_load<T, OP>(p, P));
}

// U packs `stride` bytes apart: all U reductions are issued before the
// first store.
template <typename T, int OP, int U>
__device__ __forceinline__ void nvls_packs(char* p, std::int64_t stride, int P) {
  uint4 v[U];
#pragma unroll
  for (int k = 0; k < U; ++k) v[k] = nvls_load<T, OP>(p + k * stride, P);
#pragma unroll
  for (int k = 0; k < U; ++k) nvls_store(p + k * stride, v[k]);
}

// Pipelined NVLS allreduce. Each call's half of the NVLS buffer holds two
// chunk buffers (chunk c uses buffer c & 1; slot s of a buffer holds segment
// s of the chunk). Flag phases: 0 = my copy of chunk c is in my buffer,
// 1 = I reduced my segment of chunk c and stored it to every rank.
//   local group: [wait 1(c-2)] copy in -> signal 0(c) -> [wait 1(c-1) ->
//                copy out c-1]; then the copy-out of the last chunk
//   link group:  wait 0(c) -> multimem reduce + store my segment -> signal 1(c)
template <typename T, int OP>
__global__ void __launch_bounds__(kCollThreads, 1) nvls_kernel(const __grid_constant__ CollArgs a) {
  constexpr int N = Packs<T>::N;
  __shared__ PipeShared sh;
  if (threadIdx.x == 0) {
    sh.fail[0] = sh.fail[1] = 0;
    sh.decision[0] = sh.decision[1] = 0;
    sh.folded = 0;
  }
  __syncthreads();
  const T* in = static_cast<const T*>(a.in);
  T* out = static_cast<T*>(a.out);
  const int P = a.P;
  const std::int64_t quarter = (a.nvls_bytes / 4) / static_cast<std::int64_t>(sizeof(T));
  const std::int64_t slot_cap = (quarter / P) / N * N;
  const std::int64_t seg = (((a.n + P - 1) / P + N - 1) / N) * N;
  const std::int64_t cap = pipe_chunk<T>(seg, slot_cap);
  const std::int64_t nchunks = (seg + cap - 1) / cap;
  const Grp link{1, 0, kCollThreads / 2}, local{2, kCollThreads / 2, kCollThreads / 2};
  auto ucbuf = [&](std::int64_t c) {
    return reinterpret_cast<T*>(a.nvls_uc + a.nvls_half_off) + ((c & 1) ? quarter : 0);
  };
  auto mcbuf = [&](std::int64_t c) {
    return a.nvls_mc + a.nvls_half_off + ((c & 1) ? quarter : 0) * static_cast<std::int64_t>(sizeof(T));
  };
  if (static_cast<int>(threadIdx.x) < kCollThreads / 2) {
    for (std::int64_t c = 0; c < nchunks; ++c) {
      const std::int64_t s0 = c * cap, slen = min(cap, seg - s0);
      std::int64_t lo, hi;
      piece<T>(slen, gridDim.x, blockIdx.x, lo, hi);
      const std::uint64_t seq = a.seq_base + static_cast<std::uint64_t>(c) + 1;
      if (!gawait(a, link, sh, 0, 0, seq)) return;
      fence_proxy_alias();  // every rank's unicast stores before the multicast loads
      const std::int64_t g = static_cast<std::int64_t>(a.me) * seg + s0;
      const std::int64_t mhi = min(hi, a.n - g);
      char* base = mcbuf(c) + (static_cast<std::int64_t>(a.me) * cap) * static_cast<std::int64_t>(sizeof(T));
      const std::int64_t step = static_cast<std::int64_t>(link.n) * N;
      std::int64_t i = lo + static_cast<std::int64_t>(link.tid()) * N;
      for (; i + (kNvlsUnroll - 1) * step < mhi; i += kNvlsUnroll * step)
        nvls_packs<T, OP, kNvlsUnroll>(base + i * static_cast<std::int64_t>(sizeof(T)),
                                       step * static_cast<std::int64_t>(sizeof(T)), P);
      for (; i < mhi; i += step) nvls_pack<T, OP>(base + i * static_cast<std::int64_t>(sizeof(T)), P);
      gsignal(a, link, 1, seq);
    }
  } else {
    auto copy_out = [&](std::int64_t c) -> bool {
      const std::int64_t s0 = c * cap, slen = min(cap, seg - s0);
      std::int64_t lo, hi;
      piece<T>(slen, gridDim.x, blockIdx.x, lo, hi);
      const std::uint64_t seq = a.seq_base + static_cast<std::uint64_t>(c) + 1;
      if (!gawait(a, local, sh, 1, 1, seq)) return false;
      fence_proxy_alias();  // multicast stores before the unicast loads
      for (int q = 0; q < P; ++q) {
        const int s = (a.me + q) % P;
        const std::int64_t g = static_cast<std::int64_t>(s) * seg + s0;
        gcopy(local, out, ucbuf(c) + s * cap - g, g + lo, min(g + hi, a.n));
      }
      return true;
    };
    for (std::int64_t c = 0; c < nchunks; ++c) {
      const std::int64_t s0 = c * cap, slen = min(cap, seg - s0);
      std::int64_t lo, hi;
      piece<T>(slen, gridDim.x, blockIdx.x, lo, hi);
      const std::uint64_t seq = a.seq_base + static_cast<std::uint64_t>(c) + 1;
      // buffer c&1 is free once every rank stored (and loaded) chunk c-2
      if (c >= 2 && !gawait(a, local, sh, 1, 1, seq - 2)) return;
      for (int q = 0; q < P; ++q) {
        const int s = (a.me + q) % P;
        const std::int64_t g = static_cast<std::int64_t>(s) * seg + s0;
        gcopy(local, ucbuf(c) + s * cap - g, in, g + lo, min(g + hi, a.n));
      }
      fence_proxy_alias();
      gsignal(a, local, 0, seq);
      if (c >= 1 && !copy_out(c - 1)) return;
    }
    if (nchunks >= 1) copy_out(nchunks - 1);
  }
}

template <typename T>
cudaError_t launch_nvls(const CollArgs& a, int ctas, cudaStream_t s) {
  if constexpr (std::is_same<T, float>::value || std::is_same<T, __half>::value ||
                std::is_same<T, __nv_bfloat16>::value) {
    switch (a.op) {
      case kOpSum:
        nvls_kernel<T, kOpSum><<<ctas, kCollThreads, 0, s>>>(a);
        return cudaGetLastError();
      case kOpAvg:
        nvls_kernel<T, kOpAvg><<<ctas, kCollThreads, 0, s>>>(a);
        return cudaGetLastError();
      case kOpMin:
        if constexpr (!std::is_same<T, float>::value) {
          nvls_kernel<T, kOpMin><<<ctas, kCollThreads, 0, s>>>(a);
          return cudaGetLastError();
        }
        break;
      case kOpMax:
        if constexpr (!std::is_same<T, float>::value) {
          nvls_kernel<T, kOpMax><<<ctas, kCollThreads, 0, s>>>(a);
          return cudaGetLastError();
        }
        break;
      default:
        break;
    }
  }
  return cudaErrorInvalidValue;
}

template <typename T, int OP>
cudaError_t launch_reduce_family(const CollArgs& a, int ctas, cudaStream_t s) {
  if (a.algo == kAlgoNvls) return launch_nvls<T>(a, ctas, s);
  if (a.algo == kAlgoChain) {
    chain_kernel<T, OP><<<ctas, kCollThreads, 0, s>>>(a);
    return cudaGetLastError();
  }
  if (a.algo == kAlgoOneShot)
    oneshot_kernel<T, OP><<<ctas, kCollThreads, 0, s>>>(a);
  else
    twoshot_kernel<T, OP><<<ctas, kCollThreads, 0, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_op(const CollArgs& a, int ctas, cudaStream_t s) {
  switch (a.op) {
    case kOpSum:
      return launch_reduce_family<T, kOpSum>(a, ctas, s);
    case kOpProd:
      return launch_reduce_family<T, kOpProd>(a, ctas, s);
    case kOpMin:
      return launch_reduce_family<T, kOpMin>(a, ctas, s);
    case kOpMax:
      return launch_reduce_family<T, kOpMax>(a, ctas, s);
    case kOpAvg:
      return launch_reduce_family<T, kOpAvg>(a, ctas, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_barrier(const CollArgs& a, cudaStream_t s) {
  if (a.P > kMaxCollRanks) return cudaErrorInvalidValue;
  barrier_kernel<<<1, 32, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_coll(const CollArgs& a, int ctas, cudaStream_t s) {
  if (ctas < 1 || ctas > kMaxCollCtas || a.P > kMaxCollRanks) return cudaErrorInvalidValue;
  // broadcast: the root pushes to every peer at 2 ranks (one link either
  // way); from 3 ranks scatter + allgather (the root's link carries about
  // 2(P-1)/P of the message, not P-1 times it), or the pipelined chain where
  // COMMUX_CHAIN_RANKS enables it (a.bcast_chain_ranks > 0)
  if (a.mode == kModeBroadcast && a.P > 2 && !(a.bcast_chain_ranks > 0 && a.P >= a.bcast_chain_ranks)) {
    switch (a.elem_bytes) {
      case 1:
        bcast_kernel<std::uint8_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 2:
        bcast_kernel<std::uint16_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 4:
        bcast_kernel<std::uint32_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 8:
        bcast_kernel<std::uint64_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  if (a.mode == kModeBroadcast && a.P > 2) {
    switch (a.elem_bytes) {
      case 1:
        chain_kernel<std::uint8_t, kOpSum><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 2:
        chain_kernel<std::uint16_t, kOpSum><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 4:
        chain_kernel<std::uint32_t, kOpSum><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 8:
        chain_kernel<std::uint64_t, kOpSum><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  if (a.mode == kModeAllgather || a.mode == kModeBroadcast) {
    switch (a.elem_bytes) {
      case 1:
        gather_kernel<std::uint8_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 2:
        gather_kernel<std::uint16_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 4:
        gather_kernel<std::uint32_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      case 8:
        gather_kernel<std::uint64_t><<<ctas, kCollThreads, 0, s>>>(a);
        break;
      default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  switch (a.dtype) {
    case kF32:
      return dispatch_op<float>(a, ctas, s);
    case kF64:
      return dispatch_op<double>(a, ctas, s);
    case kF16:
      return dispatch_op<__half>(a, ctas, s);
    case kBF16:
      return dispatch_op<__nv_bfloat16>(a, ctas, s);
    case kI32:
      return dispatch_op<std::int32_t>(a, ctas, s);
    case kI64:
      return dispatch_op<std::int64_t>(a, ctas, s);
    case kU8:
      return dispatch_op<std::uint8_t>(a, ctas, s);
    case kI8:
      return dispatch_op<std::int8_t>(a, ctas, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace cuda
}  // namespace commux
