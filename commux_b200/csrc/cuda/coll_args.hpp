#pragma once

// Arguments of the device collective kernels (coll_kernels.cu).
//
// Workspace of each rank (one cudaMalloc, IPC-mapped by every peer):
//   [flags: kFlagPhases x kMaxCollRanks x kMaxCollCtas x u64]
//   [region A: region_bytes][region B: region_bytes]
// The NVLS buffer (when the group has one) is a separate allocation bound to
// an NVSwitch multicast object; it is used by halves the same way.
// Each region is used by halves: a call with epoch e uses half (e & 1) of A
// and of B, so two consecutive calls never touch the same bytes; the flag
// round every call contains guarantees a peer finished call e-2 before call e
// writes into its half again.

#include <cuda_runtime.h>

#include <cstdint>

namespace commux {
namespace cuda {

constexpr int kMaxCollRanks = 16;
constexpr int kMaxCollCtas = 512;
constexpr int kFlagPhases = 4;
constexpr std::size_t kFlagBytes =
    static_cast<std::size_t>(kFlagPhases) * kMaxCollRanks * kMaxCollCtas * sizeof(std::uint64_t);

enum CollMode : int {
  kModeAllreduce = 0,
  kModeReduce = 1,
  kModeReduceScatter = 2,
  kModeAllgather = 3,
  kModeBroadcast = 4,
  kModeBarrier = 5,
};
enum CollAlgo : int { kAlgoOneShot = 0, kAlgoTwoShot = 1, kAlgoNvls = 2, kAlgoChain = 3 };
enum CollOp : int { kOpSum = 0, kOpProd = 1, kOpMin = 2, kOpMax = 3, kOpAvg = 4 };
enum CollDtype : int { kF32 = 0, kF64, kF16, kBF16, kI32, kI64, kU8, kI8 };

struct CollArgs {
  int P;
  int me;
  int root;
  int mode;
  int algo;
  int op;
  int dtype;
  int elem_bytes;
  int bcast_chain_ranks;  // broadcast: along a chain from this many ranks
  std::int64_t n;  // elements: allreduce/reduce total; reduce_scatter and
                   // allgather per-rank block; broadcast total
  const void* in;
  void* out;
  char* data[kMaxCollRanks];            // region A base of each rank (mapped)
  std::uint64_t* flags[kMaxCollRanks];  // flag area of each rank (mapped)
  std::int64_t region_bytes;            // bytes of region A (= region B)
  std::int64_t half_off;                // bytes: 0 or region_bytes / 2
  std::uint64_t seq_base;               // epoch << 20
  std::uint64_t timeout_ns;
  unsigned long long* status;
  // NVLS (kAlgoNvls): this rank's unicast mapping and the group's multicast
  // mapping of the NVLS buffer, used by halves like the regions
  char* nvls_uc;
  char* nvls_mc;
  std::int64_t nvls_bytes;     // whole buffer
  std::int64_t nvls_half_off;  // bytes: 0 or nvls_bytes / 2
  // COMMUX_COLL_TRACE: CTA 0 stamps %globaltimer at the phase boundaries of
  // each chunk into trace[chunk * kTracePoints + point] (host-mapped);
  // nullptr otherwise
  unsigned long long* trace;
};

constexpr int kTracePoints = 8;
constexpr int kTraceChunks = 64;

// True when the NVLS kernel supports (dtype, op): SUM and AVG of
// f32/f16/bf16, MIN and MAX of f16/bf16 (the multimem reductions NVSwitch
// performs).
inline bool nvls_supported(int dtype, int op) {
  if (dtype == kF32) return op == kOpSum || op == kOpAvg;
  if (dtype == kF16 || dtype == kBF16) return op == kOpSum || op == kOpAvg || op == kOpMin || op == kOpMax;
  return false;
}

cudaError_t launch_coll(const CollArgs& a, int ctas, cudaStream_t s);
// The device barrier: one flag round among all ranks (see coll_kernels.cu).
cudaError_t launch_barrier(const CollArgs& a, cudaStream_t s);

}  // namespace cuda
}  // namespace commux
