#pragma once

// Device-side helpers: system-scope acquire/release accesses for flags that a
// peer GPU writes over NVLink, the global nanosecond timer for bounded waits,
// and 16-byte vector copies.

#include <cuda_runtime.h>

#include <cstdint>

namespace commux {
namespace cuda {

__device__ __forceinline__ std::uint64_t ld_acquire_sys(const std::uint64_t* p) {
  std::uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(std::uint64_t* p, std::uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ std::uint32_t ld_acquire_sys_u32(const std::uint32_t* p) {
  std::uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u32(std::uint32_t* p, std::uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys_u32(std::uint32_t* p, std::uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ std::uint32_t ld_relaxed_sys_u32(const std::uint32_t* p) {
  std::uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ std::uint64_t globaltimer_ns() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Record the first device error (code + three words of context) in a
// host-mapped status block; later errors keep the first one.
__device__ __forceinline__ void report_status(unsigned long long* st, unsigned long long code,
                                              unsigned long long a, unsigned long long b,
                                              unsigned long long c) {
  if (st == nullptr) return;
  if (atomicCAS(st, 0ull, code) == 0ull) {
    st[1] = a;
    st[2] = b;
    st[3] = c;
    __threadfence_system();
  }
}

template <int BYTES>
struct VecT;
template <>
struct VecT<16> {
  using T = uint4;
};
template <>
struct VecT<8> {
  using T = uint2;
};
template <>
struct VecT<4> {
  using T = unsigned int;
};
template <>
struct VecT<2> {
  using T = unsigned short;
};
template <>
struct VecT<1> {
  using T = unsigned char;
};

}  // namespace cuda
}  // namespace commux
