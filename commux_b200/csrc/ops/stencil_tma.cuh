#pragma once

// TMA-pipelined 7-point Jacobi sweep (sm_100a).
//
// Each CTA owns a TX x TY column tile of the interior and marches along z over
// ZB output planes. Input planes (tile + 1-point x/y halo) arrive by
// cp.async.bulk.tensor (TMA) into a ring of kStages shared-memory buffers; a
// per-buffer mbarrier counts the bytes in. While planes z-1, z, z+1 are being
// consumed, the next kStages-3 planes are already in flight, which is what
// keeps HBM busy (one load per warp per plane left the first version latency
// bound). One elected thread issues the copies after a CTA barrier frees the
// buffer. Every mbarrier wait is bounded by %globaltimer: on timeout the
// kernel records a status word and stops issuing, waits (bounded) for its
// copies in flight and returns.
//
// TMA alignment: the innermost box coordinate times the element size must be
// a multiple of 16 bytes, so the box starts at the x coordinate rounded down
// to 16 bytes and is wide enough to cover the shift (kBoxW).

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace stencil {

constexpr int kTX = 64;      // interior points per CTA along x
constexpr int kTY = 16;      // along y
constexpr int kZB = 32;      // output planes per CTA
constexpr int kStages = 6;   // plane buffers in the ring
constexpr int kThreads = 256;

template <typename T>
struct Box {
  static constexpr int kAlign = 16 / sizeof(T);                                  // elements
  static constexpr int kW = ((kTX + 2 + kAlign - 1) + kAlign - 1) / kAlign * kAlign;  // box width
  static constexpr int kH = kTY + 2;
  static constexpr int kBytes = kW * kH * static_cast<int>(sizeof(T));
  static constexpr int kStride = (kBytes + 127) / 128 * 128;                      // per buffer
  static constexpr int kSmem = kStages * kStride + kStages * 8;
};

__device__ __forceinline__ std::uint32_t smem_u32(const void* p) {
  return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ std::uint64_t gtimer() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(std::uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(std::uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(std::uint64_t* bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.b32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait; false if it gave up.
__device__ __forceinline__ bool mbar_wait(std::uint64_t* bar, unsigned parity, std::uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const std::uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, parity)) {
    if (gtimer() - t0 > limit_ns) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// x origin of the box for tile bx (rounded down to 16 bytes) and the shift of
// the tile's first halo column inside the box.
template <typename T>
__device__ __forceinline__ void box_x(int h, int bx, int& x0, int& shift) {
  const int want = h - 1 + bx * kTX;
  x0 = want / Box<T>::kAlign * Box<T>::kAlign;
  shift = want - x0;
}

// Output sub-box of the interior: origin (oz, oy, ox) and extent (ez, ey, ex)
// in interior coordinates (the whole interior: origin 0, extent iz/iy/ix).
// A sub-box lets the core of the field (cells whose stencil reads no ghost
// cell) be updated while the halo exchange is still filling the ghosts.
struct SubBox {
  int oz, oy, ox, ez, ey, ex;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) jacobi7_tma_kernel(const __grid_constant__ CUtensorMap umap,
                                                                T* __restrict__ v, int nz, int ny, int nx,
                                                                int h, SubBox sb,
                                                                double* __restrict__ residual,
                                                                unsigned* __restrict__ status,
                                                                std::uint64_t limit_ns) {
  extern __shared__ __align__(128) unsigned char smem[];
  using B = Box<T>;
  std::uint64_t* bars = reinterpret_cast<std::uint64_t*>(smem + kStages * B::kStride);
  auto plane = [&](int s) { return reinterpret_cast<T*>(smem + s * B::kStride); };

  const int bx = blockIdx.x, by = blockIdx.y;
  int x0, shift;
  box_x<T>(h + sb.ox, bx, x0, shift);
  const int y0 = h + sb.oy - 1 + by * kTY;
  const int zs = h + sb.oz + blockIdx.z * kZB;         // first output plane
  const int nout = min(kZB, h + sb.oz + sb.ez - zs);   // output planes of this CTA
  const int nload = nout + 2;                          // input planes z-1 .. z+nout
  const int tid = threadIdx.x;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    for (int p = 0; p < kStages && p < nload; ++p) {
      mbar_expect_tx(&bars[p], B::kBytes);
      tma_load_3d(plane(p), &umap, x0, y0, zs - 1 + p, &bars[p]);
    }
  }
  // thread -> (row ty, columns tx + 16k)
  const int ty = tid / 16, tx = tid % 16;
  const int gy = h + sb.oy + by * kTY + ty;
  double acc = 0.0;
  bool ok = true;
  int done_iters = 0;  // iterations that freed their buffer
  for (int i = 0; i < nout; ++i) {
    // planes i, i+1, i+2 (z-1, z, z+1) must have landed; planes up to i+1
    // were waited for in the previous iteration
    bool fail = false;
    for (int p = (i == 0 ? 0 : i + 2); p <= i + 2 && !fail; ++p)
      fail = !mbar_wait(&bars[p % kStages], (p / kStages) & 1u, limit_ns);
    if (__syncthreads_or(fail)) {  // the CTA agrees before anyone leaves the loop
      ok = false;
      break;
    }
    const T* zm = plane(i % kStages);
    const T* zc = plane((i + 1) % kStages);
    const T* zp = plane((i + 2) % kStages);
    const int z = zs + i;
    const int r = ty + 1;
    if (gy < h + sb.oy + sb.ey) {
#pragma unroll
      for (int k = 0; k < kTX / 16; ++k) {
        const int lx = tx + 16 * k;
        const int gx = h + sb.ox + bx * kTX + lx;
        if (gx < h + sb.ox + sb.ex) {
          const int c = shift + 1 + lx;
          const T ctr = zc[r * B::kW + c];
          const T s = zm[r * B::kW + c] + zp[r * B::kW + c] + zc[r * B::kW + c - 1] +
                      zc[r * B::kW + c + 1] + zc[(r - 1) * B::kW + c] + zc[(r + 1) * B::kW + c];
          const T nv = s / T(6);
          v[(static_cast<std::int64_t>(z) * ny + gy) * nx + gx] = nv;
          const double d = static_cast<double>(nv) - static_cast<double>(ctr);
          acc += d * d;
        }
      }
    }
    __syncthreads();  // buffer of plane i is free
    if (tid == 0 && i + kStages < nload) {
      const int p = i + kStages;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&bars[p % kStages], B::kBytes);
      tma_load_3d(plane(p % kStages), &umap, x0, y0, zs - 1 + p, &bars[p % kStages]);
    }
    done_iters = i + 1;
  }
  if (!ok && tid == 0) {
    if (status != nullptr) atomicExch(status, 1u);
    // copies already issued target this CTA's shared memory: let them land
    // (bounded) before the CTA exits. Planes below done_iters + 2 were
    // consumed; planes below `issued` were requested.
    const int issued = min(nload, kStages + done_iters);
    for (int p = done_iters == 0 ? 0 : done_iters + 2; p < issued; ++p)
      mbar_wait(&bars[p % kStages], (p / kStages) & 1u, limit_ns);
  }
  __syncthreads();
  if (residual != nullptr) {
    __shared__ double red[kThreads / 32];
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if ((tid & 31) == 0) red[tid >> 5] = acc;
    __syncthreads();
    if (tid < 32) {
      acc = tid < kThreads / 32 ? red[tid] : 0.0;
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (tid == 0) atomicAdd(residual, acc);
    }
  }
}

}  // namespace stencil
