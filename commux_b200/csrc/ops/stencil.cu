// commux_b200._ops: compute kernels of the halo-exchange workload (sm_100a).
//
// jacobi7: one 7-point Jacobi sweep of a halo-padded 3-D fp64/fp32 field,
//   v[z,y,x] = (u[z±1,y,x] + u[z,y±1,x] + u[z,y,x±1]) / 6   (interior only),
// fused with the residual sum((v-u)^2) (atomically accumulated per block).
// HBM-bound: each CTA owns a 32x8 (x,y) column tile and marches along z with
// the z-1/z/z+1 values in registers and the current plane (with its x/y halo)
// in shared memory, so every input element is read from DRAM about once.
// The ghost shell of v is not written (the halo exchange fills it).

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <string>

#include "stencil_tma.cuh"

namespace {

constexpr int kTX = 32;
constexpr int kTY = 8;
constexpr int kZB = 16;  // planes per CTA

std::atomic<std::int64_t> g_launches{0};

template <typename T>
__global__ void __launch_bounds__(kTX* kTY)
    jacobi7_kernel(const T* __restrict__ u, T* __restrict__ v, int nz, int ny, int nx, int h,
                   stencil::SubBox sb, double* __restrict__ residual) {
  __shared__ T plane[kTY + 2][kTX + 2];
  __shared__ double red[kTX * kTY / 32];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int x = h + sb.ox + blockIdx.x * kTX + tx;  // padded coordinates
  const int y = h + sb.oy + blockIdx.y * kTY + ty;
  const int z0 = h + sb.oz + blockIdx.z * kZB;
  const int z1 = min(z0 + kZB, h + sb.oz + sb.ez);
  const int ix = sb.ox + sb.ex, iy = sb.oy + sb.ey;  // end of the box (interior coordinates)
  const bool active = x < h + ix && y < h + iy;
  const std::int64_t sy = nx, sz = static_cast<std::int64_t>(ny) * nx;
  const std::int64_t col = static_cast<std::int64_t>(y) * sy + x;
  double acc = 0.0;
  T below = active ? u[(z0 - 1) * sz + col] : T(0);
  T cur = active ? u[z0 * sz + col] : T(0);
  for (int z = z0; z < z1; ++z) {
    const std::int64_t zo = z * sz;
    T above = active ? u[zo + sz + col] : T(0);
    plane[ty + 1][tx + 1] = cur;
    if (active) {
      if (tx == 0) plane[ty + 1][0] = u[zo + col - 1];
      if (tx == kTX - 1 || x == h + ix - 1) plane[ty + 1][tx + 2] = u[zo + col + 1];
      if (ty == 0) plane[0][tx + 1] = u[zo + col - sy];
      if (ty == kTY - 1 || y == h + iy - 1) plane[ty + 2][tx + 1] = u[zo + col + sy];
    }
    __syncthreads();
    if (active) {
      T s = below + above + plane[ty + 1][tx] + plane[ty + 1][tx + 2] + plane[ty][tx + 1] +
            plane[ty + 2][tx + 1];
      T nv = s / T(6);
      v[zo + col] = nv;
      double d = static_cast<double>(nv) - static_cast<double>(cur);
      acc += d * d;
    }
    __syncthreads();
    below = cur;
    cur = above;
  }
  if (residual != nullptr) {
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    const int lane = (ty * kTX + tx) & 31, warp = (ty * kTX + tx) >> 5;
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (warp == 0) {
      acc = lane < kTX * kTY / 32 ? red[lane] : 0.0;
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) atomicAdd(residual, acc);
    }
  }
}

// The interior's one-cell boundary layer: the cells whose 7-point stencil
// reads a ghost cell, i.e. what a core sub-box update (origin 1, extent
// n - 2 per dim) leaves out. One thread per cell over six slabs: z = 0 and
// z = iz-1 (all y, x), y = 0 and y = iy-1 (z inside, all x), x = 0 and
// x = ix-1 (z and y inside). Needs iz, iy, ix >= 3.
template <typename T>
__global__ void __launch_bounds__(256)
    jacobi7_shell_kernel(const T* __restrict__ u, T* __restrict__ v, int ny, int nx, int h, int iz, int iy,
                         int ix, double* __restrict__ residual) {
  __shared__ double red[8];
  const std::int64_t A = static_cast<std::int64_t>(iy) * ix;         // z slab
  const std::int64_t B = static_cast<std::int64_t>(iz - 2) * ix;     // y slab
  const std::int64_t C = static_cast<std::int64_t>(iz - 2) * (iy - 2);  // x slab
  const std::int64_t total = 2 * (A + B + C);
  const std::int64_t sy = nx, sz = static_cast<std::int64_t>(ny) * nx;
  double acc = 0.0;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int z, y, x;
    std::int64_t r = t;
    if (r < 2 * A) {
      const int slab = static_cast<int>(r / A);
      r -= slab * A;
      z = slab ? iz - 1 : 0;
      y = static_cast<int>(r / ix);
      x = static_cast<int>(r - static_cast<std::int64_t>(y) * ix);
    } else if ((r -= 2 * A) < 2 * B) {
      const int slab = static_cast<int>(r / B);
      r -= slab * B;
      y = slab ? iy - 1 : 0;
      z = 1 + static_cast<int>(r / ix);
      x = static_cast<int>(r - static_cast<std::int64_t>(z - 1) * ix);
    } else {
      r -= 2 * B;
      const int slab = static_cast<int>(r / C);
      r -= slab * C;
      x = slab ? ix - 1 : 0;
      z = 1 + static_cast<int>(r / (iy - 2));
      y = 1 + static_cast<int>(r - static_cast<std::int64_t>(z - 1) * (iy - 2));
    }
    const std::int64_t o = (z + h) * sz + (y + h) * sy + (x + h);
    const T ctr = u[o];
    // same summation order as the tiled kernels (z, then x, then y), so a
    // core + shell update equals the whole-interior one bit for bit
    const T nv = (u[o - sz] + u[o + sz] + u[o - 1] + u[o + 1] + u[o - sy] + u[o + sy]) / T(6);
    v[o] = nv;
    const double d = static_cast<double>(nv) - static_cast<double>(ctr);
    acc += d * d;
  }
  if (residual != nullptr) {
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (warp == 0) {
      acc = lane < 8 ? red[lane] : 0.0;
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) atomicAdd(residual, acc);
    }
  }
}

bool use_simple() {
  static const bool v = [] {
    const char* e = std::getenv("COMMUX_JACOBI");
    return e != nullptr && std::string(e) == "simple";
  }();
  return v;
}

// host-mapped status word of the TMA kernel (nonzero: a bounded wait gave up)
unsigned* status_word(unsigned** dev) {
  static unsigned* host = nullptr;
  static unsigned* device = nullptr;
  if (host == nullptr) {
    C10_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&host), 64, cudaHostAllocMapped | cudaHostAllocPortable));
    *host = 0;
    C10_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&device), host, 0));
  }
  *dev = device;
  return host;
}

// cuTensorMapEncodeTiled, resolved through the runtime at first use: the
// extension does not link libcuda, so it imports on machines without a GPU
// driver (a build host) and only needs the driver once a kernel launches.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr,
                "jacobi7: the CUDA driver has no cuTensorMapEncodeTiled");
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

template <typename T>
void launch_tma(const at::Tensor& u, at::Tensor& v, int nz, int ny, int nx, int h, stencil::SubBox sb,
                double* res, cudaStream_t stream) {
  using B = stencil::Box<T>;
  CUtensorMap map;
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(nx), static_cast<cuuint64_t>(ny), static_cast<cuuint64_t>(nz)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(nx) * sizeof(T),
                           static_cast<cuuint64_t>(nx) * ny * sizeof(T)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(B::kW), static_cast<cuuint32_t>(B::kH), 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult rc = encode_tiled()(
      &map, sizeof(T) == 8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT64 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
      const_cast<void*>(u.data_ptr()), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(rc == CUDA_SUCCESS, "jacobi7: cuTensorMapEncodeTiled failed (", static_cast<int>(rc), ")");
  static bool attr_set[2] = {false, false};
  const int which = sizeof(T) == 8 ? 0 : 1;
  if (!attr_set[which]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(stencil::jacobi7_tma_kernel<T>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, B::kSmem));
    attr_set[which] = true;
  }
  unsigned* st_dev = nullptr;
  status_word(&st_dev);
  static const std::uint64_t limit_ns = [] {
    const char* e = std::getenv("COMMUX_KERNEL_WAIT_MS");
    return static_cast<std::uint64_t>(e ? std::atoll(e) : 2000) * 1000000ull;
  }();
  dim3 grid((sb.ex + stencil::kTX - 1) / stencil::kTX, (sb.ey + stencil::kTY - 1) / stencil::kTY,
            (sb.ez + stencil::kZB - 1) / stencil::kZB);
  stencil::jacobi7_tma_kernel<T><<<grid, stencil::kThreads, B::kSmem, stream>>>(
      map, v.data_ptr<T>(), nz, ny, nx, h, sb, res, st_dev, limit_ns);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// 0 when every TMA wait completed; nonzero after a bounded wait gave up.
int64_t kernel_status(bool reset) {
  unsigned* dev = nullptr;
  unsigned* host = status_word(&dev);
  int64_t v = *reinterpret_cast<volatile unsigned*>(host);
  if (reset) *host = 0;
  return v;
}

// v[interior] = jacobi(u); residual (optional, fp64 scalar on the device) += sum (v-u)^2.
// part 0: the whole interior; 1: its core (cells whose stencil reads no ghost
// cell); 2: the one-cell boundary layer around the core. Parts 1 and 2
// together write exactly what part 0 writes.
void jacobi7(const at::Tensor& u, at::Tensor& v, int64_t halo, c10::optional<at::Tensor> residual,
             int64_t part) {
  TORCH_CHECK(u.is_cuda() && v.is_cuda(), "jacobi7: CUDA tensors");
  TORCH_CHECK(u.dim() == 3 && u.sizes() == v.sizes(), "jacobi7: matching 3-D fields");
  TORCH_CHECK(u.is_contiguous() && v.is_contiguous(), "jacobi7: contiguous fields");
  TORCH_CHECK(u.scalar_type() == v.scalar_type(), "jacobi7: same dtype");
  TORCH_CHECK(halo >= 1, "jacobi7: halo >= 1");
  const int nz = u.size(0), ny = u.size(1), nx = u.size(2), h = static_cast<int>(halo);
  const int iz = nz - 2 * h, iy = ny - 2 * h, ix = nx - 2 * h;
  TORCH_CHECK(iz > 0 && iy > 0 && ix > 0, "jacobi7: field smaller than its halo");
  double* res = nullptr;
  if (residual.has_value()) {
    TORCH_CHECK(residual->is_cuda() && residual->scalar_type() == at::kDouble && residual->numel() >= 1,
                "jacobi7: residual must be a CUDA float64 tensor");
    res = residual->data_ptr<double>();
  }
  TORCH_CHECK(part >= 0 && part <= 2, "jacobi7: part is 0 (all), 1 (core) or 2 (shell)");
  TORCH_CHECK(part == 0 || (iz >= 3 && iy >= 3 && ix >= 3), "jacobi7: a core/shell split needs an interior of "
              "at least 3 points per dim");
  c10::cuda::CUDAGuard g(u.device());
  auto stream = c10::cuda::getCurrentCUDAStream(u.device().index()).stream();
  if (part == 2) {
    const std::int64_t cells = 2 * (static_cast<std::int64_t>(iy) * ix + static_cast<std::int64_t>(iz - 2) * ix +
                                    static_cast<std::int64_t>(iz - 2) * (iy - 2));
    int sms = 0;
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, u.device().index()));
    const int blocks = static_cast<int>(std::min<std::int64_t>((cells + 255) / 256, 8ll * sms));
    if (u.scalar_type() == at::kDouble)
      jacobi7_shell_kernel<double><<<blocks, 256, 0, stream>>>(u.data_ptr<double>(), v.data_ptr<double>(), ny, nx,
                                                               h, iz, iy, ix, res);
    else if (u.scalar_type() == at::kFloat)
      jacobi7_shell_kernel<float><<<blocks, 256, 0, stream>>>(u.data_ptr<float>(), v.data_ptr<float>(), ny, nx, h,
                                                              iz, iy, ix, res);
    else
      TORCH_CHECK(false, "jacobi7: float32 or float64 fields");
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    g_launches++;
    return;
  }
  const stencil::SubBox sb = part == 1 ? stencil::SubBox{1, 1, 1, iz - 2, iy - 2, ix - 2}
                                       : stencil::SubBox{0, 0, 0, iz, iy, ix};
  const bool tma_ok = (static_cast<std::int64_t>(nx) * u.element_size()) % 16 == 0 &&
                      (reinterpret_cast<std::uintptr_t>(u.data_ptr()) & 15u) == 0 && ix >= 1;
  if (tma_ok && !use_simple()) {
    if (u.scalar_type() == at::kDouble)
      launch_tma<double>(u, v, nz, ny, nx, h, sb, res, stream);
    else if (u.scalar_type() == at::kFloat)
      launch_tma<float>(u, v, nz, ny, nx, h, sb, res, stream);
    else
      TORCH_CHECK(false, "jacobi7: float32 or float64 fields");
    g_launches++;
    return;
  }
  dim3 block(kTX, kTY);
  dim3 grid((sb.ex + kTX - 1) / kTX, (sb.ey + kTY - 1) / kTY, (sb.ez + kZB - 1) / kZB);
  if (u.scalar_type() == at::kDouble)
    jacobi7_kernel<double><<<grid, block, 0, stream>>>(u.data_ptr<double>(), v.data_ptr<double>(), nz, ny,
                                                       nx, h, sb, res);
  else if (u.scalar_type() == at::kFloat)
    jacobi7_kernel<float><<<grid, block, 0, stream>>>(u.data_ptr<float>(), v.data_ptr<float>(), nz, ny, nx,
                                                      h, sb, res);
  else
    TORCH_CHECK(false, "jacobi7: float32 or float64 fields");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  g_launches++;
}

int64_t launches() { return g_launches.load(); }

}  // namespace

PYBIND11_MODULE(_ops, m) {
  m.doc() = "commux_b200 compute kernels (sm_100a)";
  m.def("jacobi7", &jacobi7, py::arg("u"), py::arg("v"), py::arg("halo"), py::arg("residual") = py::none(),
        py::arg("part") = 0);
  m.def("launches", &launches);
  m.def("kernel_status", &kernel_status, py::arg("reset") = false);
}
