#pragma once

// Internal to the CUDA transport (transport.cpp, plan.cpp): the records a
// sender publishes for a device message, and the host-side construction of
// the pull kernel's copy descriptors from two tensor layouts.

#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "cuda_common.hpp"
#include "layout.hpp"
#include "transport.hpp"

namespace commux {
namespace cuda {
namespace {


constexpr std::uint32_t kWireMagic = 0x54524443u;
constexpr int kWireDims = 8;
constexpr std::uint64_t kSlots = 1ull << 16;  // consumed-flag slots per device

// One tensor of a device message, as the sender describes it.
struct SegWire {
  std::uint64_t buffer_id;  // allocation id in the sender process (0: local)
  std::uint64_t base;       // allocation base address in the sender process
  std::uint64_t alloc_size;
  std::uint64_t offset;     // first element, bytes from base
  cudaIpcMemHandle_t handle;
  std::uint32_t elem;
  std::int32_t ndim;
  std::int64_t sizes[kWireDims];
  std::int64_t strides[kWireDims];  // elements
};

struct DrtsWire {
  std::uint32_t magic;
  std::uint32_t nseg;
  std::int32_t pid;
  std::int32_t device;
  unsigned char uuid[16];
  std::uint32_t sender_waits_on_device;
  std::uint32_t pad;
  std::uint64_t mbox_id;
  std::uint64_t mbox_base;
  cudaIpcMemHandle_t mbox_handle;
  std::uint64_t slot;
  std::uint64_t value;
};

cudaStream_t current_stream(int dev) {
  return c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream();
}

void cu_check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* s = nullptr;
  cuGetErrorString(r, &s);
  throw std::runtime_error(std::string("commux CUDA driver error in ") + what + ": " +
                           (s ? s : "unknown"));
}

template <typename T>
std::shared_ptr<T> state(const ReqPtr& r) {
  return std::static_pointer_cast<T>(r->dev);
}

bool contiguous_wire(const SegWire& s) {
  std::int64_t expect = 1;
  for (int k = s.ndim - 1; k >= 0; --k) {
    if (s.sizes[k] != 1 && s.strides[k] != expect) return false;
    expect *= s.sizes[k];
  }
  return true;
}

std::int64_t numel_wire(const SegWire& s) {
  std::int64_t n = 1;
  for (int k = 0; k < s.ndim; ++k) n *= s.sizes[k];
  return n;
}

// Narrow rows (a halo x-face: 16-byte runs at a row pitch) cross NVLink far
// below its bandwidth when a peer reads them one by one; such a send is
// packed into a contiguous staging buffer on its own GPU first, and the
// receiver reads that buffer.
constexpr std::int64_t kPackRunBytes = 512;

bool narrow_rows(const at::Tensor& t) {
  if (t.numel() == 0 || t.dim() > kWireDims) return false;
  std::vector<std::int64_t> sz(t.sizes().begin(), t.sizes().end()), sd(t.strides().begin(), t.strides().end());
  auto d = dims_of(sz.data(), sd.data(), t.dim());
  std::vector<Dim> m;
  if (!refine(d, d, m) || m.empty()) return false;
  const Dim& in = m.back();
  const std::int64_t run = (in.ss == 1 ? in.size : 1) * static_cast<std::int64_t>(t.element_size());
  return run < kPackRunBytes;
}


}  // namespace
}  // namespace cuda
}  // namespace commux
