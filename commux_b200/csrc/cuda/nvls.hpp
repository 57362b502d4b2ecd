#pragma once

// NVLink SHARP (NVLS) buffer: one physical allocation per rank, all bound to
// one NVSwitch multicast object. Each rank maps its own allocation (unicast,
// plain loads and stores of local HBM) and the multicast object (multimem
// loads that return the switch-side reduction over every rank's copy, and
// multimem stores that the switch replicates into every rank's copy).
//
// Set-up is collective over the group: rank 0 creates the multicast object
// and hands its file descriptor to the other ranks over a Unix-domain socket
// (SCM_RIGHTS), every rank adds its device, a store round makes sure every
// device is in before anyone binds memory, and a last round agrees on the
// outcome so that either every rank uses NVLS or none does.

#include <cuda.h>

#include <cstddef>
#include <memory>
#include <string>

namespace commux {

class Engine;

namespace cuda {

class NvlsBuffer {
 public:
  // Collective: every rank of `eng` calls this with the same `bytes` (and
  // `supported_everywhere` computed from the same exchanged records). Returns
  // nullptr on every rank if any rank could not set its part up; `why` then
  // says what failed on this rank (or that a peer failed).
  static std::unique_ptr<NvlsBuffer> create(Engine* eng, int dev, std::size_t bytes, std::string* why);
  ~NvlsBuffer();
  NvlsBuffer(const NvlsBuffer&) = delete;
  NvlsBuffer& operator=(const NvlsBuffer&) = delete;

  char* uc() const { return reinterpret_cast<char*>(uc_va_); }
  char* mc() const { return reinterpret_cast<char*>(mc_va_); }
  std::size_t size() const { return size_; }

  // True when this device can take part (driver and device support).
  static bool device_supported(int dev);

 private:
  NvlsBuffer() = default;
  void release();

  int dev_ = -1;
  CUdevice cudev_ = 0;
  std::size_t size_ = 0;
  CUmemGenericAllocationHandle mc_ = 0;
  CUmemGenericAllocationHandle phys_ = 0;
  CUdeviceptr uc_va_ = 0;
  CUdeviceptr mc_va_ = 0;
  bool added_ = false, bound_ = false, uc_mapped_ = false, mc_mapped_ = false;
};

}  // namespace cuda
}  // namespace commux
