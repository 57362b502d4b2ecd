#pragma once

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace commux {
namespace clocks {

struct Sample {
  std::int64_t t_us = 0;
  unsigned int sm_mhz = 0;
  unsigned int sm_max_mhz = 0;
  unsigned long long reasons = 0;
  unsigned int power_mw = 0;
};

// Polls NVML (read-only) for one GPU, named by PCI bus id or index.
class Sampler {
 public:
  Sampler(const std::string& gpu, int interval_us);
  ~Sampler();
  void start();
  std::vector<Sample> stop();  // joins the thread, returns every sample
  const std::string& error() const { return error_; }

 private:
  void* dev_ = nullptr;
  int interval_us_;
  std::atomic<bool> stop_{false};
  std::thread thread_;
  std::mutex mu_;
  std::vector<Sample> samples_;
  std::string error_;
};

}  // namespace clocks
}  // namespace commux
