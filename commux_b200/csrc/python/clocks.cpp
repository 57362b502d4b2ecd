// Native clock sampler for the benchmarks: a C++ thread that queries NVML
// (loaded with dlopen, so nothing links against it) every `interval_us`
// for the SM clock, the maximum SM clock, the power draw and the active
// clock-event reasons of one GPU, without the Python GIL, so a timed region
// of a few milliseconds still gets a sample per millisecond. Only NVML query
// functions are called; no GPU setting is read-modified-written.

#include "clocks.hpp"

#include <dlfcn.h>

#include <chrono>

namespace commux {
namespace clocks {

namespace {

using nvmlReturn_t = int;
using nvmlDevice_t = void*;
constexpr int kNvmlClockSm = 1;  // NVML_CLOCK_SM

struct Nvml {
  void* lib = nullptr;
  nvmlReturn_t (*init)() = nullptr;
  nvmlReturn_t (*by_bus_id)(const char*, nvmlDevice_t*) = nullptr;
  nvmlReturn_t (*by_index)(unsigned int, nvmlDevice_t*) = nullptr;
  nvmlReturn_t (*clock)(nvmlDevice_t, int, unsigned int*) = nullptr;
  nvmlReturn_t (*max_clock)(nvmlDevice_t, int, unsigned int*) = nullptr;
  nvmlReturn_t (*reasons)(nvmlDevice_t, unsigned long long*) = nullptr;
  nvmlReturn_t (*power)(nvmlDevice_t, unsigned int*) = nullptr;
  bool ok = false;
};

Nvml& nvml() {
  static Nvml n = [] {
    Nvml x;
    x.lib = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
    if (x.lib == nullptr) return x;
    auto sym = [&](const char* a) { return dlsym(x.lib, a); };
    x.init = reinterpret_cast<nvmlReturn_t (*)()>(sym("nvmlInit_v2"));
    x.by_bus_id =
        reinterpret_cast<nvmlReturn_t (*)(const char*, nvmlDevice_t*)>(sym("nvmlDeviceGetHandleByPciBusId_v2"));
    x.by_index = reinterpret_cast<nvmlReturn_t (*)(unsigned int, nvmlDevice_t*)>(sym("nvmlDeviceGetHandleByIndex_v2"));
    x.clock = reinterpret_cast<nvmlReturn_t (*)(nvmlDevice_t, int, unsigned int*)>(sym("nvmlDeviceGetClockInfo"));
    x.max_clock =
        reinterpret_cast<nvmlReturn_t (*)(nvmlDevice_t, int, unsigned int*)>(sym("nvmlDeviceGetMaxClockInfo"));
    x.reasons = reinterpret_cast<nvmlReturn_t (*)(nvmlDevice_t, unsigned long long*)>(
        sym("nvmlDeviceGetCurrentClocksEventReasons"));
    if (x.reasons == nullptr)
      x.reasons = reinterpret_cast<nvmlReturn_t (*)(nvmlDevice_t, unsigned long long*)>(
          sym("nvmlDeviceGetCurrentClocksThrottleReasons"));
    x.power = reinterpret_cast<nvmlReturn_t (*)(nvmlDevice_t, unsigned int*)>(sym("nvmlDeviceGetPowerUsage"));
    x.ok = x.init && x.by_bus_id && x.by_index && x.clock && x.max_clock && x.reasons && x.power && x.init() == 0;
    return x;
  }();
  return n;
}

}  // namespace

Sampler::Sampler(const std::string& gpu, int interval_us) : interval_us_(interval_us > 0 ? interval_us : 1000) {
  Nvml& n = nvml();
  if (!n.ok) {
    error_ = "NVML unavailable";
    return;
  }
  nvmlReturn_t r = gpu.find(':') != std::string::npos ? n.by_bus_id(gpu.c_str(), &dev_)
                                                       : n.by_index(static_cast<unsigned>(std::stoi(gpu)), &dev_);
  if (r != 0) {
    error_ = "no NVML device " + gpu;
    dev_ = nullptr;
  }
}

Sampler::~Sampler() { stop(); }

void Sampler::start() {
  if (dev_ == nullptr || thread_.joinable()) return;
  stop_.store(false);
  thread_ = std::thread([this] {
    Nvml& n = nvml();
    // the clock and the event reasons every sample; the maximum clock and
    // the power (slower queries) on every 16th, carried in between
    unsigned int smax = 0, power = 0;
    for (std::uint64_t k = 0; !stop_.load(); ++k) {
      Sample s;
      s.t_us = std::chrono::duration_cast<std::chrono::microseconds>(
                   std::chrono::steady_clock::now().time_since_epoch())
                   .count();
      unsigned int v = 0;
      if (n.clock(dev_, kNvmlClockSm, &v) == 0) s.sm_mhz = v;
      unsigned long long rs = 0;
      if (n.reasons(dev_, &rs) == 0) s.reasons = rs;
      if (k % 16 == 0) {
        if (n.max_clock(dev_, kNvmlClockSm, &v) == 0) smax = v;
        if (n.power(dev_, &v) == 0) power = v;
      }
      s.sm_max_mhz = smax;
      s.power_mw = power;
      {
        std::lock_guard<std::mutex> lk(mu_);
        samples_.push_back(s);
      }
      std::this_thread::sleep_for(std::chrono::microseconds(interval_us_));
    }
  });
}

std::vector<Sample> Sampler::stop() {
  if (thread_.joinable()) {
    stop_.store(true);
    thread_.join();
  }
  std::lock_guard<std::mutex> lk(mu_);
  return samples_;
}

}  // namespace clocks
}  // namespace commux
