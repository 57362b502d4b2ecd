#pragma once

// Diagnostics: COMMUX_DEBUG=WARN|INFO|TRACE prints to stderr with a rank
// prefix (default: warnings only), and COMMUX_TRACE=1 opens an NVTX range
// per backend operation, for Nsight timelines.

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#if defined(__has_include)
#if __has_include(<nvtx3/nvToolsExt.h>)
#include <nvtx3/nvToolsExt.h>
#define COMMUX_HAVE_NVTX 1
#endif
#endif

namespace commux {

enum class LogLevel : int { Warn = 1, Info = 2, Trace = 3 };

inline int log_level() {
  static const int lvl = [] {
    const char* v = std::getenv("COMMUX_DEBUG");
    if (v == nullptr || *v == '\0') return 1;
    if (!std::strcmp(v, "TRACE") || !std::strcmp(v, "trace")) return 3;
    if (!std::strcmp(v, "INFO") || !std::strcmp(v, "info") || !std::strcmp(v, "1")) return 2;
    if (!std::strcmp(v, "0") || !std::strcmp(v, "NONE") || !std::strcmp(v, "none")) return 0;
    return 1;
  }();
  return lvl;
}

inline bool log_on(LogLevel l) { return log_level() >= static_cast<int>(l); }

inline void logf(LogLevel l, int rank, const char* fmt, ...) {
  if (!log_on(l)) return;
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  std::fprintf(stderr, "[commux %s rank %d] %s\n",
               l == LogLevel::Warn ? "WARN" : l == LogLevel::Info ? "INFO" : "TRACE", rank, buf);
}

inline bool trace_on() {
  static const bool on = [] {
    const char* v = std::getenv("COMMUX_TRACE");
    return v != nullptr && *v != '\0' && *v != '0';
  }();
  return on;
}

// RAII NVTX range (no-op unless COMMUX_TRACE=1 and NVTX headers were found).
class TraceRange {
 public:
  explicit TraceRange(const char* name) {
#ifdef COMMUX_HAVE_NVTX
    if (trace_on()) {
      nvtxRangePushA(name);
      active_ = true;
    }
#else
    (void)name;
#endif
  }
  ~TraceRange() {
#ifdef COMMUX_HAVE_NVTX
    if (active_) nvtxRangePop();
#endif
  }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;

 private:
  bool active_ = false;
};

}  // namespace commux
