#include "reduce_cpu.hpp"

#include <c10/util/BFloat16.h>
#include <c10/util/Half.h>

#include <algorithm>
#include <vector>

namespace commux {

namespace {

template <typename T>
inline T apply(RedOp op, T a, T b) {
  switch (op) {
    case RedOp::Sum:
    case RedOp::Avg:
      return a + b;
    case RedOp::Prod:
      return a * b;
    case RedOp::Min:
      return b < a ? b : a;
    case RedOp::Max:
      return b > a ? b : a;
  }
  return a;
}

// T: storage type, A: accumulation type
template <typename T, typename A>
void fold_impl(RedOp op, void* out_v, const void* const* bufs, int nbufs, std::int64_t n,
               int nranks) {
  T* out = static_cast<T*>(out_v);
  constexpr std::int64_t kBlock = 2048;
  A acc[kBlock];
  for (std::int64_t b0 = 0; b0 < n; b0 += kBlock) {
    std::int64_t m = std::min(kBlock, n - b0);
    const T* s0 = static_cast<const T*>(bufs[0]) + b0;
    for (std::int64_t i = 0; i < m; ++i) acc[i] = static_cast<A>(s0[i]);
    for (int p = 1; p < nbufs; ++p) {
      const T* sp = static_cast<const T*>(bufs[p]) + b0;
      switch (op) {
        case RedOp::Sum:
        case RedOp::Avg:
          for (std::int64_t i = 0; i < m; ++i) acc[i] = acc[i] + static_cast<A>(sp[i]);
          break;
        case RedOp::Prod:
          for (std::int64_t i = 0; i < m; ++i) acc[i] = acc[i] * static_cast<A>(sp[i]);
          break;
        case RedOp::Min:
          for (std::int64_t i = 0; i < m; ++i) {
            A v = static_cast<A>(sp[i]);
            acc[i] = v < acc[i] ? v : acc[i];
          }
          break;
        case RedOp::Max:
          for (std::int64_t i = 0; i < m; ++i) {
            A v = static_cast<A>(sp[i]);
            acc[i] = v > acc[i] ? v : acc[i];
          }
          break;
      }
    }
    if (op == RedOp::Avg) {
      A d = static_cast<A>(nranks);
      for (std::int64_t i = 0; i < m; ++i) acc[i] = acc[i] / d;
    }
    T* o = out + b0;
    for (std::int64_t i = 0; i < m; ++i) o[i] = static_cast<T>(acc[i]);
  }
}

void fold_bool(RedOp op, void* out_v, const void* const* bufs, int nbufs, std::int64_t n) {
  auto* out = static_cast<bool*>(out_v);
  bool any_op = op == RedOp::Sum || op == RedOp::Max;
  for (std::int64_t i = 0; i < n; ++i) {
    bool a = static_cast<const bool*>(bufs[0])[i];
    for (int p = 1; p < nbufs; ++p) {
      bool b = static_cast<const bool*>(bufs[p])[i];
      a = any_op ? (a || b) : (a && b);
    }
    out[i] = a;
  }
}

bool is_floating(at::ScalarType dt) {
  return dt == at::kFloat || dt == at::kDouble || dt == at::kHalf || dt == at::kBFloat16;
}

}  // namespace

std::string check_reduce(at::ScalarType dt, RedOp op) {
  switch (dt) {
    case at::kFloat:
    case at::kDouble:
    case at::kHalf:
    case at::kBFloat16:
    case at::kChar:
    case at::kByte:
    case at::kShort:
    case at::kInt:
    case at::kLong:
    case at::kBool:
      break;
    default:
      return std::string("unsupported ReduceOp input dtype ") + c10::toString(dt);
  }
  if (op == RedOp::Avg && !is_floating(dt))
    return std::string("unsupported ReduceOp AVG for integer dtype ") + c10::toString(dt);
  return "";
}

void fold_ranks(at::ScalarType dt, RedOp op, void* out, const void* const* bufs, int nbufs,
                std::int64_t n, int nranks) {
  switch (dt) {
    case at::kFloat:
      return fold_impl<float, float>(op, out, bufs, nbufs, n, nranks);
    case at::kDouble:
      return fold_impl<double, double>(op, out, bufs, nbufs, n, nranks);
    case at::kHalf:
      return fold_impl<c10::Half, float>(op, out, bufs, nbufs, n, nranks);
    case at::kBFloat16:
      return fold_impl<c10::BFloat16, float>(op, out, bufs, nbufs, n, nranks);
    case at::kChar:
      return fold_impl<std::int8_t, std::int8_t>(op, out, bufs, nbufs, n, nranks);
    case at::kByte:
      return fold_impl<std::uint8_t, std::uint8_t>(op, out, bufs, nbufs, n, nranks);
    case at::kShort:
      return fold_impl<std::int16_t, std::int16_t>(op, out, bufs, nbufs, n, nranks);
    case at::kInt:
      return fold_impl<std::int32_t, std::int32_t>(op, out, bufs, nbufs, n, nranks);
    case at::kLong:
      return fold_impl<std::int64_t, std::int64_t>(op, out, bufs, nbufs, n, nranks);
    case at::kBool:
      return fold_bool(op, out, bufs, nbufs, n);
    default:
      TORCH_CHECK(false, "commux: unsupported ReduceOp input dtype ", dt);
  }
}

}  // namespace commux
