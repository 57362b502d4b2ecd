#pragma once

// Host-only planning of commux_strided_copy_noalloc: the caller's strided
// views become at most kNoAllocDescs pull descriptors, with no heap
// allocation (the descriptors go into caller-provided storage). Kept apart
// from the CUDA calls so the arithmetic (dim merging, vector-unit choice, the
// split of long copies into several descriptors) is tested on the CPU
// against a brute-force walk (tests/cpp/test_layout.cpp).

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "commux/noalloc.h"
#include "cuda_common.hpp"

namespace commux {
namespace cuda {
namespace noalloc {

constexpr int kDescs = 64;  // counters = copy descriptors per call
constexpr int kMaxInDims = 8;
constexpr std::int64_t kUnitsPerDesc = std::int64_t{1} << 30;
constexpr std::int64_t kMaxExtent = std::int64_t{1} << 40;  // sizes and strides, elements

using Wide = __int128;  // extents of hostile sizes x strides cannot overflow

struct NDim {
  std::int64_t size, ss, ds;  // elements, then bytes
};

inline int fail(char* err, std::size_t len, int code, const char* fmt, ...) {
  if (err != nullptr && len > 0) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(err, len, fmt, ap);
    va_end(ap);
  }
  return code;
}

// Byte extent [lo, hi) of a view (merged dims, byte strides) relative to its
// pointer; negative strides extend it below the pointer.
inline void span(const NDim* d, int n, bool src, std::int64_t unit, Wide& lo, Wide& hi) {
  lo = 0;
  hi = unit;
  for (int k = 0; k < n; ++k) {
    const Wide e = static_cast<Wide>(d[k].size - 1) * (src ? d[k].ss : d[k].ds);
    (e < 0 ? lo : hi) += e;
  }
}

struct Plan {
  NDim dims[kMaxPullDims];  // merged, byte strides, innermost in vector units
  int n = 0;
  std::int64_t unit = 0;    // bytes per vector unit
  std::uint32_t ndesc = 0;  // descriptors written (0: nothing to copy)
  std::uint32_t chunks = 0;
};

// Plans the copy of the `ndim`-dim view (sizes, element strides) at `src`
// into the same-shaped view at `dst`: descriptors d[0, plan.ndesc), each its
// own message counted into counter slot i and flagged at done_base + i.
// `units_per_desc` caps one descriptor (kUnitsPerDesc in production; tests
// pass small caps to exercise the split). Returns CMX_NOALLOC_OK or an error
// code with a message in err.
inline int plan_copy(void* dst, const std::int64_t* dst_strides, const void* src, const std::int64_t* src_strides,
                     const std::int64_t* sizes, int ndim, int elem_bytes, std::uint64_t* done_base, PullDesc* out,
                     Plan& plan, char* err, std::size_t err_len, std::int64_t units_per_desc = kUnitsPerDesc) {
  plan = Plan{};
  if (dst == nullptr || src == nullptr || sizes == nullptr || dst_strides == nullptr || src_strides == nullptr ||
      ndim < 0 || ndim > kMaxInDims)
    return fail(err, err_len, CMX_NOALLOC_EINVAL,
                "commux_strided_copy_noalloc: null pointer or ndim outside [0, %d]", kMaxInDims);
  const std::int64_t elem = elem_bytes;
  if (!(elem == 1 || elem == 2 || elem == 4 || elem == 8 || elem == 16))
    return fail(err, err_len, CMX_NOALLOC_EINVAL,
                "commux_strided_copy_noalloc: elem_bytes must be 1, 2, 4, 8 or 16 (got %d)", elem_bytes);
  if (reinterpret_cast<std::uintptr_t>(src) % elem || reinterpret_cast<std::uintptr_t>(dst) % elem)
    return fail(err, err_len, CMX_NOALLOC_EINVAL,
                "commux_strided_copy_noalloc: src and dst must be aligned to elem_bytes");

  // dims: drop size-1 dims, then merge neighbours contiguous in both views
  NDim d[kMaxInDims];
  int n = 0;
  for (int k = 0; k < ndim; ++k) {
    if (sizes[k] < 0) return fail(err, err_len, CMX_NOALLOC_EINVAL, "commux_strided_copy_noalloc: negative size");
    if (sizes[k] == 0) return CMX_NOALLOC_OK;  // nothing to copy
    if (sizes[k] == 1) continue;
    if (sizes[k] > kMaxExtent || src_strides[k] > kMaxExtent || src_strides[k] < -kMaxExtent ||
        dst_strides[k] > kMaxExtent || dst_strides[k] < -kMaxExtent)
      return fail(err, err_len, CMX_NOALLOC_ETOOBIG,
                  "commux_strided_copy_noalloc: too large, a size or stride exceeds 2^40 elements");
    NDim cur{sizes[k], src_strides[k], dst_strides[k]};
    if (n > 0 && static_cast<Wide>(d[n - 1].ss) == static_cast<Wide>(cur.size) * cur.ss &&
        static_cast<Wide>(d[n - 1].ds) == static_cast<Wide>(cur.size) * cur.ds) {
      if (d[n - 1].size > kMaxExtent / cur.size)
        return fail(err, err_len, CMX_NOALLOC_ETOOBIG, "commux_strided_copy_noalloc: view too large");
      d[n - 1] = NDim{d[n - 1].size * cur.size, cur.ss, cur.ds};
    } else {
      d[n++] = cur;
    }
  }
  if (n == 0) d[n++] = NDim{1, 1, 1};
  for (int k = 0; k < n; ++k) {
    d[k].ss *= elem;
    d[k].ds *= elem;
  }
  // widest vector unit: the innermost dim, when contiguous in both, becomes
  // a run of 16/8/4/2/1-byte units
  std::int64_t unit = elem;
  NDim& in = d[n - 1];
  if (in.ss == elem && in.ds == elem) {
    const std::int64_t inner = in.size * elem;
    for (std::int64_t u : {16, 8, 4, 2, 1}) {
      bool ok = inner % u == 0 && reinterpret_cast<std::uintptr_t>(src) % u == 0 &&
                reinterpret_cast<std::uintptr_t>(dst) % u == 0;
      for (int k = 0; ok && k + 1 < n; ++k) ok = d[k].ss % u == 0 && d[k].ds % u == 0;
      if (ok) {
        unit = u;
        break;
      }
    }
    in = NDim{inner / unit, unit, unit};
    if (in.size == 1 && n > 1) --n;
  }
  if (n > kMaxPullDims)
    return fail(err, err_len, CMX_NOALLOC_ELAYOUT,
                "commux_strided_copy_noalloc: %d dims remain after merging, at most %d are supported", n, kMaxPullDims);
  std::int64_t per0 = 1;
  for (int k = 1; k < n; ++k) {
    if (d[k].size > units_per_desc / per0)
      return fail(err, err_len, CMX_NOALLOC_ETOOBIG,
                  "commux_strided_copy_noalloc: too large, the dims inside the outermost one hold more "
                  "than %lld units of %lld bytes",
                  static_cast<long long>(units_per_desc), static_cast<long long>(unit));
    per0 *= d[k].size;
  }
  const std::int64_t step0 = units_per_desc / per0;
  const std::int64_t ndesc = (d[0].size + step0 - 1) / step0;
  if (ndesc > kDescs)
    return fail(err, err_len, CMX_NOALLOC_ETOOBIG,
                "commux_strided_copy_noalloc: too large, the copy needs %lld descriptors and the static "
                "scratch has counters for %d (at most %lld units of %lld bytes)",
                static_cast<long long>(ndesc), kDescs, static_cast<long long>(kDescs * units_per_desc),
                static_cast<long long>(unit));

  for (int k = 0; k < n; ++k) plan.dims[k] = d[k];
  plan.n = n;
  plan.unit = unit;
  // descriptors, one per slab of step0 outer rows, each its own message
  const int off = kMaxPullDims - n;
  std::uint32_t chunks = 0;
  std::uint32_t i = 0;
  for (std::int64_t s0 = 0; s0 < d[0].size; s0 += step0, ++i) {
    const std::int64_t n0 = d[0].size - s0 < step0 ? d[0].size - s0 : step0;
    PullDesc& x = out[i];
    x = PullDesc{};
    x.src = static_cast<const char*>(src) + s0 * d[0].ss;
    x.dst = static_cast<char*>(dst) + s0 * d[0].ds;
    x.ndim = static_cast<std::uint32_t>(n);
    x.unit = static_cast<std::uint32_t>(unit);
    std::int64_t units = 1;
    for (int k = 0; k < n; ++k) {
      const std::int64_t sz = k == 0 ? n0 : d[k].size;
      x.div[off + k] = FastDiv(static_cast<std::uint32_t>(sz));
      x.sst[off + k] = d[k].ss;
      x.dstr[off + k] = d[k].ds;
      units *= sz;
    }
    x.units = static_cast<std::uint32_t>(units);
    for (int k = 0; k < kMaxPullDims; ++k) {
      constexpr std::int64_t lim = std::int64_t{1} << 31;
      if (x.sst[k] >= lim || x.sst[k] <= -lim || x.dstr[k] >= lim || x.dstr[k] <= -lim) x.wide = 1;
    }
    x.nchunks = static_cast<std::uint32_t>((units + kChunkUnits - 1) / kChunkUnits);
    x.chunk0 = chunks;
    x.msg_chunks = x.nchunks;
    x.counter_idx = i;
    x.done = done_base == nullptr ? nullptr : done_base + i;
    x.done_val = 1;
    chunks += x.nchunks;
  }
  plan.ndesc = i;
  plan.chunks = chunks;
  return CMX_NOALLOC_OK;
}

}  // namespace noalloc
}  // namespace cuda
}  // namespace commux
