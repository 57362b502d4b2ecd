#pragma once

// Host-side construction of the pull kernel's copy descriptors: two tensor
// layouts with equal element counts are refined into one common walk,
// dims contiguous in both are merged, and the walk becomes descriptors with
// the widest vector unit the alignment allows. Pure host code (no CUDA
// runtime or driver calls), so it is also tested on machines without a GPU.

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <utility>
#include <vector>

#include "cuda_common.hpp"

namespace commux {
namespace cuda {
namespace {

constexpr std::uint64_t kMaxUnitsPerDesc = 1ull << 30;

// A tensor dimension as (size, src stride, dst stride), strides in elements
// or bytes depending on the stage.
struct Dim {
  std::int64_t size, ss, ds;
};

// Refine two shapes with equal element counts into one common shape (split
// dims where they differ) so a single index walks both. Returns false when no
// common refinement exists (e.g. sizes 6 and 4 facing each other).
bool refine(const std::vector<std::pair<std::int64_t, std::int64_t>>& a,
            const std::vector<std::pair<std::int64_t, std::int64_t>>& b, std::vector<Dim>& out) {
  out.clear();
  int i = static_cast<int>(a.size()) - 1, j = static_cast<int>(b.size()) - 1;
  if (i < 0 || j < 0) return false;
  std::int64_t ra = a[i].first, rb = b[j].first, sa = a[i].second, sb = b[j].second;
  while (i >= 0 && j >= 0) {
    std::int64_t m = std::min(ra, rb);
    if (m <= 0 || ra % m || rb % m) return false;
    out.push_back({m, sa, sb});
    if (ra == m) {
      if (--i >= 0) {
        ra = a[i].first;
        sa = a[i].second;
      }
    } else {
      ra /= m;
      sa *= m;
    }
    if (rb == m) {
      if (--j >= 0) {
        rb = b[j].first;
        sb = b[j].second;
      }
    } else {
      rb /= m;
      sb *= m;
    }
  }
  if (i >= 0 || j >= 0) return false;
  std::reverse(out.begin(), out.end());
  // merge dims that are contiguous in both
  std::vector<Dim> m;
  for (auto& d : out) {
    if (!m.empty() && m.back().ss == d.size * d.ss && m.back().ds == d.size * d.ds) {
      m.back().size *= d.size;
      m.back().ss = d.ss;
      m.back().ds = d.ds;
    } else {
      m.push_back(d);
    }
  }
  out.swap(m);
  return true;
}

std::vector<std::pair<std::int64_t, std::int64_t>> dims_of(const std::int64_t* sizes,
                                                           const std::int64_t* strides, int nd) {
  std::vector<std::pair<std::int64_t, std::int64_t>> v;
  for (int k = 0; k < nd; ++k)
    if (sizes[k] != 1) v.push_back({sizes[k], strides[k]});
  if (v.empty()) v.push_back({1, 1});
  return v;
}

// Turn common dims (element strides) into pull descriptors with the widest
// vector unit the alignment allows; appends to `out`.
void emit_descs(const char* sp, char* dp, std::vector<Dim> dims, std::int64_t elem,
                std::vector<PullDesc>& out) {
  // element strides -> byte strides
  for (auto& d : dims) {
    d.ss *= elem;
    d.ds *= elem;
  }
  std::int64_t unit = elem;
  Dim& in = dims.back();
  if (in.ss == elem && in.ds == elem) {
    std::int64_t inner_bytes = in.size * elem;
    for (std::int64_t u : {16, 8, 4, 2, 1}) {
      bool ok = inner_bytes % u == 0 && reinterpret_cast<std::uintptr_t>(sp) % u == 0 &&
                reinterpret_cast<std::uintptr_t>(dp) % u == 0;
      for (std::size_t k = 0; ok && k + 1 < dims.size(); ++k)
        ok = dims[k].ss % u == 0 && dims[k].ds % u == 0;
      if (ok) {
        unit = u;
        break;
      }
    }
    in.size = inner_bytes / unit;
    in.ss = unit;
    in.ds = unit;
    // a row of exactly one unit (e.g. a 16-byte x-face row): the row dim
    // adds nothing but a division per unit
    if (in.size == 1 && dims.size() > 1) dims.pop_back();
  } else if (!(elem == 1 || elem == 2 || elem == 4 || elem == 8 || elem == 16)) {
    throw std::runtime_error("commux: unsupported element size for a strided device copy");
  }
  if (dims.size() > static_cast<std::size_t>(kMaxPullDims))
    throw std::runtime_error("layout");
  // split along the outermost dim so every descriptor has < 2^30 units
  std::int64_t per0 = 1;
  for (std::size_t k = 1; k < dims.size(); ++k) per0 *= dims[k].size;
  if (per0 > static_cast<std::int64_t>(kMaxUnitsPerDesc))
    throw std::runtime_error("commux: device message row too large");
  std::int64_t step0 = std::max<std::int64_t>(1, static_cast<std::int64_t>(kMaxUnitsPerDesc) / per0);
  for (std::int64_t s0 = 0; s0 < dims[0].size; s0 += step0) {
    std::int64_t n0 = std::min(step0, dims[0].size - s0);
    PullDesc d{};
    d.src = sp + s0 * dims[0].ss;
    d.dst = dp + s0 * dims[0].ds;
    d.ndim = static_cast<std::uint32_t>(dims.size());
    d.unit = static_cast<std::uint32_t>(unit);
    const int off = kMaxPullDims - static_cast<int>(dims.size());
    for (int k = 0; k < kMaxPullDims; ++k) {
      d.div[k] = FastDiv(1);
      d.sst[k] = 0;
      d.dstr[k] = 0;
    }
    std::int64_t units = 1;
    for (std::size_t k = 0; k < dims.size(); ++k) {
      std::int64_t sz = k == 0 ? n0 : dims[k].size;
      d.div[off + k] = FastDiv(static_cast<std::uint32_t>(sz));
      d.sst[off + k] = dims[k].ss;
      d.dstr[off + k] = dims[k].ds;
      units *= sz;
    }
    d.units = static_cast<std::uint32_t>(units);
    d.nchunks = static_cast<std::uint32_t>(std::max<std::int64_t>(1, (units + kChunkUnits - 1) / kChunkUnits));
    // the kernel's common walk holds strides in 32 bits
    constexpr std::int64_t lim = std::int64_t{1} << 31;
    for (int k = 0; k < kMaxPullDims; ++k)
      if (d.sst[k] >= lim || d.sst[k] <= -lim || d.dstr[k] >= lim || d.dstr[k] <= -lim) d.wide = 1;
    out.push_back(d);
  }
}

// Host-side bounds check of every descriptor before launch: the bytes a
// descriptor touches must lie inside the source allocation (the IPC mapping)
// and the destination storage. A layout bug then raises here instead of
// reaching the GPU as an out-of-bounds access. The bounds-check build also
// hands the same limits to the kernel, which checks every unit it copies.
void check_desc(PullDesc& d, std::uintptr_t src_lo, std::uintptr_t src_hi,
                std::uintptr_t dst_lo, std::uintptr_t dst_hi) {
  if (d.units == 0) return;
  std::int64_t s_min = 0, s_max = 0, d_min = 0, d_max = 0;
  for (int k = 0; k < kMaxPullDims; ++k) {
    std::int64_t ext = static_cast<std::int64_t>(d.div[k].d) - 1;
    std::int64_t a = ext * d.sst[k], b = ext * d.dstr[k];
    (a < 0 ? s_min : s_max) += a;
    (b < 0 ? d_min : d_max) += b;
  }
  auto sp = reinterpret_cast<std::intptr_t>(d.src), dp = reinterpret_cast<std::intptr_t>(d.dst);
  bool ok = sp + s_min >= static_cast<std::intptr_t>(src_lo) &&
            sp + s_max + static_cast<std::intptr_t>(d.unit) <= static_cast<std::intptr_t>(src_hi) &&
            dp + d_min >= static_cast<std::intptr_t>(dst_lo) &&
            dp + d_max + static_cast<std::intptr_t>(d.unit) <= static_cast<std::intptr_t>(dst_hi);
  if (!ok)
    throw std::runtime_error("commux: internal error, a copy descriptor leaves its buffers "
                             "(layout bug caught before launch)");
#if defined(COMMUX_DEVICE_CHECKS)
  d.src_lo = static_cast<std::intptr_t>(src_lo) - sp;
  d.src_hi = static_cast<std::intptr_t>(src_hi) - sp;
  d.dst_lo = static_cast<std::intptr_t>(dst_lo) - dp;
  d.dst_hi = static_cast<std::intptr_t>(dst_hi) - dp;
#endif
}

}  // namespace
}  // namespace cuda
}  // namespace commux
