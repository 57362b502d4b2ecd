// Host-side checks of the pull kernel's copy descriptors; no GPU needed.
//
//  1. FastDiv (the multiply-and-shift division the kernel uses for its index
//     walk) against exact division, for every divisor up to 70000, for the
//     powers of two and their neighbours, and for random large divisors, at
//     numerators around multiples of the divisor and at the ends of the range.
//  2. refine() + emit_descs() for random strided views (sliced, permuted,
//     broadcast-free; element sizes 1 to 16 bytes; misaligned bases): the
//     descriptors are walked the way the kernel walks them (row cache, FastDiv,
//     32-bit strides unless the descriptor is marked wide), and the resulting
//     (source, destination) element pairs must equal a brute-force enumeration
//     of the two views, each pair exactly once; check_desc() must accept them.
//  3. A layout of more than 2^30 units is split into several descriptors whose
//     unit counts and start offsets tile it.
//  4. The allocation-free entry point's planner (noalloc_plan.hpp) on random
//     views, negative strides and 16-byte elements included, with small caps
//     on the units per descriptor so that copies split into many descriptors:
//     the walked descriptors must cover each element pair exactly once, and
//     a copy needing more descriptors than the static scratch holds must be
//     rejected.
//
//   test_layout [iterations]    exit code 0 when every check passes

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <set>
#include <utility>
#include <vector>

#include "layout.hpp"
#include "noalloc_plan.hpp"

using commux::cuda::Dim;
using commux::cuda::FastDiv;
using commux::cuda::PullDesc;
using commux::cuda::kMaxPullDims;

namespace {

int g_fail = 0;

void fail(const char* what) {
  if (++g_fail <= 20) std::printf("FAIL %s\n", what);
}

// the kernel's FastDiv::div, on the host (__umulhi is the high word of the
// 64-bit product)
std::uint32_t host_div(const FastDiv& f, std::uint32_t n) {
  if (f.d == 1) return n;
  return static_cast<std::uint32_t>((static_cast<std::uint64_t>(n) * f.mul) >> 32) >> f.shr;
}

void check_fastdiv(std::mt19937_64& rng) {
  std::vector<std::uint32_t> divisors;
  for (std::uint32_t d = 1; d <= 70000; ++d) divisors.push_back(d);
  for (int k = 1; k < 31; ++k)
    for (std::int64_t e : {-1, 0, 1}) divisors.push_back(static_cast<std::uint32_t>((1ll << k) + e));
  for (int k = 0; k < 4000; ++k) divisors.push_back(1 + static_cast<std::uint32_t>(rng() % 0x7FFFFFFFu));
  const std::uint32_t nmax = 0x7FFFFFFFu;  // the kernel divides numerators below 2^31
  for (std::uint32_t d : divisors) {
    if (d == 0 || d > nmax) continue;
    FastDiv f(d);
    auto one = [&](std::uint32_t n) {
      if (n > nmax) return;
      if (host_div(f, n) != n / d) {
        char buf[96];
        std::snprintf(buf, sizeof(buf), "FastDiv(%u): %u / %u gave %u", d, n, d, host_div(f, n));
        fail(buf);
      }
    };
    for (std::uint32_t n : {0u, 1u, d - 1, d, d + 1, nmax, nmax - 1, nmax - d}) one(n);
    const std::uint32_t top = nmax / d;
    for (std::uint32_t q : {top, top - 1, top / 2, 1u, 2u, 3u}) {
      const std::uint64_t base = static_cast<std::uint64_t>(q) * d;
      for (std::int64_t e : {-1, 0, 1})
        if (static_cast<std::int64_t>(base) + e >= 0 && base + e <= nmax)
          one(static_cast<std::uint32_t>(base + e));
    }
    for (int k = 0; k < 8; ++k) one(static_cast<std::uint32_t>(rng() % (static_cast<std::uint64_t>(nmax) + 1)));
  }
}

// A random view: sizes, element strides, element offset of its first element
// inside a buffer of `extent` elements.
struct View {
  std::vector<std::int64_t> sizes, strides;
  std::int64_t offset = 0, extent = 0;
};

View random_view(const std::vector<std::int64_t>& shape, std::mt19937_64& rng) {
  const int nd = static_cast<int>(shape.size());
  // a parent buffer with room for a step and an offset per dim, dims permuted
  std::vector<std::int64_t> step(nd), off(nd), parent(nd);
  for (int k = 0; k < nd; ++k) {
    step[k] = 1 + static_cast<std::int64_t>(rng() % 3);
    off[k] = static_cast<std::int64_t>(rng() % 3);
    parent[k] = off[k] + (shape[k] - 1) * step[k] + 1 + static_cast<std::int64_t>(rng() % 2);
  }
  std::vector<int> order(nd);
  for (int k = 0; k < nd; ++k) order[k] = k;
  std::shuffle(order.begin(), order.end(), rng);  // order[0] is the outermost parent dim
  std::vector<std::int64_t> pstride(nd);
  std::int64_t s = 1;
  for (int k = nd - 1; k >= 0; --k) {
    pstride[order[k]] = s;
    s *= parent[order[k]];
  }
  View v;
  v.sizes = shape;
  v.strides.resize(nd);
  v.offset = 0;
  for (int k = 0; k < nd; ++k) {
    v.strides[k] = pstride[k] * step[k];
    v.offset += off[k] * pstride[k];
  }
  v.extent = s;
  return v;
}

// every element of the shape, row-major: (source, destination) element offsets
std::vector<std::pair<std::int64_t, std::int64_t>> brute_pairs(const View& a, const View& b) {
  std::vector<std::pair<std::int64_t, std::int64_t>> out;
  const int nd = static_cast<int>(a.sizes.size());
  std::vector<std::int64_t> idx(nd, 0);
  std::int64_t n = 1;
  for (auto x : a.sizes) n *= x;
  for (std::int64_t e = 0; e < n; ++e) {
    std::int64_t so = a.offset, dof = b.offset;
    for (int k = 0; k < nd; ++k) {
      so += idx[k] * a.strides[k];
      dof += idx[k] * b.strides[k];
    }
    out.push_back({so, dof});
    for (int k = nd - 1; k >= 0; --k) {
      if (++idx[k] < a.sizes[k]) break;
      idx[k] = 0;
    }
  }
  return out;
}

// The kernel's walk of one descriptor: byte offsets of every unit.
void walk(const PullDesc& d, std::vector<std::pair<std::int64_t, std::int64_t>>& units_out) {
  constexpr int in = kMaxPullDims - 1;
  for (std::uint32_t u = 0; u < d.units; ++u) {
    const std::uint32_t row = host_div(d.div[in], u);
    const std::uint32_t col = u - row * d.div[in].d;
    std::uint32_t rem = row;
    std::int64_t rso = 0, rdo = 0;
    for (int i = in - 1; i >= 1; --i) {
      const std::uint32_t q = host_div(d.div[i], rem);
      const std::uint32_t r = rem - q * d.div[i].d;
      if (d.wide) {
        rso += static_cast<std::int64_t>(r) * d.sst[i];
        rdo += static_cast<std::int64_t>(r) * d.dstr[i];
      } else {
        rso += static_cast<std::int64_t>(r) * static_cast<std::int32_t>(d.sst[i]);
        rdo += static_cast<std::int64_t>(r) * static_cast<std::int32_t>(d.dstr[i]);
      }
      rem = q;
    }
    const std::int64_t s0 = d.wide ? d.sst[0] : static_cast<std::int32_t>(d.sst[0]);
    const std::int64_t d0 = d.wide ? d.dstr[0] : static_cast<std::int32_t>(d.dstr[0]);
    const std::int64_t sin = d.wide ? d.sst[in] : static_cast<std::int32_t>(d.sst[in]);
    const std::int64_t din = d.wide ? d.dstr[in] : static_cast<std::int32_t>(d.dstr[in]);
    rso += static_cast<std::int64_t>(rem) * s0;
    rdo += static_cast<std::int64_t>(rem) * d0;
    units_out.push_back({rso + static_cast<std::int64_t>(col) * sin, rdo + static_cast<std::int64_t>(col) * din});
  }
}

void check_layouts(std::mt19937_64& rng, int iters) {
  const std::int64_t elems[] = {1, 2, 4, 8, 16};
  for (int it = 0; it < iters; ++it) {
    const int nd = 1 + static_cast<int>(rng() % 4);
    std::vector<std::int64_t> shape(nd);
    for (auto& x : shape) x = 1 + static_cast<std::int64_t>(rng() % 9);
    if (rng() % 4 == 0) shape[nd - 1] = 1 + static_cast<std::int64_t>(rng() % 70);  // long rows
    const View a = random_view(shape, rng);
    View b = random_view(shape, rng);
    if (rng() % 3 == 0) {  // contiguous destination
      std::int64_t s = 1;
      for (int k = nd - 1; k >= 0; --k) {
        b.strides[k] = s;
        s *= shape[k];
      }
      b.offset = 0;
      b.extent = s;
    }
    const std::int64_t elem = elems[rng() % 5];
    // byte bases: 256-aligned, or shifted to test the unit choice
    const std::int64_t sbase = 4096 + (rng() % 2 ? 0 : elem * static_cast<std::int64_t>(rng() % 3));
    const std::int64_t dbase = 1 << 20;
    std::vector<std::int64_t> sz(shape), ss(a.strides), ds(b.strides);
    auto da = commux::cuda::dims_of(sz.data(), ss.data(), nd);
    auto db = commux::cuda::dims_of(sz.data(), ds.data(), nd);
    std::vector<Dim> dims;
    if (!commux::cuda::refine(da, db, dims)) {
      fail("refine rejected two views of one shape");
      continue;
    }
    if (dims.size() > static_cast<std::size_t>(kMaxPullDims)) continue;  // staged by the transport
    const char* sp = reinterpret_cast<const char*>(sbase + a.offset * elem);
    char* dp = reinterpret_cast<char*>(dbase + b.offset * elem);
    std::vector<PullDesc> descs;
    commux::cuda::emit_descs(sp, dp, dims, elem, descs);
    std::vector<std::pair<std::int64_t, std::int64_t>> got;
    for (auto& d : descs) {
      try {
        commux::cuda::check_desc(d, sbase, sbase + a.extent * elem, dbase, dbase + b.extent * elem);
      } catch (...) {
        fail("check_desc rejected a descriptor inside its buffers");
      }
      if (d.unit % elem != 0 && elem % d.unit != 0) fail("unit and element size disagree");
      if (reinterpret_cast<std::uintptr_t>(d.src) % d.unit || reinterpret_cast<std::uintptr_t>(d.dst) % d.unit)
        fail("a descriptor's base is not aligned to its unit");
      std::vector<std::pair<std::int64_t, std::int64_t>> units;
      walk(d, units);
      const std::int64_t s0 = reinterpret_cast<std::int64_t>(d.src) - sbase;
      const std::int64_t d0 = reinterpret_cast<std::int64_t>(d.dst) - dbase;
      for (auto& u : units)
        for (std::int64_t k = 0; k < d.unit; k += std::min<std::int64_t>(elem, d.unit)) {
          // one unit covers unit/elem elements (or a part of one element)
          const std::int64_t sb = s0 + u.first + k, db2 = d0 + u.second + k;
          if (elem <= d.unit) {
            if (sb % elem || db2 % elem) fail("a unit splits an element");
            got.push_back({sb / elem, db2 / elem});
          } else if (k == 0 && (sb % elem) == 0) {
            got.push_back({sb / elem, db2 / elem});
          }
        }
    }
    auto want = brute_pairs(a, b);
    std::sort(want.begin(), want.end());
    std::sort(got.begin(), got.end());
    if (got != want) {
      char buf[160];
      std::snprintf(buf, sizeof(buf), "iteration %d: %zu element pairs walked, %zu expected (nd %d, elem %lld)", it,
                    got.size(), want.size(), nd, static_cast<long long>(elem));
      fail(buf);
    }
  }
}

void check_split() {
  // 3 x 2^30 + 5 elements of 1 byte in a 2-D layout: rows of 2^29 + 1 units
  std::vector<Dim> dims{{6, (1ll << 29) + 7, (1ll << 29) + 1}, {(1ll << 29) + 1, 1, 1}};
  std::vector<PullDesc> descs;
  const char* sp = reinterpret_cast<const char*>(std::intptr_t{1} << 40);
  char* dp = reinterpret_cast<char*>(std::intptr_t{1} << 42);
  commux::cuda::emit_descs(sp, dp, dims, 1, descs);
  std::int64_t units = 0, rows = 0;
  for (auto& d : descs) {
    units += d.units;
    if (d.units > (1u << 30)) fail("a descriptor holds more than 2^30 units");
    const std::int64_t expect_src = reinterpret_cast<std::int64_t>(sp) + rows * ((1ll << 29) + 7);
    if (reinterpret_cast<std::int64_t>(d.src) != expect_src) fail("split descriptors do not tile the source");
    rows += d.div[kMaxPullDims - 2].d;
  }
  if (units != 6 * ((1ll << 29) + 1)) fail("split descriptors do not cover every unit");
  if (descs.size() < 2) fail("a layout above 2^30 units was not split");
}

void check_noalloc_plan(std::mt19937_64& rng, int iters) {
  namespace na = commux::cuda::noalloc;
  const std::int64_t elems[] = {1, 2, 4, 8, 16};
  static PullDesc descs[na::kDescs];
  for (int it = 0; it < iters; ++it) {
    const int nd = 1 + static_cast<int>(rng() % 5);
    std::vector<std::int64_t> shape(nd);
    for (auto& x : shape) x = 1 + static_cast<std::int64_t>(rng() % 7);
    View a = random_view(shape, rng), b = random_view(shape, rng);
    // negative strides: walk some dims backwards (the pointer moves to the
    // dim's last element)
    for (View* v : {&a, &b})
      for (int k = 0; k < nd; ++k)
        if (rng() % 4 == 0) {
          v->offset += (shape[k] - 1) * v->strides[k];
          v->strides[k] = -v->strides[k];
        }
    const std::int64_t elem = elems[rng() % 5];
    const std::int64_t sbase = 1 << 16, dbase = 1 << 24;
    char* sp = reinterpret_cast<char*>(sbase + a.offset * elem);
    char* dp = reinterpret_cast<char*>(dbase + b.offset * elem);
    const std::int64_t cap = 1 + static_cast<std::int64_t>(rng() % 40);
    na::Plan plan;
    char err[256];
    const int rc = na::plan_copy(dp, b.strides.data(), sp, a.strides.data(), shape.data(), nd,
                                 static_cast<int>(elem), nullptr, descs, plan, err, sizeof(err), cap);
    if (rc == CMX_NOALLOC_ELAYOUT || rc == CMX_NOALLOC_ETOOBIG) continue;  // rejected before launch
    if (rc != CMX_NOALLOC_OK) {
      fail(err);
      continue;
    }
    std::vector<std::pair<std::int64_t, std::int64_t>> got;
    for (std::uint32_t i = 0; i < plan.ndesc; ++i) {
      const PullDesc& d = descs[i];
      if (d.units > static_cast<std::uint64_t>(cap)) fail("noalloc: a descriptor exceeds the unit cap");
      if (d.counter_idx != i) fail("noalloc: counter slots are not one per descriptor");
      std::vector<std::pair<std::int64_t, std::int64_t>> units;
      walk(d, units);
      const std::int64_t s0 = reinterpret_cast<std::int64_t>(d.src) - sbase;
      const std::int64_t d0 = reinterpret_cast<std::int64_t>(d.dst) - dbase;
      for (auto& u : units)
        for (std::int64_t k = 0; k < d.unit; k += elem) {
          const std::int64_t sb = s0 + u.first + k, db2 = d0 + u.second + k;
          if (sb % elem || db2 % elem) fail("noalloc: a unit splits an element");
          got.push_back({sb / elem, db2 / elem});
        }
    }
    auto want = brute_pairs(a, b);
    std::sort(want.begin(), want.end());
    std::sort(got.begin(), got.end());
    if (got != want) {
      char buf[160];
      std::snprintf(buf, sizeof(buf),
                    "noalloc iteration %d: %zu pairs walked, %zu expected (nd %d, elem %lld, cap %lld)", it,
                    got.size(), want.size(), nd, static_cast<long long>(elem), static_cast<long long>(cap));
      fail(buf);
    }
  }
  // more descriptors than the scratch has counters: rejected
  std::int64_t sizes[2] = {na::kDescs + 1, 4}, ss[2] = {8, 1}, ds[2] = {4, 1};
  na::Plan plan;
  char err[256];
  const int rc = na::plan_copy(reinterpret_cast<void*>(1 << 20), ds, reinterpret_cast<void*>(1 << 16), ss, sizes, 2,
                               4, nullptr, descs, plan, err, sizeof(err), 1);
  if (rc != CMX_NOALLOC_ETOOBIG) fail("noalloc: a copy needing 65 descriptors was not rejected");
}

}  // namespace

int main(int argc, char** argv) {
  const int iters = argc > 1 ? std::atoi(argv[1]) : 4000;
  std::mt19937_64 rng(20261202);
  check_fastdiv(rng);
  check_layouts(rng, iters);
  check_split();
  check_noalloc_plan(rng, iters);
  if (g_fail == 0) std::printf("ALL LAYOUT CHECKS PASSED\n");
  else std::printf("%d failure(s)\n", g_fail);
  return g_fail == 0 ? 0 : 1;
}
