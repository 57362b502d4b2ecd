#pragma once

// Host reductions for the CPU collectives.
//
// Every collective folds the ranks' contributions in rank order,
// out = ((x0 op x1) op x2) ... op x_{P-1}, accumulating half-precision types
// in fp32 and rounding once, so every rank computes bit-identical results and
// a test can reproduce them exactly with the same fold. (The reference folds
// along a binomial tree with ATen ops, reference: src/process_group_ucx.cpp:
// 214-232 and :736-759; its order differs but is just as fixed.)

#include <ATen/core/Tensor.h>

#include <cstdint>
#include <string>

#include "../engine/engine.hpp"

namespace commux {

// Returns "" if (op, dtype) is supported, else an error message that starts
// with "unsupported ReduceOp" (checked on every rank before any message).
std::string check_reduce(at::ScalarType dt, RedOp op);

// out[i] = fold over p of bufs[p][i], i in [0, n). `out` may alias any of
// `bufs` (each element is read from every buffer before it is written). AVG
// divides the fold by `nranks` after summing.
void fold_ranks(at::ScalarType dt, RedOp op, void* out, const void* const* bufs,
                int nbufs, std::int64_t n, int nranks);

}  // namespace commux
