#pragma once

// Host side of the device collectives: symmetric workspace bootstrap over the
// c10d Store, algorithm choice per message size, stream ordering, results.

#include <ATen/ATen.h>

#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "coll_args.hpp"
#include "nvls.hpp"
#include "transport.hpp"

namespace commux {
namespace cuda {

class CollImpl {
 public:
  CollImpl(CudaTransport* tr, int dev);
  ~CollImpl();

  bool shared_gpu() const { return shared_gpu_; }
  DevCollPtr allreduce(std::vector<at::Tensor>& ts, RedOp op);
  DevCollPtr reduce(std::vector<at::Tensor>& ts, RedOp op, int root);
  DevCollPtr broadcast(std::vector<at::Tensor>& ts, int root);
  DevCollPtr allgather(at::Tensor& out, const at::Tensor& in);
  DevCollPtr reduce_scatter(at::Tensor& out, const at::Tensor& in, RedOp op);
  // One flag round among all ranks on the current stream, ordered after
  // the work already on it (bounded waits; a timeout sets the status word).
  DevCollPtr barrier();
  std::vector<std::pair<std::string, std::int64_t>> stats() const;
  int device() const { return dev_; }

 private:
  struct Launch {
    int mode;
    int op;
    int root;
    const at::Tensor* in;
    at::Tensor* out;
    std::int64_t n;
  };
  DevCollPtr run(const std::vector<Launch>& launches);
  void fill(CollArgs& a, const Launch& l, const at::Tensor& in, const at::Tensor& out);
  int choose_ctas(int mode, int algo, std::int64_t bytes) const;

  CudaTransport* tr_;
  Engine* eng_;
  DevCtx* ctx_;
  int dev_;
  int P_;
  int me_;
  bool shared_gpu_ = false;
  cudaStream_t stream_ = nullptr;  // collectives run here, ordered per group
  char* ws_ = nullptr;
  std::int64_t region_bytes_ = 0;
  std::int64_t oneshot_bytes_ = 0;
  std::vector<char*> data_;
  std::vector<std::uint64_t*> flags_;
  std::uint64_t epoch_ = 0;
  std::unique_ptr<NvlsBuffer> nvls_;  // null: no NVLS on this group
  std::string nvls_why_;              // why not (empty when enabled or not attempted)
  std::int64_t nvls_min_bytes_ = 0;
  int forced_algo_ = -1;  // COMMUX_ALGO
  std::int64_t st_barriers_ = 0, st_chain_ = 0;
  int chain_ranks_ = 0;  // COMMUX_CHAIN_RANKS (0: the chain is off)
  unsigned long long* trace_h_ = nullptr;  // COMMUX_COLL_TRACE (host-mapped)
  unsigned long long* trace_d_ = nullptr;
  void report_trace(int algo, int mode, std::int64_t bytes, int ctas);
  std::int64_t st_calls_ = 0, st_oneshot_ = 0, st_twoshot_ = 0, st_gather_ = 0, st_bytes_ = 0, st_nvls_ = 0;
};

}  // namespace cuda
}  // namespace commux
