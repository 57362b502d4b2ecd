// Multi-rank C++ test driver for commux::ProcessGroupUCX (same coverage as
// reference tests/test_commux.cpp: tag matching, collectives, vector p2p,
// group window, multi-threaded posting, parked-waiter wakeups, a V-tensor
// ping-pong benchmark), plus large rendezvous messages (T8), a large
// allreduce (T9) and a seeded random exchange (T10). Ranks bootstrap through a c10d::TCPStore (rank 0
// hosts it).
//
//   test_commux <rank> <world> [host] [port]
//   COMMUX_TEST_DEVICE=cuda (or UCXPG_DEVICE=cuda) runs the p2p/collective
//                            checks on CUDA tensors
//   COMMUX_BENCH=1 [COMMUX_BENCH_V=16]  adds the ping-pong benchmark
//   COMMUX_MT=1 / COMMUX_DEADLOCK=1     add the thread tests

#include <torch/torch.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>
#include <thread>
#include <torch/csrc/distributed/c10d/TCPStore.hpp>
#include <vector>

#include "commux/process_group_ucx.hpp"

namespace {

int g_fail = 0;

void check(bool ok, const std::string& what) {
  std::printf("  [%s] %s\n", ok ? "PASS" : "FAIL", what.c_str());
  if (!ok) ++g_fail;
}

bool env_on(const char* n) {
  const char* e = std::getenv(n);
  return e != nullptr && (std::string(e) == "1" || std::string(e) == "on");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: %s <rank> <world> [host=127.0.0.1] [port=29555]\n", argv[0]);
    return 2;
  }
  const int rank = std::atoi(argv[1]);
  const int world = std::atoi(argv[2]);
  const std::string host = argc > 3 ? argv[3] : "127.0.0.1";
  const int port = argc > 4 ? std::atoi(argv[4]) : 29555;
  // the driver checks the engine's threads: torch's own intra-op threads
  // (OpenMP, whose synchronisation ThreadSanitizer cannot see) stay off
  at::set_num_threads(1);

  c10d::TCPStoreOptions so;
  so.port = static_cast<std::uint16_t>(port);
  so.isServer = rank == 0;
  so.numWorkers = world;
  so.waitWorkers = true;
  auto store = c10::make_intrusive<c10d::TCPStore>(host, so);
  auto pg = c10::make_intrusive<commux::ProcessGroupUCX>(store, rank, world,
                                                        std::chrono::milliseconds(60000));

  torch::Device device(torch::kCPU);
  // COMMUX_TEST_DEVICE, or UCXPG_DEVICE as in the reference's instructions
  const char* dv = std::getenv("COMMUX_TEST_DEVICE");
  if (dv == nullptr) dv = std::getenv("UCXPG_DEVICE");
  if (dv != nullptr && std::string(dv) == "cuda") {
    if (!torch::cuda::is_available()) {
      std::fprintf(stderr, "CUDA requested but not available\n");
      return 2;
    }
    device = torch::Device(torch::kCUDA, rank % static_cast<int>(torch::cuda::device_count()));
  }
  auto f64 = torch::TensorOptions().dtype(torch::kFloat64).device(device);
  std::printf("[rank %d/%d] backend=%s device=%s\n", rank, world, pg->getBackendName().c_str(),
              device.str().c_str());

  // T1: out-of-order tag matching with non-blocking posts
  if (world >= 2 && rank <= 1) {
    if (rank == 0) {
      std::vector<at::Tensor> a{torch::full({4}, 1.0, f64)}, b{torch::full({4}, 2.0, f64)};
      auto wa = pg->send(a, 1, 100);
      auto wb = pg->send(b, 1, 200);
      wa->wait();
      wb->wait();
    } else {
      std::vector<at::Tensor> b{torch::zeros({4}, f64)}, a{torch::zeros({4}, f64)};
      auto wb = pg->recv(b, 0, 200);
      auto wa = pg->recv(a, 0, 100);
      wb->wait();
      wa->wait();
      check(b[0].eq(2.0).all().item<bool>() && a[0].eq(1.0).all().item<bool>(),
            "tag matching: out-of-order receive delivered by tag");
    }
  }
  pg->barrier()->wait();

  // T2: allreduce SUM/MIN/MAX
  {
    const double me = rank + 1;
    auto run = [&](c10d::ReduceOp::RedOpType op) {
      std::vector<at::Tensor> v{torch::full({3}, me, f64)};
      c10d::AllreduceOptions o;
      o.reduceOp = op;
      pg->allreduce(v, o)->wait();
      return v[0][0].item<double>();
    };
    check(run(c10d::ReduceOp::SUM) == world * (world + 1) / 2.0, "allreduce SUM");
    check(run(c10d::ReduceOp::MIN) == 1.0, "allreduce MIN");
    check(run(c10d::ReduceOp::MAX) == world, "allreduce MAX");
  }
  // T3: reduce to root 0
  {
    std::vector<at::Tensor> v{torch::full({2}, rank + 1.0, f64)};
    c10d::ReduceOptions o;
    o.rootRank = 0;
    pg->reduce(v, o)->wait();
    if (rank == 0) check(v[0][0].item<double>() == world * (world + 1) / 2.0, "reduce SUM on root");
  }
  pg->barrier()->wait();

  // T4: vector p2p of 3 differently shaped tensors (IOV under COMMUX_COALESCE)
  if (world >= 2 && rank <= 1) {
    const std::vector<int64_t> shapes{5, 1, 8};
    std::vector<at::Tensor> v;
    for (size_t k = 0; k < shapes.size(); ++k)
      v.push_back(rank == 0 ? torch::full({shapes[k]}, 10.0 + k, f64) : torch::zeros({shapes[k]}, f64));
    if (rank == 0) {
      pg->send(v, 1, 300)->wait();
    } else {
      pg->recv(v, 0, 300)->wait();
      bool ok = true;
      for (size_t k = 0; k < shapes.size(); ++k) ok = ok && v[k].eq(10.0 + k).all().item<bool>();
      check(ok, "vector p2p delivers all V buffers");
    }
  }

  // T5: group window (deferred recv + send, one aggregate Work)
  if (world >= 2 && rank <= 1) {
    const int peer = 1 - rank;
    std::vector<at::Tensor> out{torch::zeros({4}, f64)}, mine{torch::full({4}, rank + 1.0, f64)};
    pg->startCoalescing();
    pg->recv(out, peer, rank == 0 ? 420 : 410);
    pg->send(mine, peer, rank == 0 ? 410 : 420);
    pg->endCoalescing()->wait();
    check(out[0].eq(peer + 1.0).all().item<bool>(), "group window: deferred recv/send completed");
  }
  pg->barrier()->wait();

  // T8: large messages both ways at once (rendezvous; on one host the
  // single-copy read, split across the copy helpers)
  if (world >= 2 && rank <= 1) {
    const int peer = 1 - rank;
    const std::int64_t n = 3 << 20;  // 24 MiB of fp64 per message
    std::vector<at::Tensor> mine{torch::arange(n, f64).add_(1e7 * rank)};
    std::vector<at::Tensor> got{torch::zeros({n}, f64)};
    auto r = pg->recv(got, peer, 800);
    auto s = pg->send(mine, peer, 800);
    r->wait();
    s->wait();
    check(got[0].equal(torch::arange(n, f64).add_(1e7 * peer)),
          "large message: every byte of a 24 MiB rendezvous arrived");
  }
  pg->barrier()->wait();

  // T9: a 4 MiB allreduce (its fold runs on the copy helpers), exact values
  {
    const std::int64_t n = 1 << 19;  // fp64
    std::vector<at::Tensor> t{torch::arange(n, f64).remainder(97).add_(rank)};
    pg->allreduce(t)->wait();
    double ranks = 0;
    for (int r = 0; r < world; ++r) ranks += r;
    auto want = torch::arange(n, f64).remainder(97).mul_(static_cast<double>(world)).add_(ranks);
    check(t[0].equal(want), "large allreduce (parallel fold) exact");
  }
  pg->barrier()->wait();

  // T10: a seeded random exchange between ranks 0 and 1: 48 messages each
  // way, from empty through eager to rendezvous sizes, on 4 tags (so many
  // messages share a (source, tag) pair and must match in posting order),
  // all posted before any wait
  if (world >= 2 && rank <= 1) {
    const int peer = 1 - rank;
    const std::int64_t sizes[] = {0, 1, 7, 1000, 8192, 8193, 70000, 131072};  // fp64 elements
    std::mt19937 rng(20261202);
    struct Msg {
      std::int64_t n;
      int tag;
    };
    std::vector<Msg> msgs;
    for (int i = 0; i < 48; ++i) msgs.push_back({sizes[rng() % 8], static_cast<int>(rng() % 4)});
    auto payload = [&](int from, int i) {
      return torch::arange(msgs[i].n, f64).remainder(1009).add_(1e4 * from + i);
    };
    std::vector<c10::intrusive_ptr<c10d::Work>> works;
    std::vector<std::vector<at::Tensor>> got(msgs.size()), mine(msgs.size());
    for (std::size_t i = 0; i < msgs.size(); ++i) {
      got[i] = {torch::full({msgs[i].n}, -1.0, f64)};
      works.push_back(pg->recv(got[i], peer, 700 + msgs[i].tag));
    }
    for (std::size_t i = 0; i < msgs.size(); ++i) {
      mine[i] = {payload(rank, static_cast<int>(i))};
      works.push_back(pg->send(mine[i], peer, 700 + msgs[i].tag));
    }
    for (auto& w : works) w->wait();
    bool ok = true;
    for (std::size_t i = 0; i < msgs.size(); ++i) ok = ok && got[i][0].equal(payload(peer, static_cast<int>(i)));
    check(ok, "random exchange: 48 messages each way intact and in order");
  }
  pg->barrier()->wait();

  // Ping-pong benchmark: V tensors of 1024 fp64 per message, host-timed
  if (env_on("COMMUX_BENCH") && world >= 2 && rank <= 1) {
    const int V = std::getenv("COMMUX_BENCH_V") ? std::atoi(std::getenv("COMMUX_BENCH_V")) : 16;
    const int iters = 2000;
    std::vector<at::Tensor> sv, rv;
    for (int k = 0; k < V; ++k) {
      sv.push_back(torch::full({1024}, static_cast<double>(k), f64));
      rv.push_back(torch::zeros({1024}, f64));
    }
    auto t0 = std::chrono::steady_clock::now();
    for (int it = 0; it < 100 + iters; ++it) {
      if (it == 100) {  // after 100 warm-up round trips
        if (device.is_cuda()) torch::cuda::synchronize();
        t0 = std::chrono::steady_clock::now();
      }
      if (rank == 0) {
        pg->send(sv, 1, 900)->wait();
        pg->recv(rv, 1, 901)->wait();
      } else {
        pg->recv(rv, 0, 900)->wait();
        pg->send(sv, 0, 901)->wait();
      }
      if (it == 100 + iters - 1 && rank == 0) {
        if (device.is_cuda()) torch::cuda::synchronize();
        double us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count() / iters;
        const char* c = std::getenv("COMMUX_COALESCE");
        std::printf("[bench] V=%d iters=%d round-trip=%.2f us/iter (COMMUX_COALESCE=%s)\n", V, iters, us,
                    c ? c : "default");
      }
    }
  }
  pg->barrier()->wait();

  // T6: two threads per rank post and wait concurrently on their own tags
  if (env_on("COMMUX_MT") && world == 2) {
    const int peer = 1 - rank;
    std::atomic<int> good{0};
    auto job = [&](int t) {
      bool ok = true;
      for (int it = 0; it < 200 && ok; ++it) {
        double val = rank * 1000 + t * 10 + (it % 7);
        std::vector<at::Tensor> s{torch::full({16}, val, f64)}, r{torch::zeros({16}, f64)};
        auto wr = pg->recv(r, peer, 600 + t);
        auto ws = pg->send(s, peer, 600 + t);
        wr->wait();
        ws->wait();
        ok = r[0].eq(peer * 1000 + t * 10 + (it % 7)).all().item<bool>();
      }
      if (ok) good++;
    };
    std::thread a(job, 0), b(job, 1);
    a.join();
    b.join();
    check(good.load() == 2, "concurrent multi-threaded send/recv (2 threads)");
  }

  // T7: 8 receivers parked in wait() before a burst of sends, 16 rounds;
  // a watchdog aborts instead of hanging if a wakeup is lost.
  if (env_on("COMMUX_DEADLOCK") && world == 2) {
    const int peer = 1 - rank, NT = 8, ROUNDS = 16;
    std::atomic<bool> done{false};
    std::thread watchdog([&] {
      for (int i = 0; i < 1200 && !done.load(); ++i) std::this_thread::sleep_for(std::chrono::milliseconds(50));
      if (!done.load()) {
        std::fprintf(stderr, "[rank %d] T7 watchdog: parked waiters did not all wake\n", rank);
        std::abort();
      }
    });
    std::atomic<int> good{0};
    for (int round = 0; round < ROUNDS; ++round) {
      std::vector<std::thread> recvs;
      for (int t = 0; t < NT; ++t)
        recvs.emplace_back([&, t] {
          std::vector<at::Tensor> v{torch::zeros({1024}, f64)};
          pg->recv(v, peer, 700 + t)->wait();
          if (v[0].eq(peer * 100.0 + t).all().item<bool>()) good++;
        });
      std::this_thread::sleep_for(std::chrono::milliseconds(100));
      std::vector<at::Tensor> bufs;
      std::vector<c10::intrusive_ptr<c10d::Work>> ws;
      for (int t = 0; t < NT; ++t) {
        bufs.push_back(torch::full({1024}, rank * 100.0 + t, f64));
        std::vector<at::Tensor> v{bufs.back()};
        ws.push_back(pg->send(v, peer, 700 + t));
      }
      for (auto& w : ws) w->wait();
      for (auto& th : recvs) th.join();
    }
    check(good.load() == NT * ROUNDS, "parked waiters all wake (no lost wakeup)");
    done.store(true);
    watchdog.join();
  }

  pg->barrier()->wait();
  if (rank == 0) std::printf(g_fail == 0 ? "\nALL TESTS PASSED\n" : "\n%d TEST(S) FAILED\n", g_fail);
  return g_fail == 0 ? 0 : 1;
}
