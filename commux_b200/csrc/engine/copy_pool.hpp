#pragma once

// Helper threads for large single-copy reads (process_vm_readv) of host
// messages. One thread copies at a few GB/s; a message of several MB split
// across a few threads moves at a multiple of that until memory bandwidth
// caps it. The caller runs one piece itself and waits for the rest, so a
// read still completes inside the call that asked for it.

#include <condition_variable>
#include <deque>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace commux {

class CopyPool {
 public:
  explicit CopyPool(int threads) {
    try {
      for (int i = 0; i < threads; ++i) threads_.emplace_back([this] { run(); });
    } catch (...) {
      stop_and_join();  // a thread that failed to start leaves the others joinable
      throw;
    }
  }
  ~CopyPool() { stop_and_join(); }
  CopyPool(const CopyPool&) = delete;
  CopyPool& operator=(const CopyPool&) = delete;

  int threads() const { return static_cast<int>(threads_.size()); }

  // Runs tasks[0] on the calling thread and the others on the helpers;
  // returns once all of them have finished.
  void run_all(std::vector<std::function<void()>>& tasks) {
    if (tasks.empty()) return;
    struct Latch {
      std::mutex mu;
      std::condition_variable cv;
      std::size_t left;
    };
    auto latch = std::make_shared<Latch>();
    latch->left = tasks.size() - 1;
    {
      std::lock_guard<std::mutex> lk(mu_);
      for (std::size_t i = 1; i < tasks.size(); ++i)
        queue_.push_back([latch, f = std::move(tasks[i])] {
          f();
          std::lock_guard<std::mutex> g(latch->mu);
          if (--latch->left == 0) latch->cv.notify_all();
        });
    }
    cv_.notify_all();
    tasks[0]();
    std::unique_lock<std::mutex> lk(latch->mu);
    latch->cv.wait(lk, [&] { return latch->left == 0; });
  }

 private:
  void stop_and_join() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : threads_)
      if (t.joinable()) t.join();
  }

  void run() {
    for (;;) {
      std::function<void()> f;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
        if (queue_.empty()) return;  // stopping
        f = std::move(queue_.front());
        queue_.pop_front();
      }
      f();
    }
  }

  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::function<void()>> queue_;
  bool stop_ = false;
  std::vector<std::thread> threads_;
};

}  // namespace commux
