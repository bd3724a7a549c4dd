// Persistent worker pool shared by the host-side step code.
#pragma once

#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace dsd {
namespace detail {

// A small persistent thread pool: ParallelFor(n, fn) runs fn(0..n-1) on the
// workers and the calling thread, returning when every index is done.  Used
// for the per-request payload generation of a step, which is independent
// across requests (the page allocator stays serial).
class WorkerPool {
 public:
  explicit WorkerPool(int threads) {
    for (int t = 0; t < threads; ++t) workers_.emplace_back([this] { Loop(); });
  }
  ~WorkerPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
  }
  void ParallelFor(int n, const std::function<void(int)>& fn) {
    if (n <= 0) return;
    if (workers_.empty() || n == 1) {
      for (int i = 0; i < n; ++i) fn(i);
      return;
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      fn_.store(&fn);
      n_.store(n);
      next_.store(0);
      done_ = 0;
      ++generation_;
    }
    cv_.notify_all();
    Work();
    std::unique_lock<std::mutex> g(mu_);
    done_cv_.wait(g, [&] { return done_ == n_.load(); });
  }

 private:
  void Work() {
    int finished = 0;
    // n_ and fn_ are published before next_ is reset, so an index claimed
    // from next_ always belongs to the job they describe
    for (int i = next_.fetch_add(1); i < n_.load(); i = next_.fetch_add(1)) {
      (*fn_.load())(i);
      ++finished;
    }
    if (finished) {
      std::lock_guard<std::mutex> g(mu_);
      done_ += finished;
      if (done_ == n_.load()) done_cv_.notify_all();
    }
  }
  void Loop() {
    long seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] { return stop_ || generation_ != seen; });
        if (stop_) return;
        seen = generation_;
      }
      Work();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::atomic<const std::function<void(int)>*> fn_{nullptr};
  std::atomic<int> next_{1 << 30};
  std::atomic<int> n_{0};
  int done_ = 0;
  long generation_ = 0;
  bool stop_ = false;
};

}  // namespace detail
}  // namespace dsd
