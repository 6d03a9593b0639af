// thread_pool.hpp — a persistent fork/join pool for batch env stepping.
//
// The env batch is stepped hundreds of times per training iteration. Creating
// a team per call (an OpenMP parallel-for) was measured by the reference to
// cost milliseconds on many-core hosts; here workers live for the pool's
// lifetime, sleep on a condition variable between jobs, and the caller joins
// on an atomic counter. Work is split into contiguous static chunks so each
// worker touches the same envs every call (cache- and NUMA-friendly).
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace surf {

class ThreadPool {
 public:
  explicit ThreadPool(int threads) {
    if (threads < 1) threads = 1;
    nthreads_ = threads;
    for (int t = 1; t < threads; ++t) workers_.emplace_back([this, t] { loop(t); });
  }
  ~ThreadPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      ++generation_;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
  }
  int size() const { return nthreads_; }

  // Run fn(begin, end) over [0, n) split into size() contiguous chunks; the
  // calling thread takes chunk 0. Returns when every chunk has finished.
  void run(int n, const std::function<void(int, int)>& fn) {
    if (nthreads_ == 1 || n < 2 * nthreads_) { fn(0, n); return; }
    {
      std::lock_guard<std::mutex> g(mu_);
      job_ = &fn;
      n_ = n;
      pending_.store(nthreads_ - 1, std::memory_order_relaxed);
      ++generation_;
    }
    cv_.notify_all();
    auto [b, e] = chunk(0, n);
    fn(b, e);
    while (pending_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
  }

 private:
  std::pair<int, int> chunk(int t, int n) const {
    int64_t b = static_cast<int64_t>(n) * t / nthreads_;
    int64_t e = static_cast<int64_t>(n) * (t + 1) / nthreads_;
    return {static_cast<int>(b), static_cast<int>(e)};
  }
  void loop(int t) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(int, int)>* job;
      int n;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return generation_ != seen; });
        seen = generation_;
        if (stop_) return;
        job = job_;
        n = n_;
      }
      auto [b, e] = chunk(t, n);
      (*job)(b, e);
      pending_.fetch_sub(1, std::memory_order_acq_rel);
    }
  }
  int nthreads_ = 1;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_;
  uint64_t generation_ = 0;
  bool stop_ = false;
  const std::function<void(int, int)>* job_ = nullptr;
  int n_ = 0;
  std::atomic<int> pending_{0};
};

}  // namespace surf
