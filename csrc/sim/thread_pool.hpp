// thread_pool.hpp — a persistent fork/join pool for batch env stepping.
//
// The env batch is stepped hundreds of times per training iteration. Creating
// a team per call (an OpenMP parallel-for) was measured by the reference to
// cost milliseconds on many-core hosts; here workers live for the pool's
// lifetime, sleep on a condition variable between jobs, and the caller joins
// on an atomic counter. The range is handed out in contiguous chunks of about
// n / (8 x threads) items claimed from an atomic cursor (the caller works
// too): envs differ in cost (a surfer traces more than a faller), and with
// static per-thread chunks the slowest chunk set the pace -- 3 threads on
// 1024 envs stepped 24% faster with claimed chunks. Items are independent, so
// which thread runs which chunk changes no result.
//
// run_async() hands a job to the workers only and returns; wait() then makes
// the caller claim the chunks still open and returns when all are done, so
// the caller can do other work (launching the GPU's next graph) while the
// workers step envs.
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
    for (int t = 1; t < threads; ++t) workers_.emplace_back([this] { loop(); });
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

  // Run fn(begin, end) over [0, n) in contiguous chunks claimed by the workers
  // and the calling thread. Returns when every chunk has finished.
  void run(int n, const std::function<void(int, int)>& fn) {
    if (nthreads_ == 1 || n < 2 * nthreads_) { fn(0, n); return; }
    publish(&fn, n);
    work(fn, n);
    while (pending_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
  }

  // Start fn over [0, n) on the workers (the pool keeps its own copy of fn)
  // and return; wait() finishes it. One job at a time: run() and run_async()
  // must not be called again before wait().
  void run_async(int n, std::function<void(int, int)> fn) {
    async_fn_ = std::move(fn);
    async_n_ = n;
    if (nthreads_ == 1 || n < 2 * nthreads_) return;      // wait() runs it on the caller
    publish(&async_fn_, n);
  }
  void wait() {
    if (!async_fn_) return;
    if (nthreads_ == 1 || async_n_ < 2 * nthreads_) {
      async_fn_(0, async_n_);
    } else {
      work(async_fn_, async_n_);
      while (pending_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
    }
    async_fn_ = nullptr;
  }

 private:
  // claim chunks until the range is exhausted
  void work(const std::function<void(int, int)>& fn, int n) {
    const int grain = n / (nthreads_ * 8) > 4 ? n / (nthreads_ * 8) : 4;
    for (;;) {
      const int b = next_.fetch_add(grain, std::memory_order_relaxed);
      if (b >= n) break;
      fn(b, b + grain < n ? b + grain : n);
    }
  }
  void publish(const std::function<void(int, int)>* fn, int n) {
    {
      std::lock_guard<std::mutex> g(mu_);
      job_ = fn;
      n_ = n;
      next_.store(0, std::memory_order_relaxed);
      pending_.store(nthreads_ - 1, std::memory_order_relaxed);
      ++generation_;
    }
    cv_.notify_all();
  }
  void loop() {
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
      work(*job, n);
      pending_.fetch_sub(1, std::memory_order_acq_rel);
    }
  }
  int nthreads_ = 1;
  std::atomic<int> next_{0};
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_;
  uint64_t generation_ = 0;
  bool stop_ = false;
  std::function<void(int, int)> async_fn_;
  int async_n_ = 0;
  const std::function<void(int, int)>* job_ = nullptr;
  int n_ = 0;
  std::atomic<int> pending_{0};
};

}  // namespace surf
