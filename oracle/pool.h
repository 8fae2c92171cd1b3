// pool.h — TEST INFRASTRUCTURE (see oracle.h): a persistent worker pool, the role of milcpu's
// goroutines over GOMAXPROCS (internal/milcpu/ops.go:401-425, internal/sgemm/sgemm.go:127-162).
#ifndef HWNPU_ORACLE_POOL_H
#define HWNPU_ORACLE_POOL_H

#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace oracle {

class Pool {
 public:
  explicit Pool(int threads) : n_(threads < 1 ? 1 : threads) {
    for (int i = 1; i < n_; ++i) workers_.emplace_back([this, i] { loop(i); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto &t : workers_) t.join();
  }
  int size() const { return n_; }

  // Runs f(lo, hi) over [0, n) split in chunks of at least grain, on all threads.
  void parallel_for(long n, long grain, const std::function<void(long, long)> &f) {
    if (n <= 0) return;
    long chunks = (n + grain - 1) / grain;
    if (n_ == 1 || chunks == 1) { f(0, n); return; }
    long per = (chunks + n_ * 4 - 1) / (n_ * 4);
    long step = per * grain;
    std::atomic<long> next{0};
    auto body = [&] {
      for (;;) {
        long lo = next.fetch_add(step);
        if (lo >= n) return;
        f(lo, std::min(n, lo + step));
      }
    };
    {
      std::lock_guard<std::mutex> g(mu_);
      job_ = body;
      pending_ = n_ - 1;
      gen_++;
    }
    cv_.notify_all();
    body();
    std::unique_lock<std::mutex> g(mu_);
    done_.wait(g, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void loop(int) {
    long seen = 0;
    for (;;) {
      std::function<void()> job;
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
        job = job_;
      }
      if (job) job();
      {
        std::lock_guard<std::mutex> g(mu_);
        if (--pending_ == 0) done_.notify_one();
      }
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  std::function<void()> job_;
  long gen_ = 0;
  int pending_ = 0;
  bool stop_ = false;
};

}  // namespace oracle

#endif
