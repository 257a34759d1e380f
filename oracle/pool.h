// pool.h -- TEST INFRASTRUCTURE ONLY (see oracle.h).
// A persistent fork/join thread pool standing in for the reference's rayon
// pool (src/backend.rs:80-85, 109-112): parallel_for splits [0, n) into one
// contiguous chunk per worker and returns when every chunk is done.
#pragma once
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

class ForkJoinPool {
 public:
  explicit ForkJoinPool(int threads) : n_(threads < 1 ? 1 : threads) {
    for (int i = 1; i < n_; i++) workers_.emplace_back([this, i] { loop(i); });
  }
  ~ForkJoinPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return n_; }
  // Runs fn(begin, end) over n items split in n_ contiguous chunks.
  void parallel_for(long n, const std::function<void(long, long)>& fn) {
    if (n_ == 1 || n <= 1) {
      fn(0, n);
      return;
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      fn_ = &fn;
      total_ = n;
      pending_ = n_ - 1;
      gen_++;
    }
    cv_.notify_all();
    run_chunk(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    fn_ = nullptr;
  }

 private:
  void run_chunk(int idx) {
    long n = total_;
    long b = n * idx / n_, e = n * (idx + 1) / n_;
    if (b < e) (*fn_)(b, e);
  }
  void loop(int idx) {
    unsigned long seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
      }
      run_chunk(idx);
      {
        std::lock_guard<std::mutex> g(mu_);
        if (--pending_ == 0) done_cv_.notify_one();
      }
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(long, long)>* fn_ = nullptr;
  long total_ = 0;
  int pending_ = 0;
  unsigned long gen_ = 0;
  bool stop_ = false;
};
