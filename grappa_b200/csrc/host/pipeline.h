// Bounded producer/consumer pipeline: one worker thread produces items 0..n-1 in
// order and keeps at most `depth` of them ready; the consumer sleeps on a condition
// variable until the next one is there.  It carries the host sampler's batch
// prefetch (reference: csrc/python/py_graph.cc:50-371, where the consumer busy-waits
// on an atomic counter) and has no Python in it, so the native tests run it under
// the thread sanitizer.
#pragma once
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <exception>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>

namespace grappa {
namespace host {

template <typename T>
class BatchPipeline {
 public:
  using Producer = std::function<std::unique_ptr<T>(int64_t)>;

  explicit BatchPipeline(size_t depth = 2) : depth_(depth == 0 ? 1 : depth) {}
  BatchPipeline(const BatchPipeline&) = delete;
  BatchPipeline& operator=(const BatchPipeline&) = delete;
  ~BatchPipeline() { stop(); }

  // Stops a running worker (dropping what it had ready), then starts producing
  // items 0..n_items-1 with `fn`.
  void start(int64_t n_items, Producer fn) {
    stop();
    {
      std::lock_guard<std::mutex> lk(mu_);
      n_items_ = n_items < 0 ? 0 : n_items;
      consumed_ = 0;
      produced_ = 0;
      stop_ = false;
      err_ = false;
      err_msg_.clear();
      fn_ = std::move(fn);
    }
    worker_ = std::thread([this] { run(); });
  }

  // The next item in order; nullptr once all n_items were consumed or after stop().
  // Rethrows the producer's failure (as std::runtime_error) when it is the next
  // thing in line.
  std::unique_ptr<T> next() {
    std::unique_ptr<T> item;
    {
      std::unique_lock<std::mutex> lk(mu_);
      if (consumed_ >= n_items_) return nullptr;
      cv_.wait(lk, [this] { return !q_.empty() || err_ || stop_; });
      if (q_.empty()) {
        if (err_) throw std::runtime_error("batch producer failed: " + err_msg_);
        return nullptr;  // stopped
      }
      item = std::move(q_.front());
      q_.pop_front();
      consumed_++;
    }
    cv_.notify_all();
    return item;
  }

  // Ends the worker (waking it if it waits for room) and drops the ready items.
  void stop() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    if (worker_.joinable()) worker_.join();
    std::lock_guard<std::mutex> lk(mu_);
    q_.clear();
  }

  int64_t consumed() const {
    std::lock_guard<std::mutex> lk(mu_);
    return consumed_;
  }
  int64_t produced() const {
    std::lock_guard<std::mutex> lk(mu_);
    return produced_;
  }
  size_t ready() const {
    std::lock_guard<std::mutex> lk(mu_);
    return q_.size();
  }
  size_t depth() const { return depth_; }

 private:
  void run() {
    Producer fn;
    int64_t n;
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn = fn_;
      n = n_items_;
    }
    try {
      for (int64_t s = 0; s < n; ++s) {
        {
          std::unique_lock<std::mutex> lk(mu_);
          cv_.wait(lk, [this] { return q_.size() < depth_ || stop_; });
          if (stop_) return;
        }
        std::unique_ptr<T> item = fn(s);  // outside the lock: the consumer keeps going
        {
          std::lock_guard<std::mutex> lk(mu_);
          q_.push_back(std::move(item));
          produced_++;
        }
        cv_.notify_all();
      }
    } catch (const std::exception& ex) {
      std::lock_guard<std::mutex> lk(mu_);
      err_ = true;
      err_msg_ = ex.what();
    } catch (...) {
      std::lock_guard<std::mutex> lk(mu_);
      err_ = true;
      err_msg_ = "unknown exception";
    }
    cv_.notify_all();
  }

  const size_t depth_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::unique_ptr<T>> q_;
  std::thread worker_;
  Producer fn_;
  int64_t n_items_ = 0, consumed_ = 0, produced_ = 0;
  bool stop_ = false, err_ = false;
  std::string err_msg_;
};

}  // namespace host
}  // namespace grappa
