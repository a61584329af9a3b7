// watchdog.h -- a host thread that bounds how long enqueued work may take.
//
// The reference bounds request lifetimes on the host: a deadline per
// request, checked by the scheduler (src/scheduler/continuous_batching.rs:
// 83-100).  A verify step over a tensor-parallel group has a second failure
// mode the reference never meets: an NCCL collective whose peer has stopped
// (a crashed or stalled rank) blocks the stream for good.  The watchdog
// turns that into an error: every armed probe carries a deadline; a thread
// polls the oldest probe and, once a deadline passes with the probe still
// pending, calls the abort hook once (for NCCL: ncclCommAbort, which ends
// the stuck collective) and stops watching.  Host code only; the probes are
// opaque (CUDA events for NCCL, callbacks in the CPU tests).
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <thread>
#include <utility>

namespace kyro {

class Watchdog {
 public:
  using PollFn = int (*)(void* user, void* probe);  // 1: complete, 0: pending
  using AbortFn = void (*)(void* user);
  using SetupFn = void (*)(void* user);             // runs once on the thread

  Watchdog(PollFn poll, AbortFn abort, SetupFn setup, void* user)
      : poll_(poll), abort_(abort), setup_(setup), user_(user) {
    thread_ = std::thread([this] { run(); });
  }

  ~Watchdog() {
    {
      std::lock_guard<std::mutex> lock(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    thread_.join();
  }

  Watchdog(const Watchdog&) = delete;
  Watchdog& operator=(const Watchdog&) = delete;

  // Watch `probe` until it completes or `timeout_ns` passes.  Returns false
  // (and watches nothing) once the watchdog has fired.
  bool arm(void* probe, uint64_t timeout_ns) {
    if (fired_.load()) return false;
    {
      std::lock_guard<std::mutex> lock(mu_);
      queue_.emplace_back(probe, Clock::now() + std::chrono::nanoseconds(timeout_ns));
    }
    cv_.notify_all();
    return true;
  }

  // Whether `probe` is still queued (not yet seen complete).
  bool pending(void* probe) {
    std::lock_guard<std::mutex> lock(mu_);
    for (auto& e : queue_)
      if (e.first == probe) return true;
    return false;
  }

  bool fired() const { return fired_.load(); }

  // Block until every armed probe has completed or the watchdog has fired.
  // Returns true if it fired.
  bool wait_idle() {
    std::unique_lock<std::mutex> lock(mu_);
    idle_cv_.wait(lock, [this] { return queue_.empty() || fired_.load(); });
    return fired_.load();
  }

 private:
  using Clock = std::chrono::steady_clock;

  void run() {
    if (setup_) setup_(user_);
    std::unique_lock<std::mutex> lock(mu_);
    while (!stop_) {
      if (queue_.empty() || fired_.load()) {
        cv_.wait(lock, [this] { return stop_ || (!queue_.empty() && !fired_.load()); });
        continue;
      }
      auto [probe, deadline] = queue_.front();
      lock.unlock();
      const bool done = poll_(user_, probe) != 0;
      const bool late = !done && Clock::now() > deadline;
      if (late) abort_(user_);  // at most once: fired_ stops the loop below
      lock.lock();
      if (done) {
        if (!queue_.empty() && queue_.front().first == probe) queue_.pop_front();
        if (queue_.empty()) idle_cv_.notify_all();
        continue;  // the next probe is polled right away
      }
      if (late) {
        fired_.store(true);
        queue_.clear();
        idle_cv_.notify_all();
        continue;
      }
      cv_.wait_for(lock, std::chrono::microseconds(200));
    }
  }

  PollFn poll_;
  AbortFn abort_;
  SetupFn setup_;
  void* user_;
  std::mutex mu_;
  std::condition_variable cv_, idle_cv_;
  std::deque<std::pair<void*, Clock::time_point>> queue_;
  bool stop_ = false;
  std::atomic<bool> fired_{false};
  std::thread thread_;
};

}  // namespace kyro
