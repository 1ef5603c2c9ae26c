// Fork-join pool for data-parallel host loops, with the public interface of the reference's
// include/quiver/thread_pool.h:14-40. On the GPU build the searches themselves run on the device;
// the pool evaluates PredicateFilter::contains over the stored labels and is kept in every
// signature that takes one so callers compile unchanged.
#pragma once

#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <exception>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace quiver {

class ThreadPool {
 public:
  /// Processes items [begin, end).
  using RangeFn = std::function<void(std::size_t begin, std::size_t end)>;

  /// `num_threads` includes the calling thread (1 = everything runs inline on the caller);
  /// 0 = std::thread::hardware_concurrency().
  explicit ThreadPool(std::size_t num_threads = 0);
  ~ThreadPool();

  ThreadPool(const ThreadPool&) = delete;
  ThreadPool& operator=(const ThreadPool&) = delete;

  std::size_t num_threads() const noexcept { return threads_.size() + 1; }

  /// Runs fn over [0, n) in chunks of at most `grain` items on the workers and the caller, and
  /// returns when every chunk is done. After a chunk throws, chunks not yet started are skipped
  /// and the first exception is rethrown to the caller. Concurrent callers take turns; a call made
  /// from inside a chunk (of this or any other pool) runs inline.
  void parallel_for(std::size_t n, std::size_t grain, const RangeFn& fn);

  /// One pool per process, sized to the machine, built on first use.
  static ThreadPool& global();

 private:
  struct Loop;

  void worker(std::size_t slot);
  static void drain(Loop& loop) noexcept;

  std::vector<std::thread> threads_;
  std::mutex call_mu_;  // one parallel_for at a time

  std::mutex mu_;
  std::condition_variable wake_;
  std::condition_variable idle_;
  Loop* loop_ = nullptr;
  std::uint64_t epoch_ = 0;
  std::size_t busy_ = 0;
  bool closing_ = false;
};

}  // namespace quiver
