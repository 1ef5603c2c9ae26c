// quiver::ThreadPool: a fork-join pool with the behaviour of the reference's src/thread_pool.cc
// (chunked parallel_for with the caller taking part, first exception rethrown and later chunks
// skipped, serialized concurrent callers, nested calls run inline), written as an epoch-counted
// broadcast: a call publishes one Loop, every worker claims chunks from its atomic counter, and
// the caller waits until each worker has checked out of that epoch.
#include "quiver/thread_pool.h"

#include <algorithm>
#include <atomic>

namespace quiver {

struct ThreadPool::Loop {
  const RangeFn* fn = nullptr;
  std::size_t n = 0, grain = 1, chunks = 0;
  std::atomic<std::size_t> next{0};
  std::atomic<bool> failed{false};
  std::mutex error_mu;
  std::exception_ptr error;
};

namespace {
// Depth of chunks the current thread is running, over all pools: a parallel_for issued from inside
// one runs inline, which keeps nested and cross-pool calls from waiting on busy workers.
thread_local int t_depth = 0;

struct DepthGuard {
  DepthGuard() { ++t_depth; }
  ~DepthGuard() { --t_depth; }
};
}  // namespace

ThreadPool::ThreadPool(std::size_t num_threads) {
  std::size_t total = num_threads;
  if (total == 0) total = std::max(1u, std::thread::hardware_concurrency());
  threads_.reserve(total - 1);
  for (std::size_t i = 1; i < total; ++i) threads_.emplace_back([this, i] { worker(i); });
}

ThreadPool::~ThreadPool() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    closing_ = true;
  }
  wake_.notify_all();
  for (auto& t : threads_) t.join();
}

void ThreadPool::drain(Loop& loop) noexcept {
  DepthGuard depth;
  for (;;) {
    const std::size_t c = loop.next.fetch_add(1, std::memory_order_relaxed);
    if (c >= loop.chunks) return;
    if (loop.failed.load(std::memory_order_acquire)) continue;  // skip what has not started
    const std::size_t begin = c * loop.grain;
    const std::size_t end = std::min(loop.n, begin + loop.grain);
    try {
      (*loop.fn)(begin, end);
    } catch (...) {
      std::lock_guard<std::mutex> lk(loop.error_mu);
      if (!loop.error) loop.error = std::current_exception();
      loop.failed.store(true, std::memory_order_release);
    }
  }
}

void ThreadPool::worker(std::size_t /*slot*/) {
  std::uint64_t seen = 0;
  for (;;) {
    Loop* loop = nullptr;
    {
      std::unique_lock<std::mutex> lk(mu_);
      wake_.wait(lk, [&] { return closing_ || epoch_ != seen; });
      if (closing_) return;
      seen = epoch_;
      loop = loop_;
    }
    drain(*loop);
    std::lock_guard<std::mutex> lk(mu_);
    if (--busy_ == 0) idle_.notify_all();
  }
}

void ThreadPool::parallel_for(std::size_t n, std::size_t grain, const RangeFn& fn) {
  if (n == 0) return;
  grain = std::max<std::size_t>(1, grain);
  const std::size_t chunks = (n + grain - 1) / grain;
  if (threads_.empty() || chunks == 1 || t_depth > 0) {
    DepthGuard depth;
    for (std::size_t b = 0; b < n; b += grain) fn(b, std::min(n, b + grain));
    return;
  }
  std::lock_guard<std::mutex> call(call_mu_);
  Loop loop;
  loop.fn = &fn;
  loop.n = n;
  loop.grain = grain;
  loop.chunks = chunks;
  {
    std::lock_guard<std::mutex> lk(mu_);
    loop_ = &loop;
    busy_ = threads_.size();
    ++epoch_;
  }
  wake_.notify_all();
  drain(loop);
  {
    std::unique_lock<std::mutex> lk(mu_);
    idle_.wait(lk, [&] { return busy_ == 0; });
    loop_ = nullptr;
  }
  if (loop.error) std::rethrow_exception(loop.error);
}

ThreadPool& ThreadPool::global() {
  static ThreadPool pool(0);
  return pool;
}

}  // namespace quiver
