// Exact brute-force k-NN over every stored vector, with the interface of the reference's
// include/quiver/flat_index.h:17-58. The rows live in GPU memory; searches run the tensor-core
// screen + exact re-rank kernels behind the qv_flat_* C ABI (include/qv_gpu.h), and return the
// distances and labels the reference's CPU search returns.
//
// Thread-safe: searches may run concurrently; add() excludes them while it appends.
#pragma once

#include <cstddef>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <vector>

#include "quiver/common.h"
#include "quiver/filter.h"
#include "quiver/thread_pool.h"

struct qv_flat;

namespace quiver {

class FlatIndex {
 public:
  explicit FlatIndex(std::size_t dim, Metric metric = Metric::kL2);
  ~FlatIndex();
  FlatIndex(FlatIndex&&) noexcept;
  FlatIndex& operator=(FlatIndex&&) noexcept;

  /// Appends n row-major vectors; with labels == nullptr vector i is labelled size() + i. Labels
  /// need not be unique. At most 2^32 vectors.
  void add(const float* vectors, std::size_t n, const Label* labels = nullptr);

  /// The k nearest stored vectors, closest first; fewer than k when fewer are stored or admitted.
  std::vector<Neighbor> search(const float* query, std::size_t k,
                               const Filter* filter = nullptr) const;

  /// nq row-major queries at once; writes nq * k results, padding missing ones with
  /// kInvalidLabel / +infinity. `pool` only evaluates a PredicateFilter.
  void search_batch(const float* queries, std::size_t nq, std::size_t k, Label* labels,
                    float* distances, const Filter* filter = nullptr,
                    ThreadPool* pool = nullptr) const;

  std::size_t size() const;
  std::size_t dim() const noexcept { return dim_; }
  Metric metric() const noexcept { return metric_; }

  /// Host view of stored vector i (normalized for cosine). The rows live on the GPU; the first
  /// call after an add() copies the new rows into a host mirror, which a later add() may move, so
  /// the pointer is valid until the next add(). Returns nullptr if i is out of range or the copy
  /// fails.
  const float* vector(std::size_t i) const noexcept;
  Label label(std::size_t i) const noexcept;

  void save(const std::string& path) const;
  static FlatIndex load(const std::string& path, const LoadOptions& options = {});

  /// GPU build addition: the C ABI handle, for the _device entry points of include/qv_gpu.h.
  qv_flat* handle() const noexcept { return handle_; }

 private:
  FlatIndex(qv_flat* handle, std::size_t dim, Metric metric);

  qv_flat* handle_ = nullptr;
  std::size_t dim_;
  Metric metric_;
  std::vector<Label> labels_;
  std::unique_ptr<std::shared_mutex> mu_ = std::make_unique<std::shared_mutex>();
  // host mirror of the stored rows for vector(i), filled on demand
  mutable std::vector<float> mirror_;
  mutable std::size_t mirrored_ = 0;
  std::unique_ptr<std::mutex> mirror_mu_ = std::make_unique<std::mutex>();
};

}  // namespace quiver
