// IVF-PQ index (coarse cells + product-quantized residuals), with the interface of the reference's
// include/quiver/ivfpq_index.h:24-81. Cells, codes, labels and optional raw vectors live in GPU
// memory; add() assigns and encodes on the GPU, and search runs the coarse probe, the residual
// lookup tables, the ADC scan and the optional exact re-rank there (qv_ivfpq_* in
// include/qv_gpu.h), with the reference's assignments, codes and distances.
//
// train() gives the reference's centroids and codebooks bit for bit, with its k-means assignment
// steps on the GPU. A trained index can also come from load() of a .qvr file written by the
// reference (or by save()), or from set_trained() with centroids and codebooks trained elsewhere.
//
// Thread-safe: searches may run concurrently; add() encodes outside the lock and excludes
// searches only while it appends.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "quiver/common.h"
#include "quiver/filter.h"
#include "quiver/thread_pool.h"

struct qv_ivfpq;

namespace quiver {

struct IvfPqParams {
  std::size_t dim = 0;
  Metric metric = Metric::kL2;
  std::size_t nlist = 1024;  ///< coarse cells
  std::size_t m = 16;        ///< sub-quantizers = code bytes per vector; divides dim
  std::size_t train_iterations = 20;
  /// Keep float32 copies of the vectors so that refine_factor can re-rank exactly.
  bool store_vectors = false;
  std::uint64_t seed = 1234;
};

struct IvfPqSearchParams {
  std::size_t nprobe = 16;
  /// With store_vectors: re-rank the best k * refine_factor ADC candidates exactly (0 = off).
  std::size_t refine_factor = 0;
  const Filter* filter = nullptr;
};

class IvfPqIndex {
 public:
  explicit IvfPqIndex(const IvfPqParams& params);
  ~IvfPqIndex();
  IvfPqIndex(IvfPqIndex&&) noexcept;
  IvfPqIndex& operator=(IvfPqIndex&&) noexcept;

  /// Not available on the GPU build: throws Error (an index is trained at most once in the
  /// reference too; here the trained state comes from load() or set_trained()).
  void train(const float* vectors, std::size_t n, ThreadPool* pool = nullptr);
  bool is_trained() const noexcept;

  /// GPU build addition: installs nlist x dim coarse centroids and m x 256 x (dim / m) PQ
  /// codebooks, as load() does with a file's sections. Throws if already trained.
  void set_trained(const float* centroids, const float* codebooks);

  /// labels == nullptr labels vector i as size() + i. `pool` is accepted and unused (the
  /// assignment and encoding run on the GPU).
  void add(const float* vectors, std::size_t n, const Label* labels = nullptr,
           ThreadPool* pool = nullptr);

  std::vector<Neighbor> search(const float* query, std::size_t k,
                               const IvfPqSearchParams& params = {}) const;
  void search_batch(const float* queries, std::size_t nq, std::size_t k, Label* labels,
                    float* distances, const IvfPqSearchParams& params = {},
                    ThreadPool* pool = nullptr) const;

  void save(const std::string& path) const;
  static IvfPqIndex load(const std::string& path, const LoadOptions& options = {});

  std::size_t size() const noexcept;
  std::size_t dim() const noexcept;
  const IvfPqParams& params() const noexcept;
  /// Bytes of centroids, codebooks, precomputed terms, codes, labels and stored vectors.
  std::size_t memory_bytes() const noexcept;
  /// Entries per cell.
  std::vector<std::size_t> list_sizes() const;

  /// GPU build addition: the C ABI handle, for the _device entry points of include/qv_gpu.h.
  qv_ivfpq* handle() const noexcept;

 private:
  struct Impl;
  explicit IvfPqIndex(std::unique_ptr<Impl> impl);
  std::unique_ptr<Impl> impl_;
};

}  // namespace quiver
