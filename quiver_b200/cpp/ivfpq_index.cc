// quiver::IvfPqIndex over the qv_ivfpq C ABI. Argument checks and messages follow the reference's
// src/ivfpq_index.cc:383-463; assignment, encoding and search run on the GPU
// (quiver_b200/csrc/ivf.cu) with the results of Impl::add / Impl::search_into
// (src/ivfpq_index.cc:208-381).
#include "quiver/ivfpq_index.h"

#include <mutex>
#include <shared_mutex>
#include <utility>

#include "bridge.h"
#include "quiver/gpu.h"

namespace quiver {

struct IvfPqIndex::Impl {
  qv_ivfpq* h = nullptr;
  IvfPqParams params;
  // Held exclusively across add() and shared by searches that evaluate a filter against the
  // stored labels, so that the labels they read and the lists they scan agree.
  mutable std::shared_mutex append_mu;

  ~Impl() {
    if (h != nullptr) qv_ivfpq_destroy(h);
  }

  static IvfPqParams read_params(qv_ivfpq* h) {
    qv_ivfpq_params p{};
    bridge::check(qv_ivfpq_info(h, &p, nullptr, nullptr));
    IvfPqParams out;
    out.dim = p.dim;
    out.metric = static_cast<Metric>(p.metric);
    out.nlist = p.nlist;
    out.m = p.m;
    out.train_iterations = p.train_iterations;
    out.store_vectors = p.store_vectors != 0;
    out.seed = p.seed;
    return out;
  }

  std::vector<Label> stored_labels() const {
    std::size_t n = 0;
    bridge::check(qv_ivfpq_info(h, nullptr, &n, nullptr));
    std::vector<Label> labels(n);
    if (n != 0) bridge::check(qv_ivfpq_labels(h, labels.data()));
    return labels;
  }
};

IvfPqIndex::IvfPqIndex(const IvfPqParams& params) : impl_(std::make_unique<Impl>()) {
  const qv_ivfpq_params p{params.dim,  static_cast<std::uint32_t>(params.metric),
                          params.nlist, params.m,
                          params.train_iterations, params.store_vectors ? 1 : 0,
                          params.seed};
  bridge::check(qv_ivfpq_create(gpu::device(), &p, &impl_->h));
  impl_->params = params;
}

IvfPqIndex::IvfPqIndex(std::unique_ptr<Impl> impl) : impl_(std::move(impl)) {}
IvfPqIndex::~IvfPqIndex() = default;
IvfPqIndex::IvfPqIndex(IvfPqIndex&&) noexcept = default;
IvfPqIndex& IvfPqIndex::operator=(IvfPqIndex&&) noexcept = default;

void IvfPqIndex::train(const float* vectors, std::size_t n, ThreadPool* /*pool*/) {
  QUIVER_CHECK(vectors != nullptr, "vectors must not be null");
  bridge::check(qv_ivfpq_train(impl_->h, vectors, n));
}

bool IvfPqIndex::is_trained() const noexcept {
  int trained = 0;
  return qv_ivfpq_is_trained(impl_->h, &trained) == QV_OK && trained != 0;
}

void IvfPqIndex::set_trained(const float* centroids, const float* codebooks) {
  bridge::check(qv_ivfpq_set_trained(impl_->h, centroids, codebooks));
}

void IvfPqIndex::add(const float* vectors, std::size_t n, const Label* labels,
                     ThreadPool* /*pool*/) {
  QUIVER_CHECK(vectors != nullptr || n == 0, "vectors must not be null");
  std::unique_lock lock(impl_->append_mu);
  bridge::check(qv_ivfpq_add(impl_->h, vectors, n, labels));
}

std::vector<Neighbor> IvfPqIndex::search(const float* query, std::size_t k,
                                         const IvfPqSearchParams& params) const {
  QUIVER_CHECK(query != nullptr, "query must not be null");
  std::vector<Label> labels(k);
  std::vector<float> dist(k);
  search_batch(query, 1, k, labels.data(), dist.data(), params, nullptr);
  std::vector<Neighbor> out;
  for (std::size_t j = 0; j < k && labels[j] != kInvalidLabel; ++j) {
    out.push_back({dist[j], labels[j]});
  }
  return out;
}

void IvfPqIndex::search_batch(const float* queries, std::size_t nq, std::size_t k, Label* labels,
                              float* distances, const IvfPqSearchParams& params,
                              ThreadPool* pool) const {
  if (nq == 0 || k == 0) return;
  QUIVER_CHECK(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
  std::shared_lock<std::shared_mutex> lock(impl_->append_mu, std::defer_lock);
  if (params.filter != nullptr) lock.lock();
  const auto f = bridge::FilterArg::from(
      params.filter, [this] { return impl_->stored_labels(); }, pool);
  bridge::check(qv_ivfpq_search(impl_->h, queries, nq, k, params.nprobe, params.refine_factor,
                                f.get(), labels, distances));
}

void IvfPqIndex::save(const std::string& path) const {
  bridge::check(qv_ivfpq_save(impl_->h, path.c_str()));
}

IvfPqIndex IvfPqIndex::load(const std::string& path, const LoadOptions& options) {
  auto impl = std::make_unique<Impl>();
  bridge::check(
      qv_ivfpq_load(gpu::device(), path.c_str(), options.verify_checksums ? 1 : 0, &impl->h));
  impl->params = Impl::read_params(impl->h);
  return IvfPqIndex(std::move(impl));
}

std::size_t IvfPqIndex::size() const noexcept {
  std::size_t n = 0;
  return qv_ivfpq_info(impl_->h, nullptr, &n, nullptr) == QV_OK ? n : 0;
}

std::size_t IvfPqIndex::dim() const noexcept { return impl_->params.dim; }
const IvfPqParams& IvfPqIndex::params() const noexcept { return impl_->params; }

std::size_t IvfPqIndex::memory_bytes() const noexcept {
  std::size_t bytes = 0;
  return qv_ivfpq_info(impl_->h, nullptr, nullptr, &bytes) == QV_OK ? bytes : 0;
}

std::vector<std::size_t> IvfPqIndex::list_sizes() const {
  std::vector<std::uint64_t> sizes(impl_->params.nlist);
  bridge::check(qv_ivfpq_list_sizes(impl_->h, sizes.data()));
  return std::vector<std::size_t>(sizes.begin(), sizes.end());
}

qv_ivfpq* IvfPqIndex::handle() const noexcept { return impl_->h; }

}  // namespace quiver
