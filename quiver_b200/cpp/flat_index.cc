// quiver::FlatIndex over the qv_flat C ABI. Argument checks and messages follow the reference's
// src/flat_index.cc:40-176; the search itself runs on the GPU (quiver_b200/csrc/flat.cu,
// flat_tc.cu) and returns what search_one (src/flat_index.cc:69-107) returns.
#include "quiver/flat_index.h"

#include <utility>

#include "bridge.h"
#include "quiver/gpu.h"

namespace quiver {

FlatIndex::FlatIndex(std::size_t dim, Metric metric) : dim_(dim), metric_(metric) {
  QUIVER_CHECK(dim >= 1 && dim <= kMaxDimension,
               "dimension must be in [1, " + std::to_string(kMaxDimension) + "]");
  QUIVER_CHECK(metric == Metric::kL2 || metric == Metric::kInnerProduct ||
                   metric == Metric::kCosine,
               "unknown metric");
  bridge::check(qv_flat_create(gpu::device(), dim, static_cast<std::uint32_t>(metric), &handle_));
}

FlatIndex::FlatIndex(qv_flat* handle, std::size_t dim, Metric metric)
    : handle_(handle), dim_(dim), metric_(metric) {}

FlatIndex::~FlatIndex() {
  if (handle_ != nullptr) qv_flat_destroy(handle_);
}

FlatIndex::FlatIndex(FlatIndex&& other) noexcept
    : handle_(std::exchange(other.handle_, nullptr)),
      dim_(other.dim_),
      metric_(other.metric_),
      labels_(std::move(other.labels_)),
      mu_(std::move(other.mu_)),
      mirror_(std::move(other.mirror_)),
      mirrored_(std::exchange(other.mirrored_, 0)),
      mirror_mu_(std::move(other.mirror_mu_)) {}

FlatIndex& FlatIndex::operator=(FlatIndex&& other) noexcept {
  if (this != &other) {
    if (handle_ != nullptr) qv_flat_destroy(handle_);
    handle_ = std::exchange(other.handle_, nullptr);
    dim_ = other.dim_;
    metric_ = other.metric_;
    labels_ = std::move(other.labels_);
    mu_ = std::move(other.mu_);
    mirror_ = std::move(other.mirror_);
    mirrored_ = std::exchange(other.mirrored_, 0);
    mirror_mu_ = std::move(other.mirror_mu_);
  }
  return *this;
}

void FlatIndex::add(const float* vectors, std::size_t n, const Label* labels) {
  if (n == 0) return;
  QUIVER_CHECK(vectors != nullptr, "vectors must not be null");
  std::unique_lock lock(*mu_);
  bridge::check(qv_flat_add(handle_, vectors, n, labels));  // validates, normalizes, uploads
  const std::size_t first = labels_.size();
  labels_.reserve(first + n);
  for (std::size_t i = 0; i < n; ++i) labels_.push_back(labels != nullptr ? labels[i] : first + i);
}

std::vector<Neighbor> FlatIndex::search(const float* query, std::size_t k,
                                        const Filter* filter) const {
  QUIVER_CHECK(query != nullptr, "query must not be null");
  std::vector<Label> labels(k);
  std::vector<float> distances(k);
  search_batch(query, 1, k, labels.data(), distances.data(), filter, nullptr);
  std::vector<Neighbor> out;
  out.reserve(k);
  for (std::size_t j = 0; j < k && labels[j] != kInvalidLabel; ++j) {
    out.push_back({distances[j], labels[j]});
  }
  return out;
}

void FlatIndex::search_batch(const float* queries, std::size_t nq, std::size_t k, Label* labels,
                             float* distances, const Filter* filter, ThreadPool* pool) const {
  if (nq == 0 || k == 0) return;
  QUIVER_CHECK(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
  std::shared_lock lock(*mu_);
  const auto f = bridge::FilterArg::from(filter, [this] { return labels_; }, pool);
  static_assert(sizeof(Label) == sizeof(std::uint64_t));
  bridge::check(qv_flat_search(handle_, queries, nq, k, f.get(), labels, distances));
}

std::size_t FlatIndex::size() const {
  std::shared_lock lock(*mu_);
  return labels_.size();
}

const float* FlatIndex::vector(std::size_t i) const noexcept {
  try {
    std::lock_guard<std::mutex> lk(*mirror_mu_);
    if (i >= mirrored_) {
      std::size_t n = 0;
      if (qv_flat_info(handle_, &n, nullptr, nullptr) != QV_OK || i >= n) return nullptr;
      mirror_.resize(n * dim_);
      if (qv_flat_rows(handle_, mirrored_, n - mirrored_, mirror_.data() + mirrored_ * dim_,
                       nullptr) != QV_OK)
        return nullptr;
      mirrored_ = n;
    }
    return mirror_.data() + i * dim_;
  } catch (...) {
    return nullptr;
  }
}

Label FlatIndex::label(std::size_t i) const noexcept { return labels_[i]; }

void FlatIndex::save(const std::string& path) const {
  std::shared_lock lock(*mu_);
  bridge::check(qv_flat_save(handle_, path.c_str()));
}

FlatIndex FlatIndex::load(const std::string& path, const LoadOptions& options) {
  qv_flat* h = nullptr;
  bridge::check(qv_flat_load(gpu::device(), path.c_str(), options.verify_checksums ? 1 : 0, &h));
  std::size_t n = 0, dim = 0;
  std::uint32_t metric = 0;
  const qv_status st = qv_flat_info(h, &n, &dim, &metric);
  if (st != QV_OK) qv_flat_destroy(h);
  bridge::check(st);
  FlatIndex index(h, dim, static_cast<Metric>(metric));  // owns h from here on
  index.labels_.resize(n);
  bridge::check(qv_flat_rows(h, 0, n, nullptr, index.labels_.data()));
  return index;
}

}  // namespace quiver
