// quiver::to_string / parse_metric / detail::throw_error (reference src/common.cc:5-27), the
// GPU device choice of quiver/gpu.h, and the C ABI bridge of bridge.h.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <string>

#include "bridge.h"
#include "quiver/gpu.h"

namespace quiver {

std::string_view to_string(Metric metric) noexcept {
  switch (metric) {
    case Metric::kL2: return "l2";
    case Metric::kInnerProduct: return "ip";
    case Metric::kCosine: return "cosine";
  }
  return "unknown";
}

Metric parse_metric(std::string_view name) {
  static constexpr struct {
    std::string_view name;
    Metric metric;
  } kNames[] = {{"l2", Metric::kL2},           {"euclidean", Metric::kL2},
                {"ip", Metric::kInnerProduct}, {"inner_product", Metric::kInnerProduct},
                {"dot", Metric::kInnerProduct}, {"cosine", Metric::kCosine},
                {"cos", Metric::kCosine},       {"angular", Metric::kCosine}};
  for (const auto& e : kNames) {
    if (e.name == name) return e.metric;
  }
  throw Error("unknown metric '" + std::string(name) + "' (expected l2, ip, or cosine)");
}

namespace detail {
void throw_error(const std::string& message) { throw Error(message); }
}  // namespace detail

namespace gpu {
namespace {
std::atomic<int> g_device{-1};
}

void set_device(int device) {
  QUIVER_CHECK(device >= 0, "device must be non-negative");
  g_device.store(device);
}

int device() {
  int d = g_device.load();
  if (d >= 0) return d;
  const char* env = std::getenv("QUIVER_DEVICE");
  d = env != nullptr ? std::atoi(env) : 0;
  return d < 0 ? 0 : d;
}

int device_count() noexcept {
  int n = 0;
  return qv_device_count(&n) == QV_OK ? n : 0;
}
}  // namespace gpu

namespace bridge {

void check(qv_status status) {
  if (status == QV_OK) return;
  const char* msg = qv_last_error();
  throw Error(msg != nullptr && msg[0] != '\0' ? std::string(msg)
                                               : "GPU call failed with status " +
                                                     std::to_string(static_cast<int>(status)));
}

FilterArg FilterArg::from(const Filter* filter, const std::function<std::vector<Label>()>& stored,
                          ThreadPool* pool) {
  FilterArg a;
  if (filter == nullptr) return a;
  a.present_ = true;
  if (const auto* bits = dynamic_cast<const BitsetFilter*>(filter)) {
    a.f_ = {QV_FILTER_LABEL_BITMAP, bits->words(), bits->universe()};
    return a;
  }
  const bool listed = filter->for_each([&](Label l) { a.data_.push_back(l); });
  if (listed) {
    a.f_ = {QV_FILTER_LABEL_SET, a.data_.data(), a.data_.size()};
    return a;
  }
  // Opaque predicate: one contains() call per stored row, 64 rows per output word.
  a.data_.clear();
  const std::vector<Label> labels = stored();
  const std::size_t n = labels.size();
  a.data_.assign(std::max<std::size_t>(1, (n + 63) / 64), 0);
  auto fill = [&](std::size_t wb, std::size_t we) {
    for (std::size_t w = wb; w < we; ++w) {
      std::uint64_t word = 0;
      const std::size_t end = std::min(n, (w + 1) * 64);
      for (std::size_t i = w * 64; i < end; ++i) {
        if (filter->contains(labels[i])) word |= std::uint64_t{1} << (i & 63);
      }
      a.data_[w] = word;
    }
  };
  const std::size_t words = (n + 63) / 64;
  if (pool != nullptr && words > 1) {
    pool->parallel_for(words, 64, fill);
  } else {
    fill(0, words);
  }
  a.f_ = {QV_FILTER_POSITION_BITMAP, a.data_.data(), n};
  return a;
}

}  // namespace bridge
}  // namespace quiver
