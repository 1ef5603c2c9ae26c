// Glue between the quiver C++ API classes and the qv_* C ABI: status codes to quiver::Error, the
// process-wide device choice, and Filter objects to the qv_filter forms the GPU consumes.
#pragma once

#include <cstdint>
#include <functional>
#include <vector>

#include "qv_gpu.h"
#include "quiver/common.h"
#include "quiver/filter.h"
#include "quiver/thread_pool.h"

namespace quiver::bridge {

/// Throws quiver::Error carrying qv_last_error() unless status is QV_OK.
void check(qv_status status);

/// A Filter converted for one search call. `get()` is null when there is no filter.
class FilterArg {
 public:
  FilterArg() = default;
  FilterArg(FilterArg&&) noexcept = default;  // a moved vector keeps its buffer, so f_.data holds
  FilterArg(const FilterArg&) = delete;
  FilterArg& operator=(const FilterArg&) = delete;

  const qv_filter* get() const noexcept { return present_ ? &f_ : nullptr; }

  /// BitsetFilter -> its words (QV_FILTER_LABEL_BITMAP); a filter that enumerates -> the label
  /// list (QV_FILTER_LABEL_SET); any other -> contains() evaluated once per stored label, in the
  /// storage order `stored` reports (QV_FILTER_POSITION_BITMAP), split over `pool` when given.
  static FilterArg from(const Filter* filter,
                        const std::function<std::vector<Label>()>& stored, ThreadPool* pool);

 private:
  qv_filter f_{};
  std::vector<std::uint64_t> data_;
  bool present_ = false;
};

}  // namespace quiver::bridge
