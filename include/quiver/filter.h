// Label filters that restrict a search to a subset of the stored vectors, with the class
// hierarchy of the reference's include/quiver/filter.h:24-102.
//
// On the GPU the filter becomes a bitmap with one bit per stored row, built once per search call
// before any kernel runs: a BitsetFilter crosses as its words, a filter that can enumerate its
// labels (for_each) crosses as that label list, and any other filter (a PredicateFilter) has
// contains() called once for every stored label, on the calling thread or on the ThreadPool the
// search was given. contains() must therefore be safe to call from those threads, and must not
// call into the index being searched.
#pragma once

#include <bit>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <initializer_list>
#include <optional>
#include <unordered_set>
#include <utility>
#include <vector>

#include "quiver/common.h"

namespace quiver {

class Filter {
 public:
  virtual ~Filter() = default;

  virtual bool contains(Label label) const = 0;

  /// Number of admitted labels when it is known cheaply.
  virtual std::optional<std::size_t> cardinality() const { return std::nullopt; }

  /// Calls fn once per admitted label; returns false when the filter cannot enumerate.
  virtual bool for_each(const std::function<void(Label)>& /*fn*/) const { return false; }
};

/// Bit per label over [0, universe): bit (label & 63) of word (label >> 6).
class BitsetFilter final : public Filter {
 public:
  explicit BitsetFilter(std::size_t universe) : bits_((universe + 63) / 64, 0), universe_(universe) {}

  void insert(Label label) {
    QUIVER_CHECK(label < universe_, "label outside BitsetFilter universe");
    const std::uint64_t mask = std::uint64_t{1} << (label & 63);
    std::uint64_t& word = bits_[label >> 6];
    if ((word & mask) == 0) ++admitted_;
    word |= mask;
  }

  bool contains(Label label) const override {
    return label < universe_ && (bits_[label >> 6] & (std::uint64_t{1} << (label & 63))) != 0;
  }

  std::optional<std::size_t> cardinality() const override { return admitted_; }

  bool for_each(const std::function<void(Label)>& fn) const override {
    for (std::size_t w = 0; w < bits_.size(); ++w) {
      std::uint64_t rest = bits_[w];
      while (rest != 0) {
        fn(static_cast<Label>(w * 64 + static_cast<unsigned>(std::countr_zero(rest))));
        rest &= rest - 1;
      }
    }
    return true;
  }

  /// GPU build addition: the raw words (universe() bits), which cross to the device as they are.
  const std::uint64_t* words() const noexcept { return bits_.data(); }
  std::size_t universe() const noexcept { return universe_; }

 private:
  std::vector<std::uint64_t> bits_;
  std::size_t universe_;
  std::size_t admitted_ = 0;
};

/// Any set of labels, however large their values.
class LabelSetFilter final : public Filter {
 public:
  LabelSetFilter() = default;
  LabelSetFilter(std::initializer_list<Label> labels) : set_(labels) {}
  template <class It>
  LabelSetFilter(It first, It last) : set_(first, last) {}

  void insert(Label label) { set_.insert(label); }
  bool contains(Label label) const override { return set_.find(label) != set_.end(); }
  std::optional<std::size_t> cardinality() const override { return set_.size(); }
  bool for_each(const std::function<void(Label)>& fn) const override {
    for (const Label label : set_) fn(label);
    return true;
  }

 private:
  std::unordered_set<Label> set_;
};

/// A caller-supplied predicate; it cannot enumerate, so the GPU path evaluates it per stored row.
template <class Pred>
class PredicateFilter final : public Filter {
 public:
  explicit PredicateFilter(Pred pred) : pred_(std::move(pred)) {}
  bool contains(Label label) const override { return pred_(label); }

 private:
  Pred pred_;
};

}  // namespace quiver
