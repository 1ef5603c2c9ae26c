// Quiver's shared vocabulary (labels, metrics, neighbours, load options, errors), kept
// declaration-for-declaration with the reference's include/quiver/common.h:1-76 so that code
// written against Quiver compiles unchanged against the GPU build.
#pragma once

#include <cstddef>
#include <cstdint>
#include <limits>
#include <stdexcept>
#include <string>
#include <string_view>

namespace quiver {

/// Identifier the caller attaches to each stored vector.
using Label = std::uint64_t;

/// Row number inside an index's storage.
using NodeId = std::uint32_t;

/// Upper bound on vector dimensionality.
inline constexpr std::size_t kMaxDimension = 65536;

/// Label written into result slots that have no neighbour (k larger than what the index or the
/// filter can supply). It cannot be used as a real label.
inline constexpr Label kInvalidLabel = std::numeric_limits<Label>::max();

/// Distances always grow with dissimilarity:
///   kL2            squared Euclidean distance
///   kInnerProduct  1 - <q, x>
///   kCosine        1 - <q, x> / (|q| |x|); stored rows and queries are normalized
enum class Metric : std::uint32_t { kL2 = 0, kInnerProduct = 1, kCosine = 2 };

std::string_view to_string(Metric metric) noexcept;
/// "l2"/"euclidean", "ip"/"inner_product"/"dot", "cosine"/"cos"/"angular"; anything else throws.
Metric parse_metric(std::string_view name);

struct Neighbor {
  float distance;
  Label label;

  /// Closer first; equal distances order by label.
  friend constexpr bool operator<(const Neighbor& a, const Neighbor& b) noexcept {
    if (a.distance != b.distance) return a.distance < b.distance;
    return a.label < b.label;
  }
  friend constexpr bool operator==(const Neighbor&, const Neighbor&) noexcept = default;
};

/// How load() reads an index file.
struct LoadOptions {
  /// Only meaningful for graph indexes in the reference; the GPU indexes always read the file and
  /// upload it to device memory, so this flag is accepted and ignored.
  bool mmap = false;
  /// Check every section's CRC-32C while loading (the header, the section table and the
  /// structural checks always run).
  bool verify_checksums = true;
};

/// Every recoverable failure (bad argument, unreadable or corrupt file, device failure) is thrown
/// as this type.
class Error : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

namespace detail {
[[noreturn]] void throw_error(const std::string& message);
}  // namespace detail

}  // namespace quiver

/// Throws quiver::Error(message) unless `cond` holds; `message` is evaluated only on failure.
#define QUIVER_CHECK(cond, message)             \
  do {                                          \
    if (!(cond)) [[unlikely]] {                 \
      ::quiver::detail::throw_error((message)); \
    }                                           \
  } while (0)
