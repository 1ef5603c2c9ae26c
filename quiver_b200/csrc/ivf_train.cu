// IVF-PQ training with the assignment step on the GPU.
//
// The reference trains with Lloyd's k-means (src/product_quantizer.cc:29-117): a subsample and
// the initial centroids drawn with std::mt19937_64, an assignment of every point to its nearest
// centroid by CentroidTable::nearest_batch, cluster sums in double precision in point order,
// centroid = sum / count rounded to float, and empty clusters split from a donor chosen at random
// in proportion to its size. IvfPqIndex::train (src/ivfpq_index.cc:144-206) runs it for the coarse
// centroids (cosine rows normalized first, centroids normalized after), assigns the rows to them,
// takes residuals, draws a 65,536-row subsample of them, and trains one 256-centroid k-means per
// PQ sub-space (src/product_quantizer.cc:135-153).
//
// Here the assignment — n x k x dim multiply-adds per iteration, all of the cost — runs on the GPU
// through the same bit-exact restatement of nearest_batch that add() uses; everything that draws
// random numbers or sums into a cluster runs on the host in the reference's order, so the trained
// centroids and codebooks are bit-identical to the reference's for the same input and parameters
// (the sums are in double and in point order exactly because rounding there depends on order).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "qv_state.h"

namespace qv {
namespace {

constexpr size_t kMaxPointsPerCentroid = 256;  // KMeansParams default (include/quiver/quantizer.h:51)
constexpr size_t kPqTrainRows = 65536;         // src/ivfpq_index.cc:183

// Lloyd's k-means over the n x dim host rows x (see the file comment). The rows are uploaded once;
// each iteration uploads the centroids and downloads the assignments.
std::vector<float> kmeans(const float* x, size_t n, size_t dim, size_t k, size_t iterations,
                          uint64_t seed, cudaStream_t st) {
  QV_REQUIRE(k > 0 && dim > 0, "kmeans: k and dim must be positive");
  QV_REQUIRE(n >= k, "kmeans: need at least k=" + std::to_string(k) + " training points, got " +
                         std::to_string(n));
  std::mt19937_64 rng(seed);
  // Subsample to at most k * 256 points by a partial Fisher-Yates shuffle of the indices.
  std::vector<float> sample;
  const size_t cap = k * kMaxPointsPerCentroid;
  if (n > cap) {
    std::vector<size_t> idx(n);
    std::iota(idx.begin(), idx.end(), size_t{0});
    for (size_t i = 0; i < cap; ++i) std::swap(idx[i], idx[i + rng() % (n - i)]);
    sample.resize(cap * dim);
    for (size_t i = 0; i < cap; ++i)
      std::memcpy(sample.data() + i * dim, x + idx[i] * dim, dim * sizeof(float));
    x = sample.data();
    n = cap;
  }
  // k distinct random points start the centroids (the same partial shuffle).
  std::vector<float> cents(k * dim);
  {
    std::vector<size_t> idx(n);
    std::iota(idx.begin(), idx.end(), size_t{0});
    for (size_t i = 0; i < k; ++i) {
      std::swap(idx[i], idx[i + rng() % (n - i)]);
      std::memcpy(cents.data() + i * dim, x + idx[i] * dim, dim * sizeof(float));
    }
  }
  DeviceBuffer dx(n * dim * sizeof(float), st), dc(k * dim * sizeof(float), st),
      dn(k * sizeof(float), st), da(n * sizeof(uint32_t), st);
  QV_CUDA(cudaMemcpyAsync(dx.get(), x, n * dim * sizeof(float), cudaMemcpyHostToDevice, st));
  std::vector<uint32_t> assign(n);
  std::vector<double> sums(k * dim);
  std::vector<size_t> counts(k);
  for (size_t iter = 0; iter < iterations; ++iter) {
    QV_CUDA(cudaMemcpyAsync(dc.get(), cents.data(), k * dim * sizeof(float),
                            cudaMemcpyHostToDevice, st));
    nearest_centroids_device(dx.get<float>(), n, dc.get<float>(), k, dim, /*by_ip=*/false,
                             dn.get<float>(), da.get<uint32_t>(), st);
    QV_CUDA(cudaMemcpyAsync(assign.data(), da.get(), n * sizeof(uint32_t),
                            cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
    std::fill(sums.begin(), sums.end(), 0.0);
    std::fill(counts.begin(), counts.end(), size_t{0});
    for (size_t i = 0; i < n; ++i) {  // point order: rounding in the double sums depends on it
      const size_t c = assign[i];
      ++counts[c];
      double* sc = sums.data() + c * dim;
      const float* xi = x + i * dim;
      for (size_t j = 0; j < dim; ++j) sc[j] += static_cast<double>(xi[j]);
    }
    for (size_t c = 0; c < k; ++c) {
      if (counts[c] == 0) continue;
      const double cnt = static_cast<double>(counts[c]);
      for (size_t j = 0; j < dim; ++j)
        cents[c * dim + j] = static_cast<float>(sums[c * dim + j] / cnt);
    }
    // An empty cluster takes a clone of a donor drawn with probability proportional to its
    // size, the two copies pushed apart by +-1/1024 in alternating coordinates.
    for (size_t c = 0; c < k; ++c) {
      if (counts[c] != 0) continue;
      size_t donor;
      for (;;) {
        donor = rng() % k;
        const double share = static_cast<double>(counts[donor]) / static_cast<double>(n) *
                             static_cast<double>(k);
        if (share > std::uniform_real_distribution<double>(0.0, 1.0)(rng)) break;
      }
      const float eps = 1.0f / 1024.0f;
      for (size_t j = 0; j < dim; ++j) {
        const float v = cents[donor * dim + j];
        const float sign = (j % 2 == 0) ? 1.0f : -1.0f;
        cents[c * dim + j] = v * (1.0f + sign * eps);
        cents[donor * dim + j] = v * (1.0f - sign * eps);
      }
      counts[c] = counts[donor] / 2;
      counts[donor] -= counts[c];
    }
  }
  return cents;
}

}  // namespace

void ivf_train(IvfState& s, const float* h_in, size_t n, cudaStream_t st) {
  const size_t d = s.dim, nlist = s.nlist, m = s.m, dsub = s.dsub;
  QV_REQUIRE(n >= nlist && n >= static_cast<size_t>(kSubCentroids),
             "IVF-PQ training needs at least max(nlist, 256) vectors");
  QV_REQUIRE(!s.trained, "index is already trained");
  // Training rows, normalized like the reference's for cosine (on the GPU, bit-identical).
  std::vector<float> data(h_in, h_in + n * d);
  DeviceBuffer dx(n * d * sizeof(float), st);
  QV_CUDA(cudaMemcpyAsync(dx.get(), data.data(), n * d * sizeof(float), cudaMemcpyHostToDevice,
                          st));
  if (s.metric == QV_METRIC_COSINE) {
    normalize_rows_device(dx.get<float>(), n, d, st);
    QV_CUDA(cudaMemcpyAsync(data.data(), dx.get(), n * d * sizeof(float), cudaMemcpyDeviceToHost,
                            st));
    QV_CUDA(cudaStreamSynchronize(st));
  }
  std::vector<float> cents = kmeans(data.data(), n, d, nlist, s.train_iterations, s.seed, st);
  DeviceBuffer dc(nlist * d * sizeof(float), st), dn(nlist * sizeof(float), st),
      da(n * sizeof(uint32_t), st);
  QV_CUDA(cudaMemcpyAsync(dc.get(), cents.data(), nlist * d * sizeof(float),
                          cudaMemcpyHostToDevice, st));
  if (s.metric == QV_METRIC_COSINE) {
    normalize_rows_device(dc.get<float>(), nlist, d, st);
    QV_CUDA(cudaMemcpyAsync(cents.data(), dc.get(), nlist * d * sizeof(float),
                            cudaMemcpyDeviceToHost, st));
  }
  // Residuals of every row against its cell (assigned by inner product for the IP metric, as
  // add() assigns).
  std::vector<uint32_t> cell(n);
  nearest_centroids_device(dx.get<float>(), n, dc.get<float>(), nlist, d,
                           s.metric == QV_METRIC_IP, dn.get<float>(), da.get<uint32_t>(), st);
  QV_CUDA(cudaMemcpyAsync(cell.data(), da.get(), n * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                          st));
  QV_CUDA(cudaStreamSynchronize(st));
  std::vector<float> resid(n * d);
  for (size_t i = 0; i < n; ++i) {
    const float* x = data.data() + i * d;
    const float* c = cents.data() + static_cast<size_t>(cell[i]) * d;
    for (size_t j = 0; j < d; ++j) resid[i * d + j] = x[j] - c[j];
  }
  // A random subset of at most 65,536 residual rows, drawn by swapping rows into the front.
  const size_t pq_n = std::min(n, kPqTrainRows);
  if (pq_n < n) {
    std::mt19937_64 rng(s.seed + 2);
    for (size_t i = 0; i < pq_n; ++i) {
      const size_t j = i + rng() % (n - i);
      std::swap_ranges(resid.begin() + static_cast<std::ptrdiff_t>(i * d),
                       resid.begin() + static_cast<std::ptrdiff_t>((i + 1) * d),
                       resid.begin() + static_cast<std::ptrdiff_t>(j * d));
    }
  }
  // One 256-centroid k-means per sub-space, seeded seed + 1 + j.
  std::vector<float> books(m * kSubCentroids * dsub);
  std::vector<float> sub(pq_n * dsub);
  for (size_t j = 0; j < m; ++j) {
    for (size_t i = 0; i < pq_n; ++i)
      std::memcpy(sub.data() + i * dsub, resid.data() + i * d + j * dsub, dsub * sizeof(float));
    const std::vector<float> c =
        kmeans(sub.data(), pq_n, dsub, kSubCentroids, s.train_iterations, s.seed + 1 + j, st);
    std::copy(c.begin(), c.end(), books.begin() + static_cast<std::ptrdiff_t>(j * kSubCentroids * dsub));
  }
  ivf_set_trained(s, cents.data(), books.data(), st);
}

}  // namespace qv
