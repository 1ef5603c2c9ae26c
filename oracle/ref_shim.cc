// Test infrastructure only: a C-ABI shim over the reference Quiver library, compiled from the
// reference's own sources (see oracle/Makefile) into oracle/_ref/libquiver_ref.so.
//
// It lets the Python tests, the golden-fixture generator and bench.py's CPU-baseline leg call the
// reference's unmodified C++ implementation through ctypes. Nothing in the product links it.
// Every entry point catches quiver::Error and returns -1 with the message available from
// qvref_last_error(); 0 means success.
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "internal/centroid_table.h"
#include "quiver/distance.h"
#include "quiver/filter.h"
#include "quiver/flat_index.h"
#include "quiver/hnsw_index.h"
#include "quiver/ivfpq_index.h"
#include "quiver/quantizer.h"
#include "quiver/thread_pool.h"

namespace {

thread_local std::string g_error;

template <class F>
int guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

quiver::ThreadPool* pool_for(int threads) {
  static std::vector<std::unique_ptr<quiver::ThreadPool>> pools(1025);
  if (threads <= 0) return &quiver::ThreadPool::global();
  if (threads > 1024) threads = 1024;
  auto& p = pools[static_cast<std::size_t>(threads)];
  if (!p) p = std::make_unique<quiver::ThreadPool>(static_cast<std::size_t>(threads));
  return p.get();
}

// Same choice as the reference binding's make_filter (python/quiver_ext.cc:40-51).
std::unique_ptr<quiver::Filter> make_filter(const std::uint64_t* allowed, std::size_t n) {
  std::uint64_t max_label = 0;
  for (std::size_t i = 0; i < n; ++i) max_label = allowed[i] > max_label ? allowed[i] : max_label;
  if (max_label < (std::uint64_t{1} << 32) && max_label / 64 <= 16 * n + 1024) {
    auto f = std::make_unique<quiver::BitsetFilter>(static_cast<std::size_t>(max_label) + 1);
    for (std::size_t i = 0; i < n; ++i) f->insert(allowed[i]);
    return f;
  }
  return std::make_unique<quiver::LabelSetFilter>(allowed, allowed + n);
}

}  // namespace

extern "C" {

const char* qvref_last_error() { return g_error.c_str(); }

const char* qvref_simd_isa() {
  static std::string s(quiver::simd::to_string(quiver::simd::active().isa));
  return s.c_str();
}

unsigned qvref_hardware_threads() {
  return static_cast<unsigned>(quiver::ThreadPool::global().num_threads());
}

float qvref_dot(const float* a, const float* b, std::size_t dim) {
  return quiver::simd::active().dot(a, b, dim);
}

float qvref_l2sqr(const float* a, const float* b, std::size_t dim) {
  return quiver::simd::active().l2sqr(a, b, dim);
}

void qvref_normalize_rows(float* v, std::size_t n, std::size_t dim) {
  for (std::size_t i = 0; i < n; ++i) quiver::simd::normalize(v + i * dim, dim);
}

// ---- FlatIndex ----------------------------------------------------------------------------------

int qvref_flat_new(std::size_t dim, std::uint32_t metric, void** out) {
  return guard([&] { *out = new quiver::FlatIndex(dim, static_cast<quiver::Metric>(metric)); });
}

void qvref_flat_free(void* h) { delete static_cast<quiver::FlatIndex*>(h); }

int qvref_flat_add(void* h, const float* x, std::size_t n, const std::uint64_t* labels) {
  return guard([&] { static_cast<quiver::FlatIndex*>(h)->add(x, n, labels); });
}

int qvref_flat_search(void* h, const float* q, std::size_t nq, std::size_t k,
                      const std::uint64_t* allowed, std::size_t n_allowed, int has_filter,
                      int threads, std::uint64_t* labels, float* dists) {
  return guard([&] {
    std::unique_ptr<quiver::Filter> f;
    if (has_filter) f = make_filter(allowed, n_allowed);
    static_cast<quiver::FlatIndex*>(h)->search_batch(q, nq, k, labels, dists, f.get(),
                                                     pool_for(threads));
  });
}

// Stored (normalized for cosine) row i, as the reference holds it.
int qvref_flat_vectors(void* h, float* out) {
  return guard([&] {
    auto* ix = static_cast<quiver::FlatIndex*>(h);
    const std::size_t n = ix->size(), d = ix->dim();
    for (std::size_t i = 0; i < n; ++i) std::memcpy(out + i * d, ix->vector(i), d * sizeof(float));
  });
}

int qvref_flat_save(void* h, const char* path) {
  return guard([&] { static_cast<quiver::FlatIndex*>(h)->save(path); });
}

// ---- IvfPqIndex ---------------------------------------------------------------------------------

int qvref_ivf_new(std::size_t dim, std::uint32_t metric, std::size_t nlist, std::size_t m,
                  int store_vectors, std::size_t train_iterations, std::uint64_t seed, void** out) {
  return guard([&] {
    quiver::IvfPqParams p;
    p.dim = dim;
    p.metric = static_cast<quiver::Metric>(metric);
    p.nlist = nlist;
    p.m = m;
    p.store_vectors = store_vectors != 0;
    p.train_iterations = train_iterations;
    p.seed = seed;
    *out = new quiver::IvfPqIndex(p);
  });
}

void qvref_ivf_free(void* h) { delete static_cast<quiver::IvfPqIndex*>(h); }

int qvref_ivf_train(void* h, const float* x, std::size_t n, int threads) {
  return guard([&] { static_cast<quiver::IvfPqIndex*>(h)->train(x, n, pool_for(threads)); });
}

int qvref_ivf_add(void* h, const float* x, std::size_t n, const std::uint64_t* labels,
                  int threads) {
  return guard(
      [&] { static_cast<quiver::IvfPqIndex*>(h)->add(x, n, labels, pool_for(threads)); });
}

int qvref_ivf_save(void* h, const char* path) {
  return guard([&] { static_cast<quiver::IvfPqIndex*>(h)->save(path); });
}

int qvref_ivf_load(const char* path, void** out) {
  return guard([&] { *out = new quiver::IvfPqIndex(quiver::IvfPqIndex::load(path)); });
}

std::size_t qvref_ivf_size(void* h) { return static_cast<quiver::IvfPqIndex*>(h)->size(); }

int qvref_ivf_search(void* h, const float* q, std::size_t nq, std::size_t k, std::size_t nprobe,
                     std::size_t refine_factor, const std::uint64_t* allowed,
                     std::size_t n_allowed, int has_filter, int threads, std::uint64_t* labels,
                     float* dists) {
  return guard([&] {
    std::unique_ptr<quiver::Filter> f;
    if (has_filter) f = make_filter(allowed, n_allowed);
    quiver::IvfPqSearchParams p;
    p.nprobe = nprobe;
    p.refine_factor = refine_factor;
    p.filter = f.get();
    static_cast<quiver::IvfPqIndex*>(h)->search_batch(q, nq, k, labels, dists, p,
                                                      pool_for(threads));
  });
}

// ---- building blocks (coarse assignment, PQ encode, tables) -------------------------------------

int qvref_nearest_batch(const float* centroids, std::size_t k, std::size_t dim, const float* x,
                        std::size_t n, int max_inner_product, std::uint32_t* out) {
  return guard([&] {
    quiver::internal::CentroidTable t(centroids, k, dim);
    std::vector<std::size_t> best(n);
    t.nearest_batch(x, n, best.data(), max_inner_product != 0);
    for (std::size_t i = 0; i < n; ++i) out[i] = static_cast<std::uint32_t>(best[i]);
  });
}

int qvref_pq_encode(const float* codebooks, std::size_t dim, std::size_t m, const float* x,
                    std::size_t n, std::uint8_t* codes) {
  return guard([&] {
    quiver::ProductQuantizer pq(dim, m);
    pq.set_centroids(std::vector<float>(codebooks, codebooks + 256 * dim));
    for (std::size_t i = 0; i < n; ++i) pq.encode(x + i * dim, codes + i * m);
  });
}

int qvref_pq_tables(const float* codebooks, std::size_t dim, std::size_t m, const float* q,
                    float* ip_table, float* l2_table) {
  return guard([&] {
    quiver::ProductQuantizer pq(dim, m);
    pq.set_centroids(std::vector<float>(codebooks, codebooks + 256 * dim));
    pq.compute_ip_table(q, ip_table);
    pq.compute_l2_table(q, l2_table);
  });
}

// ---- SQ8 kernels, ScalarQuantizer and HnswIndex (the filtered exact-scan fallback) --------------

float qvref_l2sqr_sq8(const float* q, const std::uint8_t* code, const float* vmin,
                      const float* vscale, std::size_t dim) {
  return quiver::simd::active().l2sqr_sq8(q, code, vmin, vscale, dim);
}

float qvref_dot_sq8(const float* q, const std::uint8_t* code, const float* vmin,
                    const float* vscale, std::size_t dim) {
  return quiver::simd::active().dot_sq8(q, code, vmin, vscale, dim);
}

int qvref_sq8_train(const float* x, std::size_t n, std::size_t dim, float* vmin, float* vscale) {
  return guard([&] {
    quiver::ScalarQuantizer sq(dim);
    sq.train(x, n);
    std::memcpy(vmin, sq.vmin(), dim * sizeof(float));
    std::memcpy(vscale, sq.vscale(), dim * sizeof(float));
  });
}

int qvref_sq8_encode(const float* vmin, const float* vscale, std::size_t dim, const float* x,
                     std::size_t n, std::uint8_t* codes) {
  return guard([&] {
    quiver::ScalarQuantizer sq(dim);
    sq.set_params(std::vector<float>(vmin, vmin + dim), std::vector<float>(vscale, vscale + dim));
    for (std::size_t i = 0; i < n; ++i) sq.encode(x + i * dim, codes + i * dim);
  });
}

// storage: 0 = float32, 1 = SQ8 (quiver::Storage).
int qvref_hnsw_new(std::size_t dim, std::uint32_t metric, std::uint32_t storage, std::size_t M,
                   std::size_t ef_construction, std::uint64_t seed, void** out) {
  return guard([&] {
    quiver::HnswParams p;
    p.dim = dim;
    p.metric = static_cast<quiver::Metric>(metric);
    p.storage = static_cast<quiver::Storage>(storage);
    p.M = M;
    p.ef_construction = ef_construction;
    p.seed = seed;
    *out = new quiver::HnswIndex(p);
  });
}

void qvref_hnsw_free(void* h) { delete static_cast<quiver::HnswIndex*>(h); }

int qvref_hnsw_train(void* h, const float* x, std::size_t n) {
  return guard([&] { static_cast<quiver::HnswIndex*>(h)->train(x, n); });
}

int qvref_hnsw_add(void* h, const float* x, std::size_t n, const std::uint64_t* labels,
                   int threads) {
  return guard(
      [&] { static_cast<quiver::HnswIndex*>(h)->add(x, n, labels, pool_for(threads)); });
}

int qvref_hnsw_remove(void* h, std::uint64_t label) {
  return static_cast<quiver::HnswIndex*>(h)->remove(label) ? 1 : 0;
}

// The stored vector of `label` as the index holds it (decoded for SQ8, normalized for cosine).
int qvref_hnsw_vector(void* h, std::uint64_t label, float* out) {
  return guard([&] {
    const std::vector<float> v = static_cast<quiver::HnswIndex*>(h)->get_vector(label);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

// Searches with an allowed-label filter; exact_scan_threshold as HnswSearchParams (1.0 makes every
// filter whose cardinality is known take the exact scan).
int qvref_hnsw_search(void* h, const float* q, std::size_t nq, std::size_t k, std::size_t ef,
                      const std::uint64_t* allowed, std::size_t n_allowed, int has_filter,
                      double exact_scan_threshold, int threads, std::uint64_t* labels,
                      float* dists) {
  return guard([&] {
    std::unique_ptr<quiver::Filter> f;
    if (has_filter) f = make_filter(allowed, n_allowed);
    quiver::HnswSearchParams p;
    p.ef = ef;
    p.filter = f.get();
    p.exact_scan_threshold = exact_scan_threshold;
    static_cast<quiver::HnswIndex*>(h)->search_batch(q, nq, k, labels, dists, p,
                                                     pool_for(threads));
  });
}

}  // extern "C"
