// Tests of the quiver C++ API (include/quiver/*.h) as built on the GPU library.
//
// The cases restate the behaviour the reference's own C++ tests check (tests/test_flat.cc,
// tests/test_thread_pool.cc, tests/test_regressions.cc, tests/test_quantizer.cc:140-175) against
// this build; most IVF-PQ cases start from a trained .qvr file (training itself is checked bit for
// bit against the reference in tests/test_ivf_gpu.py). The program also has two dump modes that run FlatIndex / IvfPqIndex searches on inputs
// written by tests/test_cpp_api.py, which compares the outputs with the reference's results.
//
//   api_test cpu                 host-only cases (thread pool, filters, metrics, no-GPU errors)
//   api_test gpu <ivf.qvr> <tmp> cases that need a GPU
//   api_test flat <dir>          dir/spec.txt + raw inputs -> dir/out_labels.bin, out_dists.bin
//   api_test ivf <dir>           same for IvfPqIndex::load + search_batch
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <limits>
#include <random>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "quiver/common.h"
#include "quiver/filter.h"
#include "quiver/flat_index.h"
#include "quiver/gpu.h"
#include "quiver/ivfpq_index.h"
#include "quiver/thread_pool.h"

using namespace quiver;

namespace {

int g_failures = 0;
const char* g_case = "";

#define EXPECT(cond)                                                                      \
  do {                                                                                    \
    if (!(cond)) {                                                                        \
      ++g_failures;                                                                       \
      std::fprintf(stderr, "%s:%d: [%s] expected: %s\n", __FILE__, __LINE__, g_case, #cond); \
    }                                                                                     \
  } while (0)

#define EXPECT_ERROR(stmt)                       \
  do {                                           \
    bool thrown_ = false;                        \
    try {                                        \
      stmt;                                      \
    } catch (const quiver::Error&) {             \
      thrown_ = true;                            \
    }                                            \
    EXPECT(thrown_ && "throws quiver::Error: " #stmt); \
  } while (0)

struct Case {
  const char* name;
  std::function<void()> fn;
};

int run(const std::vector<Case>& cases) {
  for (const auto& c : cases) {
    g_case = c.name;
    const int before = g_failures;
    try {
      c.fn();
    } catch (const std::exception& e) {
      ++g_failures;
      std::fprintf(stderr, "[%s] unexpected exception: %s\n", c.name, e.what());
    }
    std::printf("%-48s %s\n", c.name, g_failures == before ? "ok" : "FAILED");
  }
  std::printf("%d failure(s)\n", g_failures);
  return g_failures == 0 ? 0 : 1;
}

std::vector<float> normal_rows(std::size_t n, std::size_t dim, std::uint64_t seed) {
  std::mt19937_64 gen(seed);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  std::vector<float> v(n * dim);
  for (auto& x : v) x = nd(gen);
  return v;
}

// ---- thread pool (tests/test_thread_pool.cc) ---------------------------------------------------

void pool_covers_every_index_once() {
  ThreadPool pool(4);
  for (std::size_t grain : {1, 3, 64, 1000}) {
    std::vector<std::atomic<int>> hits(997);
    pool.parallel_for(hits.size(), grain, [&](std::size_t b, std::size_t e) {
      for (std::size_t i = b; i < e; ++i) hits[i].fetch_add(1);
    });
    bool once = true;
    for (auto& h : hits) once = once && h.load() == 1;
    EXPECT(once);
  }
  pool.parallel_for(0, 1, [&](std::size_t, std::size_t) { EXPECT(false); });
}

void pool_runs_in_parallel() {
  // Two chunks that each wait for the other can only both finish if they run at once.
  ThreadPool pool(2);
  std::atomic<int> arrived{0};
  std::atomic<bool> met{true};
  pool.parallel_for(2, 1, [&](std::size_t, std::size_t) {
    arrived.fetch_add(1);
    const auto until = std::chrono::steady_clock::now() + std::chrono::seconds(10);
    while (arrived.load() < 2) {
      if (std::chrono::steady_clock::now() > until) {
        met = false;
        return;
      }
      std::this_thread::yield();
    }
  });
  EXPECT(met.load());
}

void pool_propagates_first_exception() {
  ThreadPool pool(4);
  std::atomic<int> ran{0};
  bool caught = false;
  try {
    pool.parallel_for(1000, 1, [&](std::size_t b, std::size_t) {
      ran.fetch_add(1);
      if (b == 0) throw std::runtime_error("chunk 0 failed");
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    });
  } catch (const std::runtime_error& e) {
    caught = std::string(e.what()) == "chunk 0 failed";
  }
  EXPECT(caught);
  EXPECT(ran.load() < 1000);  // later chunks were skipped
  std::atomic<int> total{0};
  pool.parallel_for(100, 7, [&](std::size_t b, std::size_t e) { total += int(e - b); });
  EXPECT(total.load() == 100);  // still usable
}

void pool_nested_runs_inline() {
  ThreadPool pool(4);
  std::atomic<int> total{0};
  pool.parallel_for(8, 1, [&](std::size_t, std::size_t) {
    const auto self = std::this_thread::get_id();
    pool.parallel_for(16, 1, [&](std::size_t b, std::size_t e) {
      EXPECT(std::this_thread::get_id() == self);
      total += int(e - b);
    });
  });
  EXPECT(total.load() == 8 * 16);
}

void pool_concurrent_callers_serialized() {
  ThreadPool pool(3);
  std::atomic<int> inside{0}, worst{0};
  auto caller = [&] {
    for (int r = 0; r < 20; ++r) {
      pool.parallel_for(6, 1, [&](std::size_t, std::size_t) {
        const int now = inside.fetch_add(1) + 1;
        int w = worst.load();
        while (now > w && !worst.compare_exchange_weak(w, now)) {
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
        inside.fetch_sub(1);
      });
    }
  };
  std::thread a(caller), b(caller);
  a.join();
  b.join();
  EXPECT(worst.load() <= 3);  // never more chunks at once than the pool has threads
}

void pool_single_thread_inline() {
  ThreadPool pool(1);
  EXPECT(pool.num_threads() == 1);
  const auto self = std::this_thread::get_id();
  int total = 0;
  pool.parallel_for(10, 3, [&](std::size_t b, std::size_t e) {
    EXPECT(std::this_thread::get_id() == self);
    total += int(e - b);
  });
  EXPECT(total == 10);
}

void pool_cross_pool_nesting() {
  ThreadPool outer(3), inner(3);
  std::atomic<int> total{0};
  outer.parallel_for(6, 1, [&](std::size_t, std::size_t) {
    inner.parallel_for(5, 1, [&](std::size_t b, std::size_t e) { total += int(e - b); });
  });
  EXPECT(total.load() == 30);
  EXPECT(ThreadPool::global().num_threads() >= 1);
}

// ---- vocabulary and filters --------------------------------------------------------------------

void metrics_and_neighbors() {
  EXPECT(parse_metric("l2") == Metric::kL2);
  EXPECT(parse_metric("euclidean") == Metric::kL2);
  EXPECT(parse_metric("inner_product") == Metric::kInnerProduct);
  EXPECT(parse_metric("dot") == Metric::kInnerProduct);
  EXPECT(parse_metric("angular") == Metric::kCosine);
  EXPECT(to_string(Metric::kCosine) == "cosine");
  EXPECT_ERROR(parse_metric("hamming"));
  EXPECT((Neighbor{1.0f, 9} < Neighbor{2.0f, 1}));
  EXPECT((Neighbor{1.0f, 1} < Neighbor{1.0f, 2}));
  EXPECT((Neighbor{1.0f, 1} == Neighbor{1.0f, 1}));
  EXPECT(kInvalidLabel == std::numeric_limits<std::uint64_t>::max());
  EXPECT_ERROR(QUIVER_CHECK(1 + 1 == 3, "arithmetic"));
}

void filters() {
  BitsetFilter bits(130);
  bits.insert(0);
  bits.insert(64);
  bits.insert(129);
  bits.insert(64);
  EXPECT(bits.cardinality() == std::optional<std::size_t>(3));
  EXPECT(bits.contains(129) && !bits.contains(128) && !bits.contains(5000));
  EXPECT_ERROR(bits.insert(130));
  std::vector<Label> seen;
  EXPECT(bits.for_each([&](Label l) { seen.push_back(l); }));
  EXPECT((seen == std::vector<Label>{0, 64, 129}));
  EXPECT(bits.universe() == 130 && bits.words()[1] == 1);

  LabelSetFilter set({5, std::uint64_t{1} << 40});
  EXPECT(set.contains(std::uint64_t{1} << 40) && !set.contains(6));
  EXPECT(set.cardinality() == std::optional<std::size_t>(2));
  PredicateFilter odd([](Label l) { return l % 2 == 1; });
  EXPECT(odd.contains(3) && !odd.contains(4));
  EXPECT(!odd.cardinality().has_value());
  EXPECT(!odd.for_each([](Label) {}));
}

void no_gpu_fails_loudly() {
  // Without a device the GPU build cannot hold an index: construction throws quiver::Error with
  // the CUDA runtime's reason instead of falling back to a host implementation.
  EXPECT(gpu::device_count() == 0);
  EXPECT_ERROR(FlatIndex(8, Metric::kL2));
  IvfPqParams p;
  p.dim = 8;
  p.nlist = 4;
  p.m = 2;
  EXPECT_ERROR(IvfPqIndex{p});
  EXPECT_ERROR(FlatIndex(0));  // argument checks come first
}

// ---- FlatIndex (tests/test_flat.cc, tests/test_regressions.cc) ----------------------------------

void flat_matches_naive() {
  const std::size_t dim = 13, n = 300, k = 7;
  const auto base = normal_rows(n, dim, 1);
  const auto q = normal_rows(1, dim, 2);
  FlatIndex index(dim);
  index.add(base.data(), n);
  const auto got = index.search(q.data(), k);
  EXPECT(got.size() == k);
  std::vector<Neighbor> naive;
  for (std::size_t i = 0; i < n; ++i) {
    float d = 0;
    for (std::size_t j = 0; j < dim; ++j) {
      const float t = q[j] - base[i * dim + j];
      d += t * t;
    }
    naive.push_back({d, i});
  }
  std::sort(naive.begin(), naive.end());
  for (std::size_t j = 0; j < std::min(k, got.size()); ++j) {
    EXPECT(got[j].label == naive[j].label);
    EXPECT(std::fabs(got[j].distance - naive[j].distance) <= 1e-3f);
  }
}

void flat_cosine_and_ip() {
  const std::size_t dim = 4;
  const std::vector<float> base = {1, 0, 0, 0, 0, 2, 0, 0, 1, 1, 0, 0};
  const std::vector<float> q = {3, 0.1f, 0, 0};
  FlatIndex cosine(dim, Metric::kCosine);
  cosine.add(base.data(), 3);
  auto r = cosine.search(q.data(), 3);
  EXPECT(r.size() == 3 && r[0].label == 0);
  EXPECT(std::fabs(r[0].distance - (1.0f - 3.0f / std::sqrt(9.01f))) <= 1e-5f);
  // vector(i) is the stored (normalized) row
  const float* v1 = cosine.vector(1);
  EXPECT(v1 != nullptr && v1[0] == 0.0f && v1[1] == 1.0f);
  EXPECT(cosine.vector(3) == nullptr);
  EXPECT(cosine.label(2) == 2);

  FlatIndex ip(dim, Metric::kInnerProduct);
  ip.add(base.data(), 3);
  r = ip.search(q.data(), 3);
  EXPECT(r.size() == 3 && r[0].label == 2);  // 3.1 beats 3.0
  EXPECT(std::fabs(r[0].distance - (1.0f - 3.1f)) <= 1e-5f);
  EXPECT(ip.metric() == Metric::kInnerProduct && ip.dim() == 4);
}

void flat_fewer_than_k_and_filters() {
  const std::size_t dim = 8;
  const auto base = normal_rows(10, dim, 3);
  FlatIndex index(dim);
  std::vector<Label> labels;
  for (Label l = 100; l < 110; ++l) labels.push_back(l);
  index.add(base.data(), 10, labels.data());
  EXPECT(index.search(base.data(), 50).size() == 10);

  LabelSetFilter only({103, 107});
  BitsetFilter bits(200);
  bits.insert(103);
  bits.insert(107);
  PredicateFilter pred([](Label l) { return l == 103 || l == 107; });
  ThreadPool pool(3);
  const Filter* filters[] = {&only, &bits, &pred};
  std::vector<Neighbor> first;
  for (const Filter* f : filters) {
    const auto r = index.search(base.data(), 5, f);
    EXPECT(r.size() == 2);
    for (const auto& nb : r) EXPECT(nb.label == 103 || nb.label == 107);
    if (first.empty()) first = r;
    EXPECT(r == first);
    std::vector<Label> out(5);
    std::vector<float> dist(5);
    index.search_batch(base.data(), 1, 5, out.data(), dist.data(), f, &pool);
    EXPECT(out[2] == kInvalidLabel);
    EXPECT(dist[4] == std::numeric_limits<float>::infinity());
  }
  // nq == 0 or k == 0 touches nothing
  index.search_batch(base.data(), 0, 5, nullptr, nullptr);
  index.search_batch(base.data(), 1, 0, nullptr, nullptr);
  EXPECT(index.search(base.data(), 0).empty());
}

void flat_save_load(const std::string& tmp) {
  const std::size_t dim = 16;
  const auto base = normal_rows(100, dim, 4);
  FlatIndex index(dim, Metric::kCosine);
  index.add(base.data(), 100);
  const std::string path = tmp + "/api_flat.qvr";
  index.save(path);
  const FlatIndex loaded = FlatIndex::load(path);
  EXPECT(loaded.size() == 100);
  EXPECT(loaded.metric() == Metric::kCosine);
  EXPECT(loaded.search(base.data(), 5) == index.search(base.data(), 5));
  EXPECT(loaded.label(99) == 99);
  EXPECT_ERROR(FlatIndex::load(tmp + "/does_not_exist.qvr"));
  FlatIndex moved = FlatIndex::load(path);
  FlatIndex target(3);
  target = std::move(moved);
  EXPECT(target.dim() == dim && target.size() == 100);
}

void flat_rejects_bad_input() {
  FlatIndex flat(4);
  std::vector<float> bad = {1, std::nanf(""), 2, 3};
  EXPECT_ERROR(flat.add(bad.data(), 1));
  bad[1] = std::numeric_limits<float>::infinity();
  EXPECT_ERROR(flat.add(bad.data(), 1));
  const std::vector<float> v(4, 1.0f);
  EXPECT_ERROR(flat.add(v.data(), 1, &kInvalidLabel));
  EXPECT(flat.size() == 0);
  EXPECT_ERROR((void)flat.search(bad.data(), 1));
  EXPECT_ERROR((void)flat.search(nullptr, 1));
  EXPECT_ERROR(FlatIndex(kMaxDimension + 1));
}

void flat_concurrent_add_and_search() {
  const std::size_t dim = 8;
  const auto base = normal_rows(4000, dim, 8);
  FlatIndex flat(dim);
  flat.add(base.data(), 100);
  std::atomic<bool> done{false};
  std::atomic<int> bad{0};
  std::thread reader([&] {
    while (!done) {
      if (flat.search(base.data(), 3).size() != 3) ++bad;
    }
  });
  for (std::size_t i = 100; i < 4000; i += 100) flat.add(base.data() + i * dim, 100);
  done = true;
  reader.join();
  EXPECT(bad.load() == 0);
  EXPECT(flat.size() == 4000);
}

// ---- IvfPqIndex (tests/test_quantizer.cc:140-175, tests/test_regressions.cc) -------------------

void ivf_untrained_and_train(const std::string&) {
  IvfPqParams p;
  p.dim = 16;
  p.nlist = 32;
  p.m = 8;
  p.store_vectors = true;
  IvfPqIndex index(p);
  EXPECT(!index.is_trained());
  const auto base = normal_rows(300, 16, 8);
  EXPECT_ERROR(index.add(base.data(), 1));  // untrained
  EXPECT_ERROR(index.train(base.data(), 200));  // fewer than max(nlist, 256) rows
  EXPECT(index.size() == 0 && index.dim() == 16 && index.params().nlist == 32);
  std::vector<Label> out(3);
  std::vector<float> dist(3);
  index.search_batch(base.data(), 1, 3, out.data(), dist.data());  // empty index: padding only
  EXPECT(out[0] == kInvalidLabel && std::isinf(dist[0]));
  IvfPqParams bad = p;
  bad.m = 5;  // does not divide dim
  EXPECT_ERROR(IvfPqIndex{bad});
  index.train(base.data(), 300);  // trains (assignments on the GPU)
  EXPECT(index.is_trained());
  EXPECT_ERROR(index.train(base.data(), 300));  // already trained
  index.add(base.data(), 300);
  index.search_batch(base.data(), 1, 3, out.data(), dist.data());
  EXPECT(out[0] == 0 && dist[0] >= 0.0f);  // the row itself is its own nearest neighbour
}

void ivf_filter_save_load(const std::string& qvr, const std::string& tmp) {
  IvfPqIndex index = IvfPqIndex::load(qvr);
  EXPECT(index.is_trained() && index.size() > 0);
  const std::size_t dim = index.dim(), nlist = index.params().nlist;
  const auto q = normal_rows(8, dim, 21);
  LabelSetFilter allowed({1, 2, 3, 1999});
  BitsetFilter bits(2000);
  for (Label l : {1, 2, 3, 1999}) bits.insert(l);
  PredicateFilter pred([](Label l) { return l == 1 || l == 2 || l == 3 || l == 1999; });
  IvfPqSearchParams sp;
  sp.nprobe = nlist;
  std::vector<Neighbor> first;
  for (const Filter* f : std::initializer_list<const Filter*>{&allowed, &bits, &pred}) {
    sp.filter = f;
    const auto r = index.search(q.data(), 10, sp);
    EXPECT(r.size() == 4);
    for (const auto& nb : r) EXPECT(allowed.contains(nb.label));
    if (first.empty()) first = r;
    EXPECT(r == first);
  }
  const std::string path = tmp + "/api_ivf.qvr";
  index.save(path);
  const IvfPqIndex loaded = IvfPqIndex::load(path);
  EXPECT(loaded.size() == index.size());
  EXPECT(loaded.list_sizes() == index.list_sizes());
  EXPECT(loaded.memory_bytes() == index.memory_bytes() && loaded.memory_bytes() > 0);
  sp.filter = nullptr;
  sp.nprobe = 4;
  sp.refine_factor = index.params().store_vectors ? 2 : 0;
  EXPECT(loaded.search(q.data() + dim, 5, sp) == index.search(q.data() + dim, 5, sp));
  std::size_t total = 0;
  for (auto s : index.list_sizes()) total += s;
  EXPECT(total == index.size());
}

void ivf_refine_overflow_saturates(const std::string& qvr) {
  IvfPqIndex index = IvfPqIndex::load(qvr);
  if (!index.params().store_vectors) return;
  const auto q = normal_rows(1, index.dim(), 5);
  IvfPqSearchParams sp;
  sp.nprobe = index.params().nlist;
  sp.refine_factor = std::size_t{1} << 63;  // k * refine_factor wraps to 0 for even k
  const auto r = index.search(q.data(), 2, sp);
  EXPECT(r.size() == 2);
  if (r.size() == 2) EXPECT(r[0].distance <= r[1].distance);
}

void ivf_add_search_add(const std::string& qvr) {
  IvfPqIndex index = IvfPqIndex::load(qvr);
  const std::size_t dim = index.dim(), n0 = index.size(), nq = 2000;
  const auto base = normal_rows(2000, dim, 9);
  const auto queries = normal_rows(nq, dim, 10);
  ThreadPool pool(4), inline_pool(1);
  std::vector<Label> labels(nq * 10);
  std::vector<float> dist(nq * 10);
  IvfPqSearchParams sp;
  sp.nprobe = index.params().nlist;
  std::atomic<int> done{0};
  std::thread b([&] {
    index.search_batch(queries.data(), nq, 10, labels.data(), dist.data(), sp, &pool);
    ++done;
  });
  std::thread a([&] {
    index.add(base.data(), 2000, nullptr, &pool);
    ++done;
  });
  std::thread c([&] {
    index.add(base.data(), 100, nullptr, &inline_pool);
    ++done;
  });
  for (int i = 0; i < 600 && done < 3; ++i) std::this_thread::sleep_for(std::chrono::milliseconds(100));
  if (done < 3) {
    std::fprintf(stderr, "deadlock: only %d/3 threads finished\n", done.load());
    std::_Exit(1);
  }
  a.join();
  b.join();
  c.join();
  EXPECT(index.size() == n0 + 2100);
}

// ---- dump modes --------------------------------------------------------------------------------

template <class T>
std::vector<T> read_raw(const std::string& path, std::size_t count) {
  std::vector<T> v(count);
  std::ifstream in(path, std::ios::binary);
  if (!in.read(reinterpret_cast<char*>(v.data()), std::streamsize(count * sizeof(T))))
    throw std::runtime_error("cannot read " + path);
  return v;
}

template <class T>
void write_raw(const std::string& path, const std::vector<T>& v) {
  std::ofstream out(path, std::ios::binary);
  out.write(reinterpret_cast<const char*>(v.data()), std::streamsize(v.size() * sizeof(T)));
  if (!out) throw std::runtime_error("cannot write " + path);
}

// spec filter kinds: 0 none, 1 LabelSetFilter, 2 BitsetFilter, 3 PredicateFilter over allowed.bin
struct FilterHolder {
  std::unique_ptr<LabelSetFilter> set;
  std::unique_ptr<BitsetFilter> bits;
  std::set<Label> members;
  std::unique_ptr<Filter> pred;
  const Filter* get(int kind) const {
    return kind == 1 ? static_cast<const Filter*>(set.get())
           : kind == 2 ? static_cast<const Filter*>(bits.get())
           : kind == 3 ? pred.get()
                       : nullptr;
  }
};

FilterHolder make_filter(const std::string& dir, int kind, std::size_t nallowed) {
  FilterHolder h;
  if (kind == 0) return h;
  const auto allowed = read_raw<Label>(dir + "/allowed.bin", nallowed);
  h.set = std::make_unique<LabelSetFilter>(allowed.begin(), allowed.end());
  Label universe = 1;
  for (Label l : allowed) universe = std::max(universe, l + 1);
  h.bits = std::make_unique<BitsetFilter>(universe);
  for (Label l : allowed) h.bits->insert(l);
  h.members.insert(allowed.begin(), allowed.end());
  const std::set<Label>* m = &h.members;
  auto fn = [m](Label l) { return m->count(l) != 0; };
  h.pred = std::make_unique<PredicateFilter<decltype(fn)>>(fn);
  return h;
}

int dump_flat(const std::string& dir) {
  std::ifstream spec(dir + "/spec.txt");
  std::string metric;
  std::size_t dim, n, nq, k, nallowed;
  int kind;
  if (!(spec >> metric >> dim >> n >> nq >> k >> kind >> nallowed)) return 2;
  const auto base = read_raw<float>(dir + "/base.bin", n * dim);
  const auto labels = read_raw<Label>(dir + "/labels.bin", n);
  const auto queries = read_raw<float>(dir + "/queries.bin", nq * dim);
  const FilterHolder f = make_filter(dir, kind, nallowed);
  FlatIndex index(dim, parse_metric(metric));
  index.add(base.data(), n / 2, labels.data());  // two adds exercise the append path
  index.add(base.data() + (n / 2) * dim, n - n / 2, labels.data() + n / 2);
  std::vector<Label> out(nq * k);
  std::vector<float> dist(nq * k);
  ThreadPool pool(4);
  index.search_batch(queries.data(), nq, k, out.data(), dist.data(), f.get(kind), &pool);
  write_raw(dir + "/out_labels.bin", out);
  write_raw(dir + "/out_dists.bin", dist);
  return 0;
}

int dump_ivf(const std::string& dir) {
  std::ifstream spec(dir + "/spec.txt");
  std::string qvr;
  std::size_t nq, k, nprobe, refine, nallowed;
  int kind;
  if (!(spec >> qvr >> nq >> k >> nprobe >> refine >> kind >> nallowed)) return 2;
  const IvfPqIndex index = IvfPqIndex::load(qvr);
  const auto queries = read_raw<float>(dir + "/queries.bin", nq * index.dim());
  const FilterHolder f = make_filter(dir, kind, nallowed);
  IvfPqSearchParams sp;
  sp.nprobe = nprobe;
  sp.refine_factor = refine;
  sp.filter = f.get(kind);
  std::vector<Label> out(nq * k);
  std::vector<float> dist(nq * k);
  index.search_batch(queries.data(), nq, k, out.data(), dist.data(), sp);
  write_raw(dir + "/out_labels.bin", out);
  write_raw(dir + "/out_dists.bin", dist);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "";
  try {
    if (mode == "flat" && argc > 2) return dump_flat(argv[2]);
    if (mode == "ivf" && argc > 2) return dump_ivf(argv[2]);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  std::vector<Case> cases = {
      {"ThreadPool.CoversEveryIndexExactlyOnce", pool_covers_every_index_once},
      {"ThreadPool.ActuallyRunsInParallel", pool_runs_in_parallel},
      {"ThreadPool.PropagatesFirstException", pool_propagates_first_exception},
      {"ThreadPool.NestedParallelForRunsInline", pool_nested_runs_inline},
      {"ThreadPool.ConcurrentCallersAreSerialized", pool_concurrent_callers_serialized},
      {"ThreadPool.SingleThreadPoolRunsInline", pool_single_thread_inline},
      {"ThreadPool.CrossPoolNestingDoesNotDeadlock", pool_cross_pool_nesting},
      {"Common.MetricsAndNeighbors", metrics_and_neighbors},
      {"Filter.Classes", filters},
  };
  if (mode == "cpu") {
    if (gpu::device_count() == 0) cases.push_back({"Gpu.NoDeviceFailsLoudly", no_gpu_fails_loudly});
    return run(cases);
  }
  if (mode == "gpu" && argc > 3) {
    const std::string qvr = argv[2], tmp = argv[3];
    cases.push_back({"FlatIndex.MatchesNaiveSearch", flat_matches_naive});
    cases.push_back({"FlatIndex.CosineAndInnerProduct", flat_cosine_and_ip});
    cases.push_back({"FlatIndex.FewerThanKAndFilters", flat_fewer_than_k_and_filters});
    cases.push_back({"FlatIndex.SaveLoadRoundTrip", [&] { flat_save_load(tmp); }});
    cases.push_back({"FlatIndex.RejectsBadInput", flat_rejects_bad_input});
    cases.push_back({"FlatIndex.ConcurrentAddAndSearch", flat_concurrent_add_and_search});
    cases.push_back({"IvfPq.UntrainedAndTrain", [&] { ivf_untrained_and_train(tmp); }});
    cases.push_back({"IvfPq.FilterSaveLoad", [&] { ivf_filter_save_load(qvr, tmp); }});
    cases.push_back({"IvfPq.RefineFactorOverflowIsSaturated",
                     [&] { ivf_refine_overflow_saturates(qvr); }});
    cases.push_back({"IvfPq.AddSearchAddDoesNotDeadlock", [&] { ivf_add_search_add(qvr); }});
    return run(cases);
  }
  std::fprintf(stderr, "usage: api_test cpu | gpu <ivf.qvr> <tmpdir> | flat <dir> | ivf <dir>\n");
  return 2;
}
