// The extern "C" boundary (include/qv_gpu.h): index handles, argument validation with the
// reference's error wording, host<->device staging, and the .qvr load/save of both index types.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <set>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <vector>

#include "qv_gpu.h"
#include "qv_state.h"
#include "qvr.h"

struct qv_flat {
  qv::FlatState s;
  mutable std::shared_mutex mu;  // searches shared, add exclusive
};

struct qv_ivfpq {
  qv::IvfState s;
  mutable std::shared_mutex mu;
};

struct qv_hnsw_store {
  qv::HnswStoreState s;
  mutable std::shared_mutex mu;  // searches shared; add, train and remove exclusive
};

namespace qv {

namespace {
thread_local std::string t_error;
thread_local SearchStats t_stats;
constexpr size_t kMaxDimension = 65536;    // include/quiver/common.h:20
constexpr size_t kMaxLists = size_t{1} << 24;  // src/ivfpq_index.cc:71
constexpr uint32_t kMeta = fourcc("META"), kVect = fourcc("VECT"), kLabl = fourcc("LABL"),
                   kCent = fourcc("CENT"), kPqcb = fourcc("PQCB"), kLoff = fourcc("LOFF"),
                   kCode = fourcc("CODE");

struct FlatMeta {  // src/flat_index.cc:24-29
  uint64_t dim, count;
  uint32_t metric, reserved;
};
struct IvfPqMeta {  // src/ivfpq_index.cc:32-43
  uint64_t dim, nlist, m, count, train_iterations, seed;
  uint32_t metric, store_vectors, trained, reserved;
};
}  // namespace

void set_error(const std::string& msg) { t_error = msg; }
const std::string& last_error() { return t_error; }
SearchStats& thread_stats() { return t_stats; }
bool& thread_timing() {
  thread_local bool on = false;
  return on;
}

namespace {
thread_local std::vector<PendingTimer> t_pending;
// The report words of this thread's last _device Flat search (read by qv_last_search_stats),
// or nullptr.
thread_local SearchFlags* t_flags = nullptr;

// Applies the report words of a host-buffer search that has completed to this thread's stats and
// turns them into the reference's errors.
void report_flags(const int* f) {
  t_stats.rescanned_queries += static_cast<uint64_t>(f[kFlagRescanned]);
  QV_REQUIRE(f[kFlagNonFinite] == 0, "vectors must not contain NaN or infinity");
  if (f[kFlagTimeout] != 0)
    fail(QV_ERR_DEVICE, "tensor-core screen timed out waiting on a pipeline barrier");
}
}  // namespace

void begin_search_stats() {
  if (!thread_timing()) t_stats = SearchStats{};
}

void defer_timer(const PendingTimer& t) { t_pending.push_back(t); }

void resolve_timers() {
  for (const PendingTimer& t : t_pending) {
    float ms = 0.0f;
    if (cudaEventSynchronize(t.e1) == cudaSuccess &&
        cudaEventElapsedTime(&ms, t.e0, t.e1) == cudaSuccess) {
      t_stats.dominant_ms += ms;
      t_stats.dominant_work += t.work + (t.count ? static_cast<double>(*t.count) * t.per_count : 0.0);
      t_stats.work_is_bytes = t.bytes;
      t_stats.dominant_name = t.name;
    }
    cudaEventDestroy(t.e0);
    cudaEventDestroy(t.e1);
  }
  t_pending.clear();
}

unsigned long long* timing_count_slot() {
  constexpr size_t kSlots = 4096;
  thread_local unsigned long long* slots = nullptr;
  thread_local size_t next = 0;
  if (slots == nullptr) {
    void* p = nullptr;
    QV_CUDA(cudaHostAlloc(&p, kSlots * sizeof(unsigned long long), cudaHostAllocPortable));
    slots = static_cast<unsigned long long*>(p);
  }
  unsigned long long* s = slots + next;
  next = (next + 1) % kSlots;
  return s;
}

// Per-thread device words that a _device search's kernels report into (rescanned queries,
// non-finite queries, screen timeouts), and a pinned host copy of them queued at the end of each
// search, read by qv_last_search_stats once the search's stream has completed.
SearchFlags& thread_search_flags(int device) {
  thread_local std::map<int, SearchFlags> flags;
  auto it = flags.find(device);
  if (it != flags.end()) return it->second;
  SearchFlags f;
  QV_CUDA(cudaMalloc(&f.dev, 2 * kSearchFlagWords * sizeof(int)));
  QV_CUDA(cudaMemset(f.dev, 0, 2 * kSearchFlagWords * sizeof(int)));
  void* h = nullptr;
  QV_CUDA(cudaHostAlloc(&h, 2 * kSearchFlagWords * sizeof(int), cudaHostAllocPortable));
  f.host = static_cast<int*>(h);
  std::memset(f.host, 0, 2 * kSearchFlagWords * sizeof(int));
  f.sync_dev = f.dev + kSearchFlagWords;
  f.sync_host = f.host + kSearchFlagWords;
  QV_CUDA(cudaEventCreateWithFlags(&f.done, cudaEventDisableTiming));
  return flags.emplace(device, f).first->second;
}

// Keeps freed stream-ordered allocations in the device's default memory pool instead of
// returning them to the driver at every synchronization, so that the temporaries of one search
// are reused by the next without remapping memory (a per-process setting of this context).
void keep_pool_memory(int device) {
  static std::mutex mu;
  static std::set<int> done;
  std::lock_guard<std::mutex> lock(mu);
  if (!done.insert(device).second) return;
  cudaMemPool_t pool = nullptr;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
}

cudaStream_t thread_stream(int device) {
  thread_local std::map<int, cudaStream_t> streams;
  auto it = streams.find(device);
  if (it != streams.end()) return it->second;
  keep_pool_memory(device);
  cudaStream_t s = nullptr;
  QV_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  streams[device] = s;
  return s;
}

// The stream a _device entry point runs on. A caller's stream is used as it is. NULL means CUDA's
// default (legacy) stream, as everywhere in the runtime API (it is also PyTorch's default stream);
// the work then runs on this thread's own stream, ordered after everything already queued on the
// default stream and before anything queued there after the call (two event waits), which keeps
// the caller's ordering without running the search itself on the default stream.
class CallerStream {
 public:
  CallerStream(void* stream, int device) {
    keep_pool_memory(device);
    st_ = static_cast<cudaStream_t>(stream);
    if (st_ != nullptr) return;
    st_ = thread_stream(device);
    ev_ = thread_event(device);
    QV_CUDA(cudaEventRecord(ev_, cudaStreamLegacy));
    QV_CUDA(cudaStreamWaitEvent(st_, ev_, 0));
  }
  ~CallerStream() {
    if (ev_ == nullptr) return;
    // Also on failure: the default stream then waits for whatever was queued before it.
    if (cudaEventRecord(ev_, st_) == cudaSuccess) cudaStreamWaitEvent(cudaStreamLegacy, ev_, 0);
  }
  CallerStream(const CallerStream&) = delete;
  CallerStream& operator=(const CallerStream&) = delete;
  cudaStream_t get() const { return st_; }

 private:
  static cudaEvent_t thread_event(int device) {
    thread_local std::map<int, cudaEvent_t> events;
    auto it = events.find(device);
    if (it != events.end()) return it->second;
    cudaEvent_t e = nullptr;
    QV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    events[device] = e;
    return e;
  }
  cudaStream_t st_ = nullptr;
  cudaEvent_t ev_ = nullptr;
};

int sm_count(int device) {
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  QV_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  cache[device] = n;
  return n;
}

void check_finite(const float* v, size_t count) {
  // A float is NaN or infinite exactly when its exponent bits are all ones; the branch-free
  // integer test vectorizes (the whole query batch is checked on every search).
  uint32_t bad = 0;
  for (size_t i = 0; i < count; ++i) {
    uint32_t b;
    std::memcpy(&b, v + i, sizeof(b));
    bad |= static_cast<uint32_t>((b & 0x7f800000u) == 0x7f800000u);
  }
  QV_REQUIRE(bad == 0, "vectors must not contain NaN or infinity");
}

namespace {

void check_metric(uint32_t metric) {
  QV_REQUIRE(metric == QV_METRIC_L2 || metric == QV_METRIC_IP || metric == QV_METRIC_COSINE,
             "unknown metric");
}

void check_labels(const uint64_t* labels, size_t n) {
  if (labels == nullptr) return;
  QV_REQUIRE(std::find(labels, labels + n, kInvalidLabel) == labels + n,
             "label 2^64-1 is reserved (it marks empty result slots)");
}

template <class T>
void h2d(DeviceBuffer& dst, const T* src, size_t n, cudaStream_t st) {
  dst.allocate(std::max<size_t>(1, n) * sizeof(T), st);
  if (n > 0) QV_CUDA(cudaMemcpyAsync(dst.get(), src, n * sizeof(T), cudaMemcpyHostToDevice, st));
}

// Device position bitmap for a host filter (nullptr when there is no filter).
DeviceBuffer device_filter(const uint64_t* d_labels, size_t count, const qv_filter* f,
                           cudaStream_t st) {
  DeviceBuffer bm;
  if (f == nullptr) return bm;
  bm.allocate(std::max<size_t>(1, (count + 63) / 64) * sizeof(uint64_t), st);
  build_position_bitmap(d_labels, count, *f, bm.get<uint64_t>(), st);
  return bm;
}

void fill_unfilled(uint64_t* labels, float* dists, size_t n) {
  std::fill(labels, labels + n, kInvalidLabel);
  std::fill(dists, dists + n, std::numeric_limits<float>::infinity());
}

size_t result_size(size_t nq, size_t k) {
  size_t total = 0;
  QV_REQUIRE(!__builtin_mul_overflow(nq, k, &total) && total <= (size_t{1} << 40),
             "nq * k is too large");
  return total;
}

// ---- IVF list bookkeeping ----------------------------------------------------------------------

// Gathers rows of `src_old` (old storage order) and `src_new` (new rows) into `dst` following
// `from`: value < n_old picks an old row, otherwise row (value - n_old) of the new batch.
__global__ void gather_rows_kernel(const float* src_old, size_t n_old, const float* src_new,
                                   const uint64_t* from, size_t n_total, int dim, float* dst) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= n_total * dim) return;
  const size_t r = i / dim;
  const int c = static_cast<int>(i - r * dim);
  const uint64_t f = from[r];
  dst[i] = f < n_old ? src_old[f * dim + c] : src_new[(f - n_old) * dim + c];
}

void ivf_append(IvfState& s, const std::vector<uint32_t>& assign, const std::vector<uint8_t>& codes,
                const std::vector<uint64_t>& labels, const float* d_new_vectors, cudaStream_t st) {
  const size_t n = assign.size(), m = s.m, nlist = s.nlist;
  std::vector<uint64_t> extra(nlist, 0);
  for (uint32_t l : assign) ++extra[l];
  for (size_t l = 0; l < nlist; ++l) {
    const uint64_t len = s.host_offsets[l + 1] - s.host_offsets[l];
    QV_REQUIRE(len + extra[l] <= std::numeric_limits<uint32_t>::max(),
               "too many vectors in one IVF cell (2^32 limit); use a larger nlist");
  }
  std::vector<uint64_t> off(nlist + 1, 0);
  for (size_t l = 0; l < nlist; ++l)
    off[l + 1] = off[l] + (s.host_offsets[l + 1] - s.host_offsets[l]) + extra[l];
  const size_t total = s.count + n;
  std::vector<uint8_t> new_codes(total * m);
  std::vector<uint64_t> new_labels(total);
  std::vector<uint64_t> from(total);
  std::vector<uint64_t> cursor(nlist);
  for (size_t l = 0; l < nlist; ++l) {  // old entries first, in their order
    const uint64_t b = s.host_offsets[l], e = s.host_offsets[l + 1];
    std::memcpy(new_codes.data() + off[l] * m, s.host_codes.data() + b * m, (e - b) * m);
    for (uint64_t i = b; i < e; ++i) {
      new_labels[off[l] + (i - b)] = s.host_labels[i];
      from[off[l] + (i - b)] = i;
    }
    cursor[l] = off[l] + (e - b);
  }
  for (size_t i = 0; i < n; ++i) {  // then the new ones in input order (src/ivfpq_index.cc:263-269)
    const uint64_t pos = cursor[assign[i]]++;
    std::memcpy(new_codes.data() + pos * m, codes.data() + i * m, m);
    new_labels[pos] = labels[i];
    from[pos] = s.count + i;
  }
  if (s.store_vectors) {
    DeviceBuffer dfrom, nv(std::max<size_t>(1, total * s.dim) * sizeof(float));
    h2d(dfrom, from.data(), total, st);
    gather_rows_kernel<<<ceil_div(total * s.dim, 256), 256, 0, st>>>(
        s.vectors.get<float>(), s.count, d_new_vectors, dfrom.get<uint64_t>(), total,
        static_cast<int>(s.dim), nv.get<float>());
    check_launch("gather_rows_kernel");
    QV_CUDA(cudaStreamSynchronize(st));
    s.vectors = std::move(nv);
  }
  s.host_offsets = std::move(off);
  s.host_codes = std::move(new_codes);
  s.host_labels = std::move(new_labels);
  s.count = total;
  ivf_upload_lists(s, st);
}

void ivf_validate_params(const qv_ivfpq_params& p) {
  QV_REQUIRE(p.dim >= 1 && p.dim <= kMaxDimension,
             "dimension must be in [1, " + std::to_string(kMaxDimension) + "]");
  QV_REQUIRE(p.m > 0 && p.dim % p.m == 0, "PQ: dimension " + std::to_string(p.dim) +
                                              " must be divisible by m=" + std::to_string(p.m));
  QV_REQUIRE(p.nlist >= 1 && p.nlist <= kMaxLists, "nlist must be in [1, 2^24]");
  check_metric(p.metric);
}

std::unique_ptr<qv_ivfpq> ivf_new(int device, const qv_ivfpq_params& p) {
  ivf_validate_params(p);
  auto h = std::make_unique<qv_ivfpq>();
  IvfState& s = h->s;
  s.device = device;
  s.dim = p.dim;
  s.nlist = p.nlist;
  s.m = p.m;
  s.dsub = p.dim / p.m;
  s.metric = p.metric;
  s.train_iterations = p.train_iterations;
  s.store_vectors = p.store_vectors != 0;
  s.seed = p.seed;
  s.host_offsets.assign(p.nlist + 1, 0);
  s.host_global_base.assign(p.nlist, 0);
  DeviceScope scope(device);
  ivf_upload_lists(s, thread_stream(device));
  return h;
}

void ivf_load_into(qv_ivfpq** out, int device, const char* path, bool verify, bool shard,
                   uint64_t label_begin, uint64_t label_end) {
  QV_REQUIRE(path != nullptr && out != nullptr, "null argument");
  QvrFile f(path, QvrKind::kIvfPq, verify);
  const std::string corrupt = std::string("corrupt index file '") + path + "': ";
  IvfPqMeta meta;
  std::memcpy(&meta, f.array(kMeta, 1, sizeof(IvfPqMeta)), sizeof(meta));
  auto chk = [&](bool c, const char* what) {
    if (!c) fail(QV_ERR_IO, corrupt + what);
  };
  chk(meta.dim >= 1 && meta.dim <= 65536, "bad dimension");
  chk(meta.m >= 1 && meta.m <= meta.dim && meta.dim % meta.m == 0, "bad m");
  chk(meta.nlist >= 1 && meta.nlist <= kMaxLists, "bad nlist");
  chk((meta.nlist + 1) * sizeof(uint64_t) <= f.size(), "bad nlist");
  chk(meta.metric <= QV_METRIC_COSINE, "bad metric");
  chk(meta.count <= f.size(), "bad count");
  qv_ivfpq_params p{meta.dim, meta.metric, meta.nlist, meta.m, meta.train_iterations,
                    meta.store_vectors != 0, meta.seed};
  auto h = ivf_new(device, p);
  IvfState& s = h->s;
  DeviceScope scope(device);
  cudaStream_t st = thread_stream(device);
  const size_t count = meta.count, d = s.dim;
  if (meta.trained != 0) {
    const float* cent = reinterpret_cast<const float*>(f.array(kCent, s.nlist * d, 4));
    const float* cb =
        reinterpret_cast<const float*>(f.array(kPqcb, s.m * kSubCentroids * s.dsub, 4));
    bool finite = true;
    for (size_t i = 0; i < s.nlist * d; ++i) finite &= std::isfinite(cent[i]);
    for (size_t i = 0; i < s.m * kSubCentroids * s.dsub; ++i) finite &= std::isfinite(cb[i]);
    chk(finite, "non-finite centroids");
    ivf_set_trained(s, cent, cb, st);
  } else {
    chk(count == 0, "untrained index with vectors");
  }
  const uint64_t* offsets = reinterpret_cast<const uint64_t*>(f.array(kLoff, s.nlist + 1, 8));
  chk(offsets[0] == 0 && offsets[s.nlist] == count, "bad list offsets");
  for (size_t l = 0; l < s.nlist; ++l) chk(offsets[l] <= offsets[l + 1], "bad list offsets");
  const uint8_t* codes = f.array(kCode, count * s.m, 1);
  const uint64_t* labels = reinterpret_cast<const uint64_t*>(f.array(kLabl, count, 8));
  const float* vectors = nullptr;
  if (s.store_vectors) {
    vectors = reinterpret_cast<const float*>(f.array(kVect, count * d, 4));
    bool finite = true;
    for (size_t i = 0; i < count * d; ++i) finite &= std::isfinite(vectors[i]);
    chk(finite, "non-finite stored vectors");
  }
  // Keep every entry, or (shard) the entries whose label is in [label_begin, label_end).
  std::vector<uint64_t> keep_pos;
  keep_pos.reserve(shard ? count / 2 : count);
  std::vector<uint64_t> off(s.nlist + 1, 0);
  std::vector<uint32_t> gbase(s.nlist, 0);
  for (size_t l = 0; l < s.nlist; ++l) {
    bool first = true;
    for (uint64_t i = offsets[l]; i < offsets[l + 1]; ++i) {
      if (shard && (labels[i] < label_begin || labels[i] >= label_end)) continue;
      if (first) {
        gbase[l] = static_cast<uint32_t>(i - offsets[l]);
        first = false;
      }
      keep_pos.push_back(i);
    }
    off[l + 1] = keep_pos.size();
  }
  s.count = keep_pos.size();
  s.host_offsets = std::move(off);
  s.host_global_base = std::move(gbase);
  s.host_codes.resize(s.count * s.m);
  s.host_labels.resize(s.count);
  for (size_t i = 0; i < s.count; ++i) {
    std::memcpy(s.host_codes.data() + i * s.m, codes + keep_pos[i] * s.m, s.m);
    s.host_labels[i] = labels[keep_pos[i]];
  }
  if (shard) {  // entries of a list kept by one shard must be contiguous in the full list
    for (size_t l = 0; l < s.nlist; ++l) {
      const uint64_t b = s.host_offsets[l], e = s.host_offsets[l + 1];
      if (e > b)
        chk(keep_pos[e - 1] - keep_pos[b] == e - b - 1,
            "label range of a shard is not contiguous within an inverted list");
    }
  }
  ivf_upload_lists(s, st);
  if (s.store_vectors) {
    s.vectors.allocate(std::max<size_t>(1, s.count * d) * sizeof(float));
    std::vector<float> v(s.count * d);
    for (size_t i = 0; i < s.count; ++i)
      std::memcpy(v.data() + i * d, vectors + keep_pos[i] * d, d * sizeof(float));
    if (!v.empty())
      QV_CUDA(cudaMemcpyAsync(s.vectors.get(), v.data(), v.size() * sizeof(float),
                              cudaMemcpyHostToDevice, st));
    QV_CUDA(cudaStreamSynchronize(st));
  }
  *out = h.release();
}

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" {

const char* qv_last_error(void) { return qv::last_error().c_str(); }
const char* qv_version(void) { return "quiver-b200 0.1.0 (sm_100a)"; }

qv_status qv_device_count(int* count) {
  return guarded([&] {
    QV_REQUIRE(count != nullptr, "null argument");
    QV_CUDA(cudaGetDeviceCount(count));
  });
}

qv_status qv_last_search_stats(qv_search_stats* stats) {
  return guarded([&] {
    QV_REQUIRE(stats != nullptr, "null argument");
    std::memset(stats, 0, sizeof(*stats));
    if (thread_timing()) resolve_timers();
    // The rescan count of this thread's _device Flat searches (the last one, or with timing on
    // every one since the previous read), once their report words have come back.
    if (t_flags != nullptr) {
      QV_CUDA(cudaEventSynchronize(t_flags->done));
      t_stats.rescanned_queries += static_cast<uint64_t>(t_flags->host[kFlagRescanned]);
      if (thread_timing()) {  // the words accumulate while timing is on: start again
        QV_CUDA(cudaMemset(t_flags->dev, 0, kSearchFlagWords * sizeof(int)));
        std::memset(t_flags->host, 0, kSearchFlagWords * sizeof(int));
      }
      t_flags = nullptr;
    }
    stats->kernel_launches = t_stats.kernel_launches;
    stats->rescanned_queries = t_stats.rescanned_queries;
    stats->dominant_kernel_ms = t_stats.dominant_ms;
    stats->dominant_kernel_work = t_stats.dominant_work;
    stats->dominant_work_is_bytes = t_stats.work_is_bytes ? 1u : 0u;
    std::strncpy(stats->dominant_kernel, t_stats.dominant_name.c_str(),
                 sizeof(stats->dominant_kernel) - 1);
    if (thread_timing()) t_stats = SearchStats{};  // accumulated since the previous read
  });
}

qv_status qv_set_timing(int enable) {
  return guarded([&] {
    if (thread_timing() && enable == 0) resolve_timers();  // release pending events
    if (enable != 0 && !thread_timing()) {
      t_stats = SearchStats{};
      timing_count_slot();  // allocate the pinned slots now, not inside a timed search
    }
    thread_timing() = enable != 0;
  });
}

qv_status qv_device_free(int device, void* ptr) {
  return guarded([&] {
    DeviceScope scope(device);
    if (ptr != nullptr) QV_CUDA(cudaFree(ptr));
  });
}

// ---- Flat --------------------------------------------------------------------------------------

qv_status qv_flat_create(int device, size_t dim, uint32_t metric, qv_flat** out) {
  return guarded([&] {
    QV_REQUIRE(out != nullptr, "null argument");
    QV_REQUIRE(dim >= 1 && dim <= kMaxDimension,
               "dimension must be in [1, " + std::to_string(kMaxDimension) + "]");
    check_metric(metric);
    int ndev = 0;
    QV_CUDA(cudaGetDeviceCount(&ndev));
    QV_REQUIRE(device >= 0 && device < ndev, "no CUDA device " + std::to_string(device));
    auto h = std::make_unique<qv_flat>();
    h->s.device = device;
    h->s.dim = dim;
    h->s.metric = metric;
    *out = h.release();
  });
}

qv_status qv_flat_destroy(qv_flat* index) {
  return guarded([&] {
    if (index == nullptr) return;
    DeviceScope scope(index->s.device);
    delete index;
  });
}

qv_status qv_flat_add(qv_flat* index, const float* vectors, size_t n, const uint64_t* labels) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    if (n == 0) return;  // src/flat_index.cc:50
    QV_REQUIRE(vectors != nullptr, "vectors must not be null");
    FlatState& s = index->s;
    check_finite(vectors, n * s.dim);
    check_labels(labels, n);
    std::unique_lock lock(index->mu);
    QV_REQUIRE(s.n + n <= std::numeric_limits<uint32_t>::max(),
               "FlatIndex holds at most 2^32 vectors");
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    std::vector<uint64_t> lab(n);
    for (size_t i = 0; i < n; ++i) lab[i] = labels ? labels[i] : s.n + i;
    flat_reserve(s, s.n + n, st);
    QV_CUDA(cudaMemcpyAsync(s.x.get<float>() + s.n * s.dim, vectors, n * s.dim * sizeof(float),
                            cudaMemcpyHostToDevice, st));
    DeviceBuffer dl;
    h2d(dl, lab.data(), n, st);
    flat_append(s, s.x.get<float>() + s.n * s.dim, dl.get<uint64_t>(), n, st);
    s.host_labels.insert(s.host_labels.end(), lab.begin(), lab.end());
    // The rows are complete on the device when add() returns, as in the reference, so that a
    // search on any stream (the _device entry points take the caller's) sees them.
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_flat_reserve(qv_flat* index, size_t n) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    FlatState& s = index->s;
    QV_REQUIRE(n <= std::numeric_limits<uint32_t>::max(), "FlatIndex holds at most 2^32 vectors");
    std::unique_lock lock(index->mu);
    DeviceScope scope(s.device);
    flat_reserve(s, n, thread_stream(s.device));
  });
}

qv_status qv_flat_add_device(qv_flat* index, const float* vectors, size_t n,
                             const uint64_t* labels, void* stream) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    if (n == 0) return;  // src/flat_index.cc:50
    QV_REQUIRE(vectors != nullptr, "vectors must not be null");
    FlatState& s = index->s;
    std::unique_lock lock(index->mu);
    QV_REQUIRE(s.n + n <= std::numeric_limits<uint32_t>::max(),
               "FlatIndex holds at most 2^32 vectors");
    DeviceScope scope(s.device);
    CallerStream call_stream(stream, s.device);
    cudaStream_t st = call_stream.get();
    // The reference's checks (src/flat_index.cc:51-57), on the device, before the index changes.
    DeviceBuffer flags(2 * sizeof(int), st);
    QV_CUDA(cudaMemsetAsync(flags.get(), 0, 2 * sizeof(int), st));
    flat_check_rows(vectors, n * s.dim, labels, n, flags.get<int>(), st);
    int h[2] = {0, 0};
    QV_CUDA(cudaMemcpyAsync(h, flags.get(), sizeof(h), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
    QV_REQUIRE(h[0] == 0, "vectors must not contain NaN or infinity");
    QV_REQUIRE(h[1] == 0, "label 2^64-1 is reserved (it marks empty result slots)");
    flat_reserve(s, s.n + n, st);
    float* dst = s.x.get<float>() + s.n * s.dim;
    QV_CUDA(cudaMemcpyAsync(dst, vectors, n * s.dim * sizeof(float), cudaMemcpyDeviceToDevice, st));
    DeviceBuffer dl(n * sizeof(uint64_t), st);
    if (labels != nullptr) {
      QV_CUDA(cudaMemcpyAsync(dl.get(), labels, n * sizeof(uint64_t), cudaMemcpyDeviceToDevice, st));
    } else {
      sequential_labels(dl.get<uint64_t>(), n, s.n, st);
    }
    const size_t first = s.host_labels.size();
    s.host_labels.resize(first + n);
    QV_CUDA(cudaMemcpyAsync(s.host_labels.data() + first, dl.get(), n * sizeof(uint64_t),
                            cudaMemcpyDeviceToHost, st));
    flat_append(s, dst, dl.get<uint64_t>(), n, st);  // normalizes cosine rows; waits for the GPU
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_flat_search(const qv_flat* index, const float* queries, size_t nq, size_t k,
                         const qv_filter* filter, uint64_t* labels, float* distances) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(index != nullptr, "null index");
    if (nq == 0 || k == 0) return;  // src/flat_index.cc:128
    QV_REQUIRE(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
    const FlatState& s = index->s;
    const size_t total = result_size(nq, k);
    std::shared_lock lock(index->mu);
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    // The device search marks queries holding NaN or infinity (the reference rejects them,
    // src/flat_index.cc:131); the report words come back with the results, in one round trip.
    SearchFlags& flags = thread_search_flags(s.device);
    DeviceBuffer dq, dl(total * sizeof(uint64_t), st), dd(total * sizeof(float), st);
    QV_CUDA(cudaMemsetAsync(flags.sync_dev, 0, kSearchFlagWords * sizeof(int), st));
    h2d(dq, queries, nq * s.dim, st);
    DeviceBuffer bm = device_filter(s.labels.get<uint64_t>(), s.n, filter, st);
    flat_search(s, dq.get<float>(), nq, k, bm.get<uint64_t>(), dl.get<uint64_t>(),
                dd.get<float>(), nullptr, flags.sync_dev, st);
    QV_CUDA(cudaMemcpyAsync(flags.sync_host, flags.sync_dev, kSearchFlagWords * sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaMemcpyAsync(labels, dl.get(), total * sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaMemcpyAsync(distances, dd.get(), total * sizeof(float), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
    report_flags(flags.sync_host);
  });
}

qv_status qv_flat_search_device(const qv_flat* index, const float* queries, size_t nq, size_t k,
                                const uint64_t* position_bitmap, uint64_t* labels,
                                float* distances, uint64_t* keys, void* stream) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(index != nullptr, "null index");
    if (nq == 0 || k == 0) return;
    QV_REQUIRE(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
    result_size(nq, k);
    const FlatState& s = index->s;
    std::shared_lock lock(index->mu);
    DeviceScope scope(s.device);
    CallerStream call_stream(stream, s.device);
    cudaStream_t st = call_stream.get();
    // Nothing here waits for the GPU: device-detected conditions (queries holding NaN or
    // infinity, a screen that gave up on a barrier, rescans) land in this thread's report words,
    // whose host copy qv_last_search_stats reads once the stream has completed.
    SearchFlags& flags = thread_search_flags(s.device);
    if (!thread_timing())
      QV_CUDA(cudaMemsetAsync(flags.dev, 0, kSearchFlagWords * sizeof(int), st));
    flat_search(s, queries, nq, k, position_bitmap, labels, distances, keys, flags.dev, st);
    QV_CUDA(cudaMemcpyAsync(flags.host, flags.dev, kSearchFlagWords * sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaEventRecord(flags.done, st));
    t_flags = &flags;
  });
}

qv_status qv_flat_search_device_noalloc(const qv_flat* index, const float* queries, size_t nq,
                                        size_t k, const uint64_t* position_bitmap,
                                        uint64_t* labels, float* distances, uint64_t* keys,
                                        void* stream) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(index != nullptr, "null index");
    if (nq == 0 || k == 0) return;
    QV_REQUIRE(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
    result_size(nq, k);
    const FlatState& s = index->s;
    std::shared_lock lock(index->mu);
    DeviceScope scope(s.device);
    CallerStream call_stream(stream, s.device);
    cudaStream_t st = call_stream.get();
    flat_search_noalloc(s, queries, nq, k, position_bitmap, labels, distances, keys, st);
  });
}

size_t qv_flat_noalloc_max_bytes(void) { return flat_noalloc_max_bytes(); }

qv_status qv_flat_set_row_offset(qv_flat* index, uint64_t row_offset) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    std::unique_lock lock(index->mu);
    index->s.row_offset = row_offset;
  });
}

qv_status qv_flat_info(const qv_flat* index, size_t* size, size_t* dim, uint32_t* metric) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    std::shared_lock lock(index->mu);
    if (size) *size = index->s.n;
    if (dim) *dim = index->s.dim;
    if (metric) *metric = index->s.metric;
  });
}

qv_status qv_flat_rows(const qv_flat* index, size_t first, size_t count, float* vectors,
                       uint64_t* labels) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    std::shared_lock lock(index->mu);
    const FlatState& s = index->s;
    QV_REQUIRE(first <= s.n && count <= s.n - first, "row range out of bounds");
    if (count == 0) return;
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    if (vectors)
      QV_CUDA(cudaMemcpyAsync(vectors, s.x.get<float>() + first * s.dim,
                              count * s.dim * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (labels) std::memcpy(labels, s.host_labels.data() + first, count * sizeof(uint64_t));
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_flat_filter_bitmap(const qv_flat* index, const qv_filter* filter,
                                uint64_t** device_bitmap) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && filter != nullptr && device_bitmap != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    const FlatState& s = index->s;
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    const size_t words = std::max<size_t>(1, (s.n + 63) / 64);
    void* p = nullptr;
    QV_CUDA(cudaMalloc(&p, words * sizeof(uint64_t)));
    build_position_bitmap(s.labels.get<uint64_t>(), s.n, *filter, static_cast<uint64_t*>(p), st);
    QV_CUDA(cudaStreamSynchronize(st));
    *device_bitmap = static_cast<uint64_t*>(p);
  });
}

qv_status qv_flat_save(const qv_flat* index, const char* path) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && path != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    const FlatState& s = index->s;
    std::vector<float> v(s.n * s.dim);
    if (!v.empty()) {
      DeviceScope scope(s.device);
      cudaStream_t st = thread_stream(s.device);
      QV_CUDA(cudaMemcpyAsync(v.data(), s.x.get(), v.size() * sizeof(float), cudaMemcpyDeviceToHost, st));
      QV_CUDA(cudaStreamSynchronize(st));
    }
    FlatMeta meta{s.dim, s.n, s.metric, 0};
    QvrWriter w(QvrKind::kFlat);
    w.add(kMeta, &meta, sizeof(meta));
    w.add(kVect, v.data(), v.size() * sizeof(float));
    w.add(kLabl, s.host_labels.data(), s.host_labels.size() * sizeof(uint64_t));
    w.commit(path);
  });
}

qv_status qv_flat_load(int device, const char* path, int verify_checksums, qv_flat** out) {
  return guarded([&] {
    QV_REQUIRE(path != nullptr && out != nullptr, "null argument");
    QvrFile f(path, QvrKind::kFlat, verify_checksums != 0);
    FlatMeta meta;
    std::memcpy(&meta, f.array(kMeta, 1, sizeof(FlatMeta)), sizeof(meta));
    const std::string corrupt = "corrupt index file: ";
    if (!(meta.dim > 0 && meta.dim <= kMaxDimension)) fail(QV_ERR_IO, corrupt + "bad dimension");
    if (meta.metric > QV_METRIC_COSINE) fail(QV_ERR_IO, corrupt + "unknown metric");
    if (meta.count > f.size() / sizeof(uint64_t)) fail(QV_ERR_IO, corrupt + "bad vector count");
    if (meta.count > f.size() / (meta.dim * sizeof(float) + 1))
      fail(QV_ERR_IO, corrupt + "bad vector count");
    const float* v = reinterpret_cast<const float*>(f.array(kVect, meta.count * meta.dim, 4));
    const uint64_t* l = reinterpret_cast<const uint64_t*>(f.array(kLabl, meta.count, 8));
    for (size_t i = 0; i < meta.count * meta.dim; ++i)
      if (!std::isfinite(v[i])) fail(QV_ERR_IO, corrupt + "non-finite vector values");
    qv_flat* h = nullptr;
    qv_status st = qv_flat_create(device, meta.dim, meta.metric, &h);
    if (st != QV_OK) fail(st, last_error());
    std::unique_ptr<qv_flat> owner(h);
    // Stored rows are already normalized: append them without re-normalizing.
    FlatState& s = h->s;
    if (meta.count > 0) {
      DeviceScope scope(device);
      cudaStream_t cs = thread_stream(device);
      flat_reserve(s, meta.count, cs);
      QV_CUDA(cudaMemcpyAsync(s.x.get(), v, meta.count * meta.dim * sizeof(float),
                              cudaMemcpyHostToDevice, cs));
      DeviceBuffer dl;
      h2d(dl, l, meta.count, cs);
      const uint32_t metric = s.metric;
      s.metric = QV_METRIC_L2;  // skip the normalization pass of flat_append
      flat_append(s, s.x.get<float>(), dl.get<uint64_t>(), meta.count, cs);
      s.metric = metric;
      s.host_labels.assign(l, l + meta.count);
      QV_CUDA(cudaStreamSynchronize(cs));
    }
    *out = owner.release();
  });
}

// ---- IVF-PQ ------------------------------------------------------------------------------------

qv_status qv_ivfpq_create(int device, const qv_ivfpq_params* params, qv_ivfpq** out) {
  return guarded([&] {
    QV_REQUIRE(params != nullptr && out != nullptr, "null argument");
    int ndev = 0;
    QV_CUDA(cudaGetDeviceCount(&ndev));
    QV_REQUIRE(device >= 0 && device < ndev, "no CUDA device " + std::to_string(device));
    *out = ivf_new(device, *params).release();
  });
}

qv_status qv_ivfpq_destroy(qv_ivfpq* index) {
  return guarded([&] {
    if (index == nullptr) return;
    DeviceScope scope(index->s.device);
    delete index;
  });
}

qv_status qv_ivfpq_train(qv_ivfpq* index, const float* vectors, size_t n) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    QV_REQUIRE(vectors != nullptr || n == 0, "vectors must not be null");
    IvfState& s = index->s;
    QV_REQUIRE(n >= s.nlist && n >= static_cast<size_t>(kSubCentroids),
               "IVF-PQ training needs at least max(nlist, 256) vectors");
    check_finite(vectors, n * s.dim);  // src/ivfpq_index.cc:147
    std::unique_lock lock(index->mu);
    QV_REQUIRE(!s.trained, "index is already trained");
    DeviceScope scope(s.device);
    ivf_train(s, vectors, n, thread_stream(s.device));
  });
}

qv_status qv_ivfpq_set_trained(qv_ivfpq* index, const float* centroids, const float* codebooks) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && centroids != nullptr && codebooks != nullptr, "null argument");
    std::unique_lock lock(index->mu);
    IvfState& s = index->s;
    QV_REQUIRE(!s.trained, "index is already trained");
    check_finite(centroids, s.nlist * s.dim);
    check_finite(codebooks, s.m * kSubCentroids * s.dsub);
    DeviceScope scope(s.device);
    ivf_set_trained(s, centroids, codebooks, thread_stream(s.device));
  });
}

qv_status qv_ivfpq_is_trained(const qv_ivfpq* index, int* trained) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && trained != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    *trained = index->s.trained ? 1 : 0;
  });
}

namespace {
constexpr size_t kAddChunkBytes = size_t{64} << 20;  // rows per streamed add() chunk: 64 MiB

// This thread's pinned staging buffer for streamed uploads (grown on demand, kept for reuse).
unsigned char* thread_staging(size_t bytes) {
  struct Staging {
    void* p = nullptr;
    size_t bytes = 0;
    ~Staging() {
      if (p != nullptr) cudaFreeHost(p);
    }
  };
  thread_local Staging st;
  if (st.bytes < bytes) {
    if (st.p != nullptr) QV_CUDA(cudaFreeHost(st.p));
    st.p = nullptr;
    st.bytes = 0;
    QV_CUDA(cudaHostAlloc(&st.p, bytes, cudaHostAllocPortable));
    st.bytes = bytes;
  }
  return static_cast<unsigned char*>(st.p);
}
}  // namespace

// add()'s assignment and PQ encode of n host rows (src/ivfpq_index.cc:234-246), streamed: chunks
// of kAddChunkBytes (QV_IVF_ADD_CHUNK_ROWS rows when set) are copied into one of two pinned
// staging halves on the host while the GPU uploads, normalizes (cosine) and encodes the previous
// chunk. The rows stay on the device (dx) only when the index stores vectors; otherwise the
// device holds two chunks, so a batch larger than the GPU's memory can be added. Every row is
// encoded on its own, so the chunking does not change any code or assignment.
static void ivf_encode_host(const IvfState& s, const float* vectors, size_t n, cudaStream_t st,
                            DeviceBuffer& dx, std::vector<uint32_t>& assign,
                            std::vector<uint8_t>& codes) {
  const size_t row_bytes = s.dim * sizeof(float);
  size_t chunk = std::max<size_t>(1, kAddChunkBytes / row_bytes);
  if (const char* e = std::getenv("QV_IVF_ADD_CHUNK_ROWS"); e != nullptr && *e != '\0')
    chunk = static_cast<size_t>(std::max(1LL, std::atoll(e)));
  chunk = std::min(chunk, n);
  DeviceBuffer da(n * sizeof(uint32_t), st), dc(n * s.m, st);
  DeviceBuffer dchunk[2];
  if (s.store_vectors) {
    dx.allocate(n * row_bytes, st);
  } else {
    dchunk[0].allocate(chunk * row_bytes, st);
    if (chunk < n) dchunk[1].allocate(chunk * row_bytes, st);
  }
  unsigned char* stage = thread_staging(2 * chunk * row_bytes);
  cudaEvent_t uploaded[2] = {nullptr, nullptr};  // a staging half's upload has finished
  for (cudaEvent_t& e : uploaded) QV_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  try {
    for (size_t c = 0, i = 0; c < n; c += chunk, ++i) {
      const size_t rows = std::min(chunk, n - c);
      const int b = static_cast<int>(i & 1);
      unsigned char* half = stage + b * chunk * row_bytes;
      if (i >= 2) QV_CUDA(cudaEventSynchronize(uploaded[b]));
      std::memcpy(half, vectors + c * s.dim, rows * row_bytes);
      float* dst = s.store_vectors ? dx.get<float>() + c * s.dim : dchunk[b].get<float>();
      QV_CUDA(cudaMemcpyAsync(dst, half, rows * row_bytes, cudaMemcpyHostToDevice, st));
      QV_CUDA(cudaEventRecord(uploaded[b], st));
      if (s.metric == QV_METRIC_COSINE) normalize_rows_device(dst, rows, s.dim, st);
      ivf_encode_device(s, dst, rows, da.get<uint32_t>() + c, dc.get<uint8_t>() + c * s.m, st);
    }
    QV_CUDA(cudaStreamSynchronize(st));
  } catch (...) {
    cudaStreamSynchronize(st);
    for (cudaEvent_t e : uploaded) cudaEventDestroy(e);
    throw;
  }
  for (cudaEvent_t e : uploaded) cudaEventDestroy(e);
  assign.resize(n);
  codes.resize(n * s.m);
  QV_CUDA(cudaMemcpyAsync(assign.data(), da.get(), n * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaMemcpyAsync(codes.data(), dc.get(), n * s.m, cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaStreamSynchronize(st));
}

qv_status qv_ivfpq_add(qv_ivfpq* index, const float* vectors, size_t n, const uint64_t* labels) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    QV_REQUIRE(vectors != nullptr || n == 0, "vectors must not be null");
    if (n == 0) return;
    IvfState& s = index->s;
    check_finite(vectors, n * s.dim);
    check_labels(labels, n);
    {
      std::shared_lock lock(index->mu);
      QV_REQUIRE(s.trained, "IVF-PQ index must be trained before add()");
    }
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    DeviceBuffer dx;
    std::vector<uint32_t> assign;
    std::vector<uint8_t> codes;
    ivf_encode_host(s, vectors, n, st, dx, assign, codes);  // trained state is immutable
    std::unique_lock lock(index->mu);
    std::vector<uint64_t> lab(n);
    for (size_t i = 0; i < n; ++i) lab[i] = labels ? labels[i] : s.count + i;
    ivf_append(s, assign, codes, lab, dx.get<float>(), st);
  });
}

qv_status qv_ivfpq_encode(const qv_ivfpq* index, const float* vectors, size_t n, uint32_t* assign,
                          uint8_t* codes) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && (n == 0 || (vectors && assign && codes)), "null argument");
    if (n == 0) return;
    const IvfState& s = index->s;
    check_finite(vectors, n * s.dim);
    std::shared_lock lock(index->mu);
    QV_REQUIRE(s.trained, "IVF-PQ index must be trained before add()");
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    DeviceBuffer dx;
    std::vector<uint32_t> a;
    std::vector<uint8_t> c;
    ivf_encode_host(s, vectors, n, st, dx, a, c);
    std::memcpy(assign, a.data(), n * sizeof(uint32_t));
    std::memcpy(codes, c.data(), n * s.m);
  });
}

qv_status qv_ivfpq_search(const qv_ivfpq* index, const float* queries, size_t nq, size_t k,
                          size_t nprobe, size_t refine_factor, const qv_filter* filter,
                          uint64_t* labels, float* distances) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(index != nullptr, "null index");
    if (nq == 0 || k == 0) return;  // src/ivfpq_index.cc:424
    QV_REQUIRE(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
    const IvfState& s = index->s;
    const size_t total = result_size(nq, k);
    std::shared_lock lock(index->mu);
    if (!s.trained || s.count == 0) {
      check_finite(queries, nq * s.dim);
      fill_unfilled(labels, distances, total);
      return;
    }
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    DeviceBuffer dq, dl(total * sizeof(uint64_t), st), dd(total * sizeof(float), st);
    h2d(dq, queries, nq * s.dim, st);
    DeviceBuffer bm = device_filter(s.labels.get<uint64_t>(), s.count, filter, st);
    ivf_search(s, dq.get<float>(), nq, k, nprobe, refine_factor, bm.get<uint64_t>(),
               dl.get<uint64_t>(), dd.get<float>(), st);
    // The reference rejects non-finite queries before searching (src/ivfpq_index.cc:428):
    // the host scans the batch while the device searches, and on failure nothing is copied out.
    try {
      check_finite(queries, nq * s.dim);
    } catch (...) {
      cudaStreamSynchronize(st);
      throw;
    }
    QV_CUDA(cudaMemcpyAsync(labels, dl.get(), total * sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaMemcpyAsync(distances, dd.get(), total * sizeof(float), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_ivfpq_search_device(const qv_ivfpq* index, const float* queries, size_t nq, size_t k,
                                 size_t nprobe, size_t refine_factor,
                                 const uint64_t* position_bitmap, uint64_t* labels,
                                 float* distances, void* stream) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(index != nullptr, "null index");
    if (nq == 0 || k == 0) return;
    result_size(nq, k);
    const IvfState& s = index->s;
    std::shared_lock lock(index->mu);
    DeviceScope scope(s.device);
    CallerStream call_stream(stream, s.device);
    cudaStream_t st = call_stream.get();
    ivf_search(s, queries, nq, k, nprobe, refine_factor, position_bitmap, labels, distances, st);
  });
}

qv_status qv_ivfpq_candidates_device(const qv_ivfpq* index, const float* queries, size_t nq,
                                     size_t keep, size_t nprobe, const uint64_t* position_bitmap,
                                     float* distances, uint64_t* keys, uint64_t* labels,
                                     void* stream) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(index != nullptr && distances && keys && labels, "null argument");
    const IvfState& s = index->s;
    std::shared_lock lock(index->mu);
    DeviceScope scope(s.device);
    CallerStream call_stream(stream, s.device);
    cudaStream_t st = call_stream.get();
    ivf_candidates(s, queries, nq, keep, nprobe, position_bitmap, distances, keys, labels, st);
  });
}

qv_status qv_ivfpq_refine_device(const qv_ivfpq* index, const float* queries, size_t nq,
                                 size_t keep, const uint64_t* keys, float* exact, void* stream) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && keys && exact, "null argument");
    const IvfState& s = index->s;
    std::shared_lock lock(index->mu);
    DeviceScope scope(s.device);
    CallerStream call_stream(stream, s.device);
    cudaStream_t st = call_stream.get();
    ivf_refine(s, queries, nq, keep, keys, exact, st);
  });
}

qv_status qv_ivfpq_filter_bitmap(const qv_ivfpq* index, const qv_filter* filter,
                                 uint64_t** device_bitmap) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && filter != nullptr && device_bitmap != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    const IvfState& s = index->s;
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    const size_t words = std::max<size_t>(1, (s.count + 63) / 64);
    void* p = nullptr;
    QV_CUDA(cudaMalloc(&p, words * sizeof(uint64_t)));
    build_position_bitmap(s.labels.get<uint64_t>(), s.count, *filter, static_cast<uint64_t*>(p), st);
    QV_CUDA(cudaStreamSynchronize(st));
    *device_bitmap = static_cast<uint64_t*>(p);
  });
}

qv_status qv_ivfpq_info(const qv_ivfpq* index, qv_ivfpq_params* params, size_t* size,
                        size_t* memory_bytes) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr, "null index");
    std::shared_lock lock(index->mu);
    const IvfState& s = index->s;
    if (params) {
      params->dim = s.dim;
      params->metric = s.metric;
      params->nlist = s.nlist;
      params->m = s.m;
      params->train_iterations = s.train_iterations;
      params->store_vectors = s.store_vectors ? 1 : 0;
      params->seed = s.seed;
    }
    if (size) *size = s.count;
    if (memory_bytes) {  // src/ivfpq_index.cc:446-455
      size_t b = (s.trained ? s.nlist * s.dim + s.m * kSubCentroids * s.dsub : 0) * sizeof(float);
      b += s.precomputed.bytes();
      b += s.count * s.m + s.count * sizeof(uint64_t);
      if (s.store_vectors) b += s.count * s.dim * sizeof(float);
      *memory_bytes = b;
    }
  });
}

qv_status qv_ivfpq_list_sizes(const qv_ivfpq* index, uint64_t* sizes) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && sizes != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    const IvfState& s = index->s;
    for (size_t l = 0; l < s.nlist; ++l) sizes[l] = s.host_offsets[l + 1] - s.host_offsets[l];
  });
}

qv_status qv_ivfpq_labels(const qv_ivfpq* index, uint64_t* labels) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && labels != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    std::memcpy(labels, index->s.host_labels.data(), index->s.count * sizeof(uint64_t));
  });
}

qv_status qv_ivfpq_save(const qv_ivfpq* index, const char* path) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && path != nullptr, "null argument");
    std::shared_lock lock(index->mu);
    const IvfState& s = index->s;
    IvfPqMeta meta{s.dim, s.nlist, s.m, s.count, s.train_iterations, s.seed, s.metric,
                   s.store_vectors ? 1u : 0u, s.trained ? 1u : 0u, 0};
    std::vector<float> vec;
    if (s.store_vectors && s.count > 0) {
      vec.resize(s.count * s.dim);
      DeviceScope scope(s.device);
      cudaStream_t st = thread_stream(s.device);
      QV_CUDA(cudaMemcpyAsync(vec.data(), s.vectors.get(), vec.size() * sizeof(float),
                              cudaMemcpyDeviceToHost, st));
      QV_CUDA(cudaStreamSynchronize(st));
    }
    QvrWriter w(QvrKind::kIvfPq);
    w.add(kMeta, &meta, sizeof(meta));
    w.add(kCent, s.host_centroids.data(), s.host_centroids.size() * sizeof(float));
    w.add(kPqcb, s.host_codebooks.data(), s.host_codebooks.size() * sizeof(float));
    w.add(kLoff, s.host_offsets.data(), s.host_offsets.size() * sizeof(uint64_t));
    w.add(kCode, s.host_codes.data(), s.host_codes.size());
    w.add(kLabl, s.host_labels.data(), s.host_labels.size() * sizeof(uint64_t));
    if (s.store_vectors) w.add(kVect, vec.data(), vec.size() * sizeof(float));
    w.commit(path);
  });
}

qv_status qv_ivfpq_load(int device, const char* path, int verify_checksums, qv_ivfpq** out) {
  return guarded(
      [&] { ivf_load_into(out, device, path, verify_checksums != 0, false, 0, UINT64_MAX); });
}

qv_status qv_ivfpq_load_shard(int device, const char* path, int verify_checksums,
                              uint64_t label_begin, uint64_t label_end, qv_ivfpq** out) {
  return guarded([&] {
    ivf_load_into(out, device, path, verify_checksums != 0, true, label_begin, label_end);
  });
}

qv_status qv_ivfpq_set_list_base(qv_ivfpq* index, const uint32_t* base) {
  return guarded([&] {
    QV_REQUIRE(index != nullptr && base != nullptr, "null argument");
    std::unique_lock lock(index->mu);
    IvfState& s = index->s;
    QV_REQUIRE(s.trained, "IVF-PQ index must be trained before set_list_base()");
    s.host_global_base.assign(base, base + s.nlist);
    DeviceScope scope(s.device);
    cudaStream_t st = thread_stream(s.device);
    s.global_base.allocate(s.nlist * sizeof(uint32_t));
    QV_CUDA(cudaMemcpyAsync(s.global_base.get(), s.host_global_base.data(),
                            s.nlist * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

// ---- HNSW storage and exact scan -------------------------------------------------------------------

qv_status qv_hnsw_store_create(int device, size_t dim, uint32_t metric, uint32_t storage,
                               qv_hnsw_store** out) {
  return guarded([&] {
    QV_REQUIRE(out != nullptr, "null argument");
    QV_REQUIRE(dim >= 1 && dim <= kMaxDimension,
               "dimension must be in [1, " + std::to_string(kMaxDimension) + "]");
    check_metric(metric);
    QV_REQUIRE(storage == QV_STORAGE_FLOAT32 || storage == QV_STORAGE_SQ8, "unknown storage");
    int ndev = 0;
    QV_CUDA(cudaGetDeviceCount(&ndev));
    QV_REQUIRE(device >= 0 && device < ndev, "no CUDA device " + std::to_string(device));
    auto h = std::make_unique<qv_hnsw_store>();
    h->s.flat.device = device;
    h->s.flat.dim = dim;
    h->s.flat.metric = metric;
    h->s.storage = storage;
    h->s.flat.sum_order = storage == QV_STORAGE_SQ8 ? kSumOrderSq8 : kSumOrderF32;
    *out = h.release();
  });
}

qv_status qv_hnsw_store_destroy(qv_hnsw_store* store) {
  return guarded([&] {
    if (store == nullptr) return;
    DeviceScope scope(store->s.flat.device);
    delete store;
  });
}

namespace {
// Uploads n host rows and prepares them as HnswIndex does (src/hnsw_index.cc:334-339).
DeviceBuffer upload_prepared(const HnswStoreState& s, const float* vectors, size_t n,
                             cudaStream_t st) {
  DeviceBuffer d;
  h2d(d, vectors, n * s.flat.dim, st);
  if (s.flat.metric == QV_METRIC_COSINE) normalize_rows_device(d.get<float>(), n, s.flat.dim, st);
  return d;
}
}  // namespace

qv_status qv_hnsw_store_train(qv_hnsw_store* store, const float* vectors, size_t n) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr, "null store");
    HnswStoreState& s = store->s;
    QV_REQUIRE(s.storage == QV_STORAGE_SQ8, "train() only applies to SQ8 storage");
    QV_REQUIRE(vectors != nullptr && n > 0, "train() needs at least one vector");
    check_finite(vectors, n * s.flat.dim);
    std::unique_lock lock(store->mu);
    QV_REQUIRE(!s.trained, "index is already trained (SQ8 parameters cannot change once set)");
    DeviceScope scope(s.flat.device);
    cudaStream_t st = thread_stream(s.flat.device);
    DeviceBuffer d = upload_prepared(s, vectors, n, st);
    hnsw_sq8_train(s, d.get<float>(), n, st);
  });
}

qv_status qv_hnsw_store_is_trained(const qv_hnsw_store* store, int* trained) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr && trained != nullptr, "null argument");
    std::shared_lock lock(store->mu);
    *trained = store->s.storage == QV_STORAGE_FLOAT32 || store->s.trained ? 1 : 0;
  });
}

qv_status qv_hnsw_store_add(qv_hnsw_store* store, const float* vectors, size_t n,
                            const uint64_t* labels) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr, "null store");
    if (n == 0) return;
    QV_REQUIRE(vectors != nullptr, "vectors must not be null");
    HnswStoreState& s = store->s;
    check_finite(vectors, n * s.flat.dim);
    check_labels(labels, n);
    if (labels != nullptr && n > 1) {
      std::vector<uint64_t> sorted(labels, labels + n);
      std::sort(sorted.begin(), sorted.end());
      QV_REQUIRE(std::adjacent_find(sorted.begin(), sorted.end()) == sorted.end(),
                 "duplicate labels within one add() call");
    }
    std::unique_lock lock(store->mu);
    DeviceScope scope(s.flat.device);
    cudaStream_t st = thread_stream(s.flat.device);
    const size_t base = s.flat.n;
    QV_REQUIRE(base + n <= std::numeric_limits<uint32_t>::max(),
               "index is full (maximum " + std::to_string(std::numeric_limits<uint32_t>::max()) +
                   " vectors)");
    std::vector<uint64_t> lab(n);
    for (size_t i = 0; i < n; ++i) lab[i] = labels ? labels[i] : base + i;
    // Validate everything before changing anything (src/hnsw_index.cc:588-596): a label may map
    // to a removed node (the mapping is replaced), not to a live one.
    for (uint64_t l : lab) {
      const auto it = s.label_to_id.find(l);
      QV_REQUIRE(it == s.label_to_id.end() ||
                     ((s.host_removed[it->second >> 6] >> (it->second & 63)) & 1ull) != 0,
                 "label " + std::to_string(l) + " is already in the index");
    }
    DeviceBuffer d = upload_prepared(s, vectors, n, st);
    if (s.storage == QV_STORAGE_SQ8 && !s.trained) {
      QV_REQUIRE(n >= 256,
                 "SQ8 index is untrained: call train() with a representative sample, or make the "
                 "first add() at least 256 vectors");
      hnsw_sq8_train(s, d.get<float>(), n, st);
    }
    DeviceBuffer dl;
    h2d(dl, lab.data(), n, st);
    hnsw_store_append(s, d.get<float>(), dl.get<uint64_t>(), n, st);  // waits for the GPU
    s.flat.host_labels.insert(s.flat.host_labels.end(), lab.begin(), lab.end());
    for (size_t i = 0; i < n; ++i) s.label_to_id[lab[i]] = static_cast<uint32_t>(base + i);
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_hnsw_store_remove(qv_hnsw_store* store, uint64_t label, int* removed) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr, "null store");
    HnswStoreState& s = store->s;
    std::unique_lock lock(store->mu);
    int done = 0;
    const auto it = s.label_to_id.find(label);
    if (it != s.label_to_id.end()) {
      const uint32_t id = it->second;
      if (((s.host_removed[id >> 6] >> (id & 63)) & 1ull) == 0) {
        DeviceScope scope(s.flat.device);
        hnsw_store_mark_removed(s, id, thread_stream(s.flat.device));
        done = 1;
      }
    }
    if (removed) *removed = done;
  });
}

qv_status qv_hnsw_store_info(const qv_hnsw_store* store, size_t* live, size_t* nodes, size_t* dim,
                             uint32_t* metric, uint32_t* storage) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr, "null store");
    std::shared_lock lock(store->mu);
    const HnswStoreState& s = store->s;
    if (live) *live = s.flat.n - s.removed_count;
    if (nodes) *nodes = s.flat.n;
    if (dim) *dim = s.flat.dim;
    if (metric) *metric = s.flat.metric;
    if (storage) *storage = s.storage;
  });
}

qv_status qv_hnsw_store_vector(const qv_hnsw_store* store, uint64_t label, float* vector) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr && vector != nullptr, "null argument");
    std::shared_lock lock(store->mu);
    const HnswStoreState& s = store->s;
    const auto it = s.label_to_id.find(label);
    QV_REQUIRE(it != s.label_to_id.end() &&
                   ((s.host_removed[it->second >> 6] >> (it->second & 63)) & 1ull) == 0,
               "label " + std::to_string(label) + " is not in the index");
    DeviceScope scope(s.flat.device);
    cudaStream_t st = thread_stream(s.flat.device);
    QV_CUDA(cudaMemcpyAsync(vector, s.flat.x.get<float>() + it->second * s.flat.dim,
                            s.flat.dim * sizeof(float), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_hnsw_store_codes(const qv_hnsw_store* store, size_t first, size_t count,
                              uint8_t* codes) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr && codes != nullptr, "null argument");
    std::shared_lock lock(store->mu);
    const HnswStoreState& s = store->s;
    QV_REQUIRE(s.storage == QV_STORAGE_SQ8, "the store does not hold SQ8 codes");
    QV_REQUIRE(first <= s.flat.n && count <= s.flat.n - first, "node range out of bounds");
    if (count == 0) return;
    DeviceScope scope(s.flat.device);
    cudaStream_t st = thread_stream(s.flat.device);
    QV_CUDA(cudaMemcpyAsync(codes, s.codes.get<uint8_t>() + first * s.flat.dim,
                            count * s.flat.dim, cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
  });
}

qv_status qv_hnsw_store_sq8_params(const qv_hnsw_store* store, float* vmin, float* vscale) {
  return guarded([&] {
    QV_REQUIRE(store != nullptr, "null store");
    std::shared_lock lock(store->mu);
    const HnswStoreState& s = store->s;
    QV_REQUIRE(s.storage == QV_STORAGE_SQ8 && s.trained, "the store holds no SQ8 parameters");
    if (vmin) std::memcpy(vmin, s.host_vmin.data(), s.flat.dim * sizeof(float));
    if (vscale) std::memcpy(vscale, s.host_vscale.data(), s.flat.dim * sizeof(float));
  });
}

qv_status qv_hnsw_store_search(const qv_hnsw_store* store, const float* queries, size_t nq,
                               size_t k, const qv_filter* filter, uint64_t* labels,
                               float* distances) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(store != nullptr, "null store");
    if (nq == 0 || k == 0) return;
    QV_REQUIRE(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
    const HnswStoreState& s = store->s;
    const size_t total = result_size(nq, k);
    std::shared_lock lock(store->mu);
    DeviceScope scope(s.flat.device);
    cudaStream_t st = thread_stream(s.flat.device);
    SearchFlags& flags = thread_search_flags(s.flat.device);
    DeviceBuffer dq, dl(total * sizeof(uint64_t), st), dd(total * sizeof(float), st);
    QV_CUDA(cudaMemsetAsync(flags.sync_dev, 0, kSearchFlagWords * sizeof(int), st));
    h2d(dq, queries, nq * s.flat.dim, st);
    DeviceBuffer bm = s.flat.n > 0 ? device_filter(s.flat.labels.get<uint64_t>(), s.flat.n,
                                                   filter, st)
                                   : DeviceBuffer();
    if (bm.bytes() == 0) bm.allocate(std::max<size_t>(1, (s.flat.n + 63) / 64) * 8, st);
    hnsw_store_search(s, dq.get<float>(), nq, k, bm.get<uint64_t>(), filter != nullptr,
                      dl.get<uint64_t>(), dd.get<float>(), nullptr, flags.sync_dev, st);
    QV_CUDA(cudaMemcpyAsync(flags.sync_host, flags.sync_dev, kSearchFlagWords * sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaMemcpyAsync(labels, dl.get(), total * sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaMemcpyAsync(distances, dd.get(), total * sizeof(float), cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaStreamSynchronize(st));
    report_flags(flags.sync_host);
  });
}

qv_status qv_hnsw_store_search_device(const qv_hnsw_store* store, const float* queries, size_t nq,
                                      size_t k, const uint64_t* position_bitmap, uint64_t* labels,
                                      float* distances, uint64_t* node_ids, void* stream) {
  return guarded([&] {
    begin_search_stats();
    QV_REQUIRE(store != nullptr, "null store");
    if (nq == 0 || k == 0) return;
    QV_REQUIRE(queries != nullptr && labels != nullptr && distances != nullptr,
               "search_batch: null buffer");
    result_size(nq, k);
    const HnswStoreState& s = store->s;
    std::shared_lock lock(store->mu);
    DeviceScope scope(s.flat.device);
    CallerStream call_stream(stream, s.flat.device);
    cudaStream_t st = call_stream.get();
    SearchFlags& flags = thread_search_flags(s.flat.device);
    if (!thread_timing())
      QV_CUDA(cudaMemsetAsync(flags.dev, 0, kSearchFlagWords * sizeof(int), st));
    // The caller's bitmap is read only: the live-node mask is applied to a copy.
    const size_t words = std::max<size_t>(1, (s.flat.n + 63) / 64);
    DeviceBuffer bm(words * sizeof(uint64_t), st);
    if (position_bitmap != nullptr)
      QV_CUDA(cudaMemcpyAsync(bm.get(), position_bitmap, words * sizeof(uint64_t),
                              cudaMemcpyDeviceToDevice, st));
    hnsw_store_search(s, queries, nq, k, bm.get<uint64_t>(), position_bitmap != nullptr, labels,
                      distances, node_ids, flags.dev, st);
    QV_CUDA(cudaMemcpyAsync(flags.host, flags.dev, kSearchFlagWords * sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    QV_CUDA(cudaEventRecord(flags.done, st));
    t_flags = &flags;
  });
}

// ---- merge -------------------------------------------------------------------------------------

qv_status qv_merge_topk_device(int device, size_t parts, size_t nq, size_t k,
                               const float* distances, const uint64_t* keys,
                               const uint64_t* labels, float* out_distances, uint64_t* out_keys,
                               uint64_t* out_labels, void* stream) {
  return guarded([&] {
    QV_REQUIRE(distances && keys && out_distances, "null argument");
    DeviceScope scope(device);
    CallerStream call_stream(stream, device);
    cudaStream_t st = call_stream.get();
    merge_topk(parts, nq, k, distances, keys, labels, out_distances, out_keys, out_labels, st);
  });
}

qv_status qv_select_topk_device(int device, size_t nq, size_t n, size_t k, const float* distances,
                                const uint64_t* keys, const uint64_t* labels,
                                float* out_distances, uint64_t* out_keys, uint64_t* out_labels,
                                void* stream) {
  return guarded([&] {
    QV_REQUIRE(distances && keys && out_distances, "null argument");
    QV_REQUIRE(k <= n || n == 0, "select_topk: k > n");
    DeviceScope scope(device);
    CallerStream call_stream(stream, device);
    cudaStream_t st = call_stream.get();
    select_topk(nq, n, k, distances, keys, labels, out_distances, out_keys, out_labels, st);
  });
}

}  // extern "C"
