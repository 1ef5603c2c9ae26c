// Internal helpers shared by the quiver-b200 CUDA translation units: error state behind the C ABI,
// device memory ownership, per-thread streams, and the device restatements of the reference's
// float reductions that make distances, assignments and codes bit-identical to the CPU library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>
#include <utility>

#include "qv_gpu.h"

namespace qv {

// ---- error state ------------------------------------------------------------------------------

void set_error(const std::string& msg);
const std::string& last_error();

// Thrown inside the library only; every extern "C" entry point catches it and returns its status.
struct Failure {
  qv_status status;
  std::string msg;
};

[[noreturn]] inline void fail(qv_status s, const std::string& msg) { throw Failure{s, msg}; }

#define QV_REQUIRE(cond, msg)                          \
  do {                                                 \
    if (!(cond)) ::qv::fail(QV_ERR_INVALID, (msg));    \
  } while (0)

#define QV_CUDA(call)                                                                         \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) {                                                                  \
      ::qv::fail(e_ == cudaErrorMemoryAllocation ? QV_ERR_OOM : QV_ERR_CUDA,                  \
                 std::string(#call) + ": " + cudaGetErrorString(e_));                         \
    }                                                                                         \
  } while (0)

// Runs `f` and converts any Failure (or std::bad_alloc) into a status + thread-local message.
template <class F>
qv_status guarded(F&& f) {
  try {
    f();
    return QV_OK;
  } catch (const Failure& e) {
    set_error(e.msg);
    return e.status;
  } catch (const std::bad_alloc&) {
    set_error("out of host memory");
    return QV_ERR_OOM;
  } catch (const std::exception& e) {
    set_error(e.what());
    return QV_ERR_INVALID;
  }
}

// ---- devices, streams, memory -------------------------------------------------------------------

// Makes `device` current for the scope and restores the previous device.
class DeviceScope {
 public:
  explicit DeviceScope(int device) {
    QV_CUDA(cudaGetDevice(&prev_));
    if (prev_ != device) QV_CUDA(cudaSetDevice(device));
  }
  ~DeviceScope() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
  }
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;

 private:
  int prev_ = 0;
};

// The calling thread's non-blocking stream on `device` (created on first use, kept for the
// thread's lifetime), so concurrent host threads never serialize on one stream.
cudaStream_t thread_stream(int device);

// Owning device allocation. Allocated with cudaMallocAsync on a stream when given one.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  DeviceBuffer(size_t bytes, cudaStream_t stream = nullptr) { allocate(bytes, stream); }
  ~DeviceBuffer() { release(); }
  DeviceBuffer(DeviceBuffer&& o) noexcept { swap(o); }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
      release();
      swap(o);
    }
    return *this;
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;

  void allocate(size_t bytes, cudaStream_t stream = nullptr) {
    release();
    if (bytes == 0) return;
    if (stream != nullptr) {
      QV_CUDA(cudaMallocAsync(&ptr_, bytes, stream));
      stream_ = stream;
    } else {
      QV_CUDA(cudaMalloc(&ptr_, bytes));
    }
    bytes_ = bytes;
  }
  void release() noexcept {
    if (ptr_ != nullptr) {
      if (stream_ != nullptr) {
        cudaFreeAsync(ptr_, stream_);
      } else {
        cudaFree(ptr_);
      }
    }
    ptr_ = nullptr;
    bytes_ = 0;
    stream_ = nullptr;
  }
  template <class T = void>
  T* get() const noexcept {
    return static_cast<T*>(ptr_);
  }
  size_t bytes() const noexcept { return bytes_; }

 private:
  void swap(DeviceBuffer& o) noexcept {
    std::swap(ptr_, o.ptr_);
    std::swap(bytes_, o.bytes_);
    std::swap(stream_, o.stream_);
  }
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
  cudaStream_t stream_ = nullptr;
};

// Per-thread launch accounting behind qv_last_search_stats().
struct SearchStats {
  uint64_t kernel_launches = 0;
  uint64_t rescanned_queries = 0;
  double dominant_ms = 0.0;
  double dominant_work = 0.0;
  bool work_is_bytes = false;
  std::string dominant_name;
};
SearchStats& thread_stats();
bool& thread_timing();  // qv_set_timing

// Starts a new search's accounting: with timing off the counters describe the last search only;
// with timing on they accumulate until qv_last_search_stats reads (and resets) them.
void begin_search_stats();

// A timed launch whose CUDA events have not been read yet. `count` (a pinned host slot, filled by
// a copy queued on the launch's stream, or nullptr) adds count * per_count to the work once the
// events have completed (work that is only known on the device, e.g. the list lengths a scan
// visited).
struct PendingTimer {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  const char* name = "";
  double work = 0.0;
  bool bytes = false;
  const unsigned long long* count = nullptr;
  double per_count = 0.0;
};
// Queues a timed launch; resolve_timers() waits for the queued events, adds their elapsed time
// and work to the thread's stats and releases them.
void defer_timer(const PendingTimer& t);
void resolve_timers();
// A pinned host slot for a device-side work counter of a timed launch (per thread, reused
// round-robin; valid until several thousand later timed launches).
unsigned long long* timing_count_slot();

// Brackets one launch with CUDA events when timing is on. Nothing waits for them here: stop()
// queues them, so timing adds no host synchronization to the search.
class KernelTimer {
 public:
  KernelTimer(cudaStream_t st, const char* name, double work, bool is_bytes)
      : st_(st), on_(thread_timing()) {
    t_.name = name;
    t_.work = work;
    t_.bytes = is_bytes;
    if (on_) {
      cudaEventCreate(&t_.e0);
      cudaEventCreate(&t_.e1);
      cudaEventRecord(t_.e0, st_);
    }
  }
  // Work counted on the device: count (a timing_count_slot filled on the stream) * per_count.
  void set_device_count(const unsigned long long* count, double per_count) {
    t_.count = count;
    t_.per_count = per_count;
  }
  bool on() const { return on_; }
  void stop() {
    if (!on_) return;
    cudaEventRecord(t_.e1, st_);
    defer_timer(t_);
    on_ = false;
  }
  ~KernelTimer() {
    if (on_) {  // not stopped (the launch failed)
      cudaEventDestroy(t_.e0);
      cudaEventDestroy(t_.e1);
    }
  }
  KernelTimer(const KernelTimer&) = delete;
  KernelTimer& operator=(const KernelTimer&) = delete;

 private:
  cudaStream_t st_;
  bool on_;
  PendingTimer t_;
};
inline void count_launch(uint64_t n = 1) { thread_stats().kernel_launches += n; }

inline void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) fail(QV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  count_launch();
}

// Host-side input validation, as the reference's check_finite (src/flat_index.cc:34-38).
void check_finite(const float* v, size_t count);

// Number of SMs of `device` (cached).
int sm_count(int device);

constexpr int kSubCentroids = 256;
constexpr uint64_t kInvalidLabel = UINT64_MAX;

inline size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }
inline size_t next_pow2(size_t x) {
  size_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace qv

// ---- device restatements of the reference's float reductions ------------------------------------
//
// Every operation names its rounding: __fmaf_rn where the reference executes an FMA,
// __fmul_rn/__fadd_rn/__fsub_rn where it rounds a product and a sum separately. nvcc would otherwise
// contract a*b+c into an FMA and change the last bit.

namespace qv::dev {

constexpr unsigned kFull = 0xffffffffu;

// simd::avx2::dot (src/simd/kernels_avx2.cc:63-83), evaluated by one warp. Lane l owns the AVX2
// accumulator element s[l >> 3][l & 7], so the 32-element blocks are read coalesced; the combine
// is (s0+s1)+(s2+s3) per lane, then hsum (:17-23): (t[l]+t[l+4]) pairs, then (lo0+lo1)+(lo2+lo3).
// The dim % 8 tail follows what GCC emits for the reference's scalar loop under its build flags:
// with 4 or more elements left, the first 4 products are rounded and added in order, the rest
// are FMAs. All lanes return the same value.
template <bool kDiff>
__device__ __forceinline__ float warp_reduce_avx2(const float* __restrict__ a,
                                                  const float* __restrict__ b, int dim, int lane) {
  float s = 0.0f;
  int i = 0;
  for (; i + 32 <= dim; i += 32) {
    float u = a[i + lane], v = b[i + lane];
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    s = __fmaf_rn(u, v, s);
  }
  for (; i + 8 <= dim; i += 8) {
    if (lane < 8) {
      float u = a[i + lane], v = b[i + lane];
      if (kDiff) {
        u = __fsub_rn(u, v);
        v = u;
      }
      s = __fmaf_rn(u, v, s);
    }
  }
  const float s1 = __shfl_down_sync(kFull, s, 8);
  const float s2 = __shfl_down_sync(kFull, s, 16);
  const float s3 = __shfl_down_sync(kFull, s, 24);
  const float t = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
  const float lo = __fadd_rn(t, __shfl_down_sync(kFull, t, 4));
  const float lo1 = __shfl_down_sync(kFull, lo, 1);
  const float lo2 = __shfl_down_sync(kFull, lo, 2);
  const float lo3 = __shfl_down_sync(kFull, lo, 3);
  float sum = __fadd_rn(__fadd_rn(lo, lo1), __fadd_rn(lo2, lo3));
  sum = __shfl_sync(kFull, sum, 0);
  int j = i;
  if (dim - i >= 4) {
    for (; j < i + 4; ++j) {
      float u = a[j], v = b[j];
      if (kDiff) {
        u = __fsub_rn(u, v);
        v = u;
      }
      sum = __fadd_rn(sum, __fmul_rn(u, v));
    }
  }
  for (; j < dim; ++j) {
    float u = a[j], v = b[j];
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    sum = __fmaf_rn(u, v, sum);
  }
  return sum;
}

// The same reduction for four rows b[0..3] against one vector a, with the four rows' loads
// interleaved so that their memory latencies overlap. Each result is bit-identical to
// warp_reduce_avx2<kDiff>(a, b[r], dim, lane).
template <bool kDiff>
__device__ __forceinline__ void warp_reduce_avx2_x4(const float* __restrict__ a,
                                                    const float* const (&b)[4], int dim,
                                                    int lane, float (&out)[4]) {
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int i = 0;
  for (; i + 32 <= dim; i += 32) {
    const float u = a[i + lane];
    float v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = b[r][i + lane];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float x = u, y = v[r];
      if (kDiff) {
        x = __fsub_rn(u, v[r]);
        y = x;
      }
      s[r] = __fmaf_rn(x, y, s[r]);
    }
  }
  for (; i + 8 <= dim; i += 8) {
    if (lane < 8) {
      const float u = a[i + lane];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float x = u, y = b[r][i + lane];
        if (kDiff) {
          x = __fsub_rn(u, y);
          y = x;
        }
        s[r] = __fmaf_rn(x, y, s[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float s1 = __shfl_down_sync(kFull, s[r], 8);
    const float s2 = __shfl_down_sync(kFull, s[r], 16);
    const float s3 = __shfl_down_sync(kFull, s[r], 24);
    const float t = __fadd_rn(__fadd_rn(s[r], s1), __fadd_rn(s2, s3));
    const float lo = __fadd_rn(t, __shfl_down_sync(kFull, t, 4));
    const float lo1 = __shfl_down_sync(kFull, lo, 1);
    const float lo2 = __shfl_down_sync(kFull, lo, 2);
    const float lo3 = __shfl_down_sync(kFull, lo, 3);
    out[r] = __shfl_sync(kFull, __fadd_rn(__fadd_rn(lo, lo1), __fadd_rn(lo2, lo3)), 0);
  }
  int j = i;
  if (dim - i >= 4) {
    for (; j < i + 4; ++j) {
      const float u = a[j];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float x = u, y = b[r][j];
        if (kDiff) {
          x = __fsub_rn(u, y);
          y = x;
        }
        out[r] = __fadd_rn(out[r], __fmul_rn(x, y));
      }
    }
  }
  for (; j < dim; ++j) {
    const float u = a[j];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float x = u, y = b[r][j];
      if (kDiff) {
        x = __fsub_rn(u, y);
        y = x;
      }
      out[r] = __fmaf_rn(x, y, out[r]);
    }
  }
}

// simd::avx2::l2sqr_sq8 / dot_sq8 (src/simd/kernels_avx2.cc:85-129) evaluated by one warp on
// the decoded row b (b[i] = vmin[i] + code[i] * vscale[i] rounded once, the FMA those kernels
// decode with): lane l < 16 owns accumulator s[l >> 3][l & 7] of the 16-element blocks,
// 8-element blocks go to s0 (lanes 0..7), then s0 + s1 per lane, the hsum (:17-23), and the
// scalar tail, every element of which is one FMA. All lanes return the same value.
template <bool kDiff>
__device__ __forceinline__ float warp_reduce_sq8(const float* __restrict__ a,
                                                 const float* __restrict__ b, int dim, int lane) {
  float s = 0.0f;
  int i = 0;
  for (; i + 16 <= dim; i += 16) {
    if (lane < 16) {
      float u = a[i + lane], v = b[i + lane];
      if (kDiff) {
        u = __fsub_rn(u, v);
        v = u;
      }
      s = __fmaf_rn(u, v, s);
    }
  }
  for (; i + 8 <= dim; i += 8) {
    if (lane < 8) {
      float u = a[i + lane], v = b[i + lane];
      if (kDiff) {
        u = __fsub_rn(u, v);
        v = u;
      }
      s = __fmaf_rn(u, v, s);
    }
  }
  const float t = __fadd_rn(s, __shfl_down_sync(kFull, s, 8));
  const float lo = __fadd_rn(t, __shfl_down_sync(kFull, t, 4));
  const float lo1 = __shfl_down_sync(kFull, lo, 1);
  const float lo2 = __shfl_down_sync(kFull, lo, 2);
  const float lo3 = __shfl_down_sync(kFull, lo, 3);
  float sum = __shfl_sync(kFull, __fadd_rn(__fadd_rn(lo, lo1), __fadd_rn(lo2, lo3)), 0);
  for (; i < dim; ++i) {
    float u = a[i], v = b[i];
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    sum = __fmaf_rn(u, v, sum);
  }
  return sum;
}

// The SQ8 kernels' distance (src/hnsw_index.cc:202-218): l2sqr_sq8, or 1 - dot_sq8.
__device__ __forceinline__ float warp_exact_distance_sq8(const float* q, const float* x, int dim,
                                                         bool l2, int lane) {
  if (l2) return warp_reduce_sq8<true>(q, x, dim, lane);
  return __fsub_rn(1.0f, warp_reduce_sq8<false>(q, x, dim, lane));
}

// CentroidTable::l2 / ::dot (src/internal/centroid_table.h:65-85): one sequential sum from 0.0f,
// every multiply and add rounded on its own. Every lane computes the same sum.
template <bool kDiff>
__device__ __forceinline__ float seq_reduce(const float* __restrict__ a, const float* __restrict__ b,
                                            int dim) {
  float s = 0.0f;
  for (int i = 0; i < dim; ++i) {
    float u = a[i], v = b[i];
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    s = __fadd_rn(s, __fmul_rn(u, v));
  }
  return s;
}

// CentroidTable::nearest_batch's distance (src/internal/centroid_table.h:94-144): ||x||^2 and
// <q,x> as sequential, separately rounded sums, then ||x||^2 - 2<q,x> rounded once.
__device__ __forceinline__ float seq_norm_minus_2dot(const float* __restrict__ q,
                                                     const float* __restrict__ x, int dim) {
  float dot = 0.0f, nn = 0.0f;
  for (int i = 0; i < dim; ++i) {
    const float v = x[i];
    dot = __fadd_rn(dot, __fmul_rn(q[i], v));
    nn = __fadd_rn(nn, __fmul_rn(v, v));
  }
  return __fsub_rn(nn, __fmul_rn(2.0f, dot));
}

// The exact distance of one row for an exact-distance kind (summation order | kKindNegIp).
__device__ __forceinline__ float warp_exact_distance_kind(const float* q, const float* x, int dim,
                                                          bool l2, int lane, int kind) {
  const int order = kind & 3;
  if (order == 1) return warp_exact_distance_sq8(q, x, dim, l2, lane);
  if (order == 3 && l2) return seq_norm_minus_2dot(q, x, dim);
  if (order >= 2) {
    if (l2) return seq_reduce<true>(q, x, dim);
    const float s = seq_reduce<false>(q, x, dim);
    return (kind & 4) ? -s : __fsub_rn(1.0f, s);
  }
  if (l2) return warp_reduce_avx2<true>(q, x, dim, lane);
  const float s = warp_reduce_avx2<false>(q, x, dim, lane);
  return (kind & 4) ? -s : __fsub_rn(1.0f, s);
}

// warp_exact_distance for four rows at once (see warp_reduce_avx2_x4); kind as
// warp_exact_distance_kind (the float32 kernels' order, 1 - <q,x>, by default).
__device__ __forceinline__ void warp_exact_distance_x4(const float* q, const float* const (&x)[4],
                                                       int dim, bool l2, int lane,
                                                       float (&out)[4], int kind = 0) {
  if (kind != 0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] = warp_exact_distance_kind(q, x[r], dim, l2, lane, kind);
  } else if (l2) {
    warp_reduce_avx2_x4<true>(q, x, dim, lane, out);
  } else {
    warp_reduce_avx2_x4<false>(q, x, dim, lane, out);
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] = __fsub_rn(1.0f, out[r]);
  }
}

__device__ __forceinline__ float warp_dot_avx2(const float* a, const float* b, int dim, int lane) {
  return warp_reduce_avx2<false>(a, b, dim, lane);
}
__device__ __forceinline__ float warp_l2sqr_avx2(const float* a, const float* b, int dim,
                                                 int lane) {
  return warp_reduce_avx2<true>(a, b, dim, lane);
}

// The reference's exact distance (src/flat_index.cc:87, src/ivfpq_index.cc:138-142).
__device__ __forceinline__ float warp_exact_distance(const float* q, const float* x, int dim,
                                                     bool l2, int lane) {
  if (l2) return warp_l2sqr_avx2(q, x, dim, lane);
  return __fsub_rn(1.0f, warp_dot_avx2(q, x, dim, lane));
}

// Distances order NaN after everything (src/flat_index.cc:88).
__device__ __forceinline__ float nan_to_inf(float d) { return d == d ? d : __int_as_float(0x7f800000); }

// Strict weak order on (distance, key): the canonical tie-break used by every selection.
// Bitwise, not short-circuit, operators: the compare stays branch-free (in the sorting networks
// the short-circuit form was compiled to divergent branches and ran ~3x slower).
__device__ __forceinline__ bool key_less(float da, uint64_t ka, float db, uint64_t kb) {
  return (da < db) | ((da == db) & (ka < kb));
}

// float -> uint32 whose unsigned order matches the float order (for atomicMin on thresholds).
__device__ __forceinline__ uint32_t ordered_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_ordered_bits(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__device__ __forceinline__ bool bitmap_test(const uint64_t* bm, uint64_t pos) {
  return bm == nullptr || ((bm[pos >> 6] >> (pos & 63)) & 1ull) != 0;
}

// Block-wide bitonic sort of n (power of two) (distance, key) pairs in shared memory, ascending.
// Optionally carries a 64-bit payload. All threads of the block must call it.
template <bool kPayload>
__device__ void block_bitonic_sort(float* d, uint64_t* k, uint64_t* p, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = ((lo & size) == 0);
        const bool swap = up ? key_less(d[hi], k[hi], d[lo], k[lo])
                             : key_less(d[lo], k[lo], d[hi], k[hi]);
        if (swap) {
          float td = d[lo];
          d[lo] = d[hi];
          d[hi] = td;
          uint64_t tk = k[lo];
          k[lo] = k[hi];
          k[hi] = tk;
          if (kPayload) {
            uint64_t tp = p[lo];
            p[lo] = p[hi];
            p[hi] = tp;
          }
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace qv::dev
