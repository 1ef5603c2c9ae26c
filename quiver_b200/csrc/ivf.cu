// IVF-PQ on the GPU: trained-state preparation, the assign + PQ encode of add(), and search
// (coarse probe, lookup tables, ADC scan of the probed inverted lists with a bitmap filter, and
// the optional exact re-rank). Reference: src/ivfpq_index.cc, src/product_quantizer.cc,
// src/internal/centroid_table.h.
//
// Bit-exactness: every value the reference computes in float32 (centroid norms, coarse distances,
// assignments, residuals, codes, lookup tables, ADC sums, precomputed terms, exact re-rank
// distances) is computed here with the same operations in the same order and the same rounding
// (__fmul_rn/__fadd_rn/__fsub_rn for separately rounded steps). Ties between equal distances are
// broken by the candidate key (list << 32 | offset in the full list) and probes by list id; the
// reference leaves both unspecified.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include "qv_state.h"

namespace qv {
namespace {

constexpr float kInf = __builtin_huge_valf();
constexpr size_t kMaxPrecomputedBytes = size_t{256} << 20;  // src/ivfpq_index.cc:74
constexpr int kScanThreads = 256;
constexpr int kSeqLists = 256;  // probes up to which inner-product scans run as one sequence

// ---- trained state -------------------------------------------------------------------------------

// CentroidTable::reset norms (src/internal/centroid_table.h:43-59): sequential, separately rounded.
__global__ void centroid_norms_kernel(const float* c, size_t k, int dim, float* out) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= k) return;
  const float* v = c + i * dim;
  float s = 0.0f;
  for (int j = 0; j < dim; ++j) s = __fadd_rn(s, __fmul_rn(v[j], v[j]));
  out[i] = s;
}

// Impl::precompute (src/ivfpq_index.cc:112-129): v += r*r + 2*c*r over t, each step rounded.
__global__ void precompute_kernel(const float* cents, size_t nlist, const float* cb, int m,
                                  int dsub, float* pre) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t total = nlist * m * kSubCentroids;
  if (i >= total) return;
  const int c = static_cast<int>(i % kSubCentroids);
  const int j = static_cast<int>((i / kSubCentroids) % m);
  const size_t l = i / (static_cast<size_t>(kSubCentroids) * m);
  const float* cl = cents + l * (static_cast<size_t>(m) * dsub) + static_cast<size_t>(j) * dsub;
  const float* r = cb + (static_cast<size_t>(j) * kSubCentroids + c) * dsub;
  float v = 0.0f;
  for (int t = 0; t < dsub; ++t) {
    const float rr = __fmul_rn(r[t], r[t]);
    const float cr = __fmul_rn(__fmul_rn(2.0f, cl[t]), r[t]);
    v = __fadd_rn(v, __fadd_rn(rr, cr));
  }
  pre[i] = v;
}

// ---- coarse distances and assignment ---------------------------------------------------------------

// Search-time coarse distances (src/ivfpq_index.cc:285-297 with CentroidTable::l2 / ::dot):
// L2: sum_j (q_j - c_j)^2; IP/cosine: -(sum_j q_j c_j), j ascending, separately rounded.
// 4 queries x 8 centroids per thread (a block covers 128 queries x 64 centroids): each dimension
// step issues three 16-byte shared loads for 32 (query, centroid) updates. Each sum is sequential
// in j with every operation rounded separately.
constexpr int kTileP4 = 128;  // queries per block (4 per thread)
constexpr int kTileC4 = 64;   // centroids per block (8 per thread)
constexpr int kTileD4 = 32;   // dimensions per shared tile
constexpr int kXs4 = kTileP4 + 4;  // padded row strides (16-byte aligned, 4-way store conflicts)
constexpr int kCs4 = kTileC4 + 4;

__global__ void __launch_bounds__(256) coarse_dist_kernel4(const float* __restrict__ q, size_t nq,
                                                           const float* __restrict__ cents,
                                                           size_t nlist, int dim, bool ip,
                                                           float* __restrict__ out) {
  __shared__ __align__(16) float xs[kTileD4 * kXs4];  // xs[j][p]
  __shared__ __align__(16) float cs[kTileD4 * kCs4];  // cs[j][c]
  const int pl = threadIdx.x & 31, cl = threadIdx.x >> 5;  // queries 4pl.., centroids 8cl..
  const size_t p0 = static_cast<size_t>(blockIdx.x) * kTileP4;
  const size_t c0 = static_cast<size_t>(blockIdx.y) * kTileC4;
  float acc[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[a][i] = 0.0f;
  for (int d0 = 0; d0 < dim; d0 += kTileD4) {
    const int nd = min(kTileD4, dim - d0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < kTileP4 * kTileD4; idx += 256) {
      const int p = idx / kTileD4, j = idx - p * kTileD4;
      const size_t gp = p0 + p;
      xs[j * kXs4 + p] = (gp < nq && j < nd) ? q[gp * dim + d0 + j] : 0.0f;
    }
    for (int idx = threadIdx.x; idx < kTileC4 * kTileD4; idx += 256) {
      const int c = idx / kTileD4, j = idx - c * kTileD4;
      const size_t gc = c0 + c;
      cs[j * kCs4 + c] = (gc < nlist && j < nd) ? cents[gc * dim + d0 + j] : 0.0f;
    }
    __syncthreads();
    for (int j = 0; j < nd; ++j) {
      const float4 xq = *reinterpret_cast<const float4*>(xs + j * kXs4 + 4 * pl);
      const float4 c_lo = *reinterpret_cast<const float4*>(cs + j * kCs4 + 8 * cl);
      const float4 c_hi = *reinterpret_cast<const float4*>(cs + j * kCs4 + 8 * cl + 4);
      const float xv[4] = {xq.x, xq.y, xq.z, xq.w};
      const float cv[8] = {c_lo.x, c_lo.y, c_lo.z, c_lo.w, c_hi.x, c_hi.y, c_hi.z, c_hi.w};
#pragma unroll
      for (int a = 0; a < 4; ++a) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (ip) {
            acc[a][i] = __fadd_rn(acc[a][i], __fmul_rn(xv[a], cv[i]));
          } else {
            const float d = __fsub_rn(xv[a], cv[i]);
            acc[a][i] = __fadd_rn(acc[a][i], __fmul_rn(d, d));
          }
        }
      }
    }
  }
  const size_t cb = c0 + 8 * static_cast<size_t>(cl);
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const size_t gp = p0 + 4 * pl + a;
    if (gp >= nq) continue;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (cb + i < nlist) out[gp * nlist + cb + i] = ip ? -acc[a][i] : acc[a][i];
  }
}

// CentroidTable::nearest_batch (src/internal/centroid_table.h:94-144) with the register tiling of
// coarse_dist_kernel4: a block covers 128 points and loops over every 64-centroid tile; a thread
// accumulates <x, c> for 4 points x 8 centroids (each sum sequential in the dimension, separately
// rounded), turns them into d = ||c||^2 - 2<x,c> (or -<x,c> by_ip) and keeps, per point, the
// first strict minimum over its ascending centroids; the 8 centroid lanes are then merged by
// (distance, centroid), which keeps the lowest centroid among equal minima. (+inf, 0) start, as
// the reference's zero-initialized output, so a point whose every distance is +inf or NaN gets 0.
__global__ void __launch_bounds__(256) coarse_assign_kernel4(const float* __restrict__ x, size_t n,
                                                             const float* __restrict__ cents,
                                                             const float* __restrict__ cnorm2,
                                                             size_t nlist, int dim, bool by_ip,
                                                             uint32_t* __restrict__ out) {
  __shared__ __align__(16) float xs[kTileD4 * kXs4];  // xs[j][p]
  __shared__ __align__(16) float cs[kTileD4 * kCs4];  // cs[j][c]
  __shared__ float rbd[8][kTileP4];
  __shared__ uint32_t rbc[8][kTileP4];
  const int pl = threadIdx.x & 31, cl = threadIdx.x >> 5;  // points 4pl.., centroids 8cl..
  const size_t p0 = static_cast<size_t>(blockIdx.x) * kTileP4;
  float best_d[4];
  uint32_t best_c[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    best_d[a] = kInf;
    best_c[a] = 0;
  }
  for (size_t c0 = 0; c0 < nlist; c0 += kTileC4) {
    float acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[a][i] = 0.0f;
    for (int d0 = 0; d0 < dim; d0 += kTileD4) {
      const int nd = min(kTileD4, dim - d0);
      __syncthreads();
      for (int idx = threadIdx.x; idx < kTileP4 * kTileD4; idx += 256) {
        const int p = idx / kTileD4, j = idx - p * kTileD4;
        const size_t gp = p0 + p;
        xs[j * kXs4 + p] = (gp < n && j < nd) ? x[gp * dim + d0 + j] : 0.0f;
      }
      for (int idx = threadIdx.x; idx < kTileC4 * kTileD4; idx += 256) {
        const int c = idx / kTileD4, j = idx - c * kTileD4;
        const size_t gc = c0 + c;
        cs[j * kCs4 + c] = (gc < nlist && j < nd) ? cents[gc * dim + d0 + j] : 0.0f;
      }
      __syncthreads();
      for (int j = 0; j < nd; ++j) {
        const float4 xq = *reinterpret_cast<const float4*>(xs + j * kXs4 + 4 * pl);
        const float4 c_lo = *reinterpret_cast<const float4*>(cs + j * kCs4 + 8 * cl);
        const float4 c_hi = *reinterpret_cast<const float4*>(cs + j * kCs4 + 8 * cl + 4);
        const float xv[4] = {xq.x, xq.y, xq.z, xq.w};
        const float cv[8] = {c_lo.x, c_lo.y, c_lo.z, c_lo.w, c_hi.x, c_hi.y, c_hi.z, c_hi.w};
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[a][i] = __fadd_rn(acc[a][i], __fmul_rn(xv[a], cv[i]));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const size_t c = c0 + 8 * static_cast<size_t>(cl) + i;
      if (c >= nlist) continue;
      const float cn = by_ip ? 0.0f : cnorm2[c];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float d = by_ip ? -acc[a][i] : __fsub_rn(cn, __fmul_rn(2.0f, acc[a][i]));
        if (d < best_d[a]) {  // ascending c within this thread: strict < keeps the first minimum
          best_d[a] = d;
          best_c[a] = static_cast<uint32_t>(c);
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    rbd[cl][4 * pl + a] = best_d[a];
    rbc[cl][4 * pl + a] = best_c[a];
  }
  __syncthreads();
  if (cl == 0) {
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int p = 4 * pl + a;
      float d = rbd[0][p];
      uint32_t c = rbc[0][p];
      for (int i = 1; i < 8; ++i) {
        const float di = rbd[i][p];
        const uint32_t ci = rbc[i][p];
        if (di < d || (di == d && ci < c)) {
          d = di;
          c = ci;
        }
      }
      const size_t gp = p0 + p;
      if (gp < n) out[gp] = c;
    }
  }
}

// partial_sort of the nlist probe candidates (src/ivfpq_index.cc:298-300), ties by list id.
__global__ void select_probes_kernel(const float* __restrict__ coarse, size_t nlist, int pool,
                                     int nprobe, uint32_t* __restrict__ probes,
                                     float* __restrict__ probe_d) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sd = reinterpret_cast<float*>(smem_raw);
  uint64_t* sk = reinterpret_cast<uint64_t*>(sd + pool);
  const size_t q = blockIdx.x;
  for (int i = threadIdx.x; i < pool; i += blockDim.x) {
    if (static_cast<size_t>(i) < nlist) {
      sd[i] = coarse[q * nlist + i];
      sk[i] = static_cast<uint64_t>(i);
    } else {
      sd[i] = kInf;
      sk[i] = ~0ull;
    }
  }
  dev::block_bitonic_sort<false>(sd, sk, nullptr, pool);
  for (int i = threadIdx.x; i < nprobe; i += blockDim.x) {
    probes[q * nprobe + i] = static_cast<uint32_t>(sk[i]);
    probe_d[q * nprobe + i] = sd[i];
  }
}

// The same selection for nprobe <= kRadixProbeMax without sorting all nlist candidates: a radix
// select on the 64-bit composite (order-preserving bits of the distance, with -0 read as +0 since
// the reference compares distances with <) << 32 | list id, eight bits a pass from the top, one
// shared 256-bin histogram per pass, until the nprobe-th smallest composite is known. Composites
// are distinct, so exactly nprobe of them lie at or below it; those are gathered and sorted.
// kShared keeps the composites in shared memory; without it (nlist too large for that) every pass
// recomputes them from the coarse distances in global memory.
constexpr int kRadixProbeMax = 1024;
constexpr int kRadixThreads = 256;
constexpr size_t kRadixSharedMax = 160 * 1024;  // composites held in shared memory up to this

template <bool kShared>
__global__ void __launch_bounds__(kRadixThreads) select_probes_radix_kernel(
    const float* __restrict__ coarse, size_t nlist, int nprobe, int id_passes, int sort_n,
    uint32_t* __restrict__ probes, float* __restrict__ probe_d) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* sel = reinterpret_cast<uint64_t*>(smem_raw);   // sort_n selected (padded with ~0)
  uint64_t* comp = sel + sort_n;                           // nlist composites (kShared)
  __shared__ unsigned hist[256];
  __shared__ uint64_t s_prefix;
  __shared__ unsigned s_need;
  __shared__ int s_count;
  const size_t q = blockIdx.x;
  const float* row = coarse + q * nlist;
  auto composite = [&](size_t i) {
    const float d = row[i] + 0.0f;  // -0 -> +0
    return (static_cast<uint64_t>(dev::ordered_bits(d)) << 32) | i;
  };
  if (kShared)
    for (size_t i = threadIdx.x; i < nlist; i += kRadixThreads) comp[i] = composite(i);
  uint64_t prefix = 0;
  unsigned need = static_cast<unsigned>(nprobe);  // rank (1-based) of the target among matches
  const int passes = 4 + id_passes;
  static_assert(kRadixThreads == 256, "one histogram bin per thread");
  for (int p = 0; p < passes; ++p) {
    // Distance bytes from the top, then the id's bytes below 256^id_passes (the higher id bytes
    // are zero in every composite).
    const int shift = p < 4 ? 56 - 8 * p : 8 * (id_passes - 1 - (p - 4));
    hist[threadIdx.x] = 0;
    __syncthreads();
    const uint64_t above = p == 0 ? 0ull : ~0ull << (shift + 8);
    for (size_t i = threadIdx.x; i < nlist; i += kRadixThreads) {
      const uint64_t c = kShared ? comp[i] : composite(i);
      if ((c & above) == prefix) atomicAdd(&hist[(c >> shift) & 255], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      unsigned h[8], sum = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        h[b] = hist[lane * 8 + b];
        sum += h[b];
      }
      unsigned incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      unsigned cum = incl - sum;  // matches in the bins before this lane's
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (cum < need && need <= cum + h[b]) {
          s_prefix = prefix | (static_cast<uint64_t>(lane * 8 + b) << shift);
          s_need = need - cum;
        }
        cum += h[b];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
  }
  // prefix is now the nprobe-th smallest composite.
  if (threadIdx.x == 0) s_count = 0;
  for (int i = threadIdx.x; i < sort_n; i += kRadixThreads) sel[i] = ~0ull;
  __syncthreads();
  for (size_t i = threadIdx.x; i < nlist; i += kRadixThreads) {
    const uint64_t c = kShared ? comp[i] : composite(i);
    if (c <= prefix) {
      const int at = atomicAdd(&s_count, 1);
      if (at < sort_n) sel[at] = c;  // exactly nprobe <= sort_n arrive
    }
  }
  __syncthreads();
  for (int size = 2; size <= sort_n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < sort_n / 2; i += kRadixThreads) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t a = sel[lo], b = sel[hi];
        if ((a > b) == up) {
          sel[lo] = b;
          sel[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < nprobe; i += kRadixThreads) {
    const uint32_t l = static_cast<uint32_t>(sel[i] & 0xffffffffu);
    probes[q * nprobe + i] = l;
    probe_d[q * nprobe + i] = row[l];
  }
}

// ---- encode ------------------------------------------------------------------------------------------

// residual = v - c_l (src/ivfpq_index.cc:243)
__global__ void residual_kernel(const float* __restrict__ x, size_t n, int dim,
                                const float* __restrict__ cents, const uint32_t* __restrict__ assign,
                                float* __restrict__ out) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= n * dim) return;
  const size_t row = i / dim;
  const int j = static_cast<int>(i - row * dim);
  out[i] = __fsub_rn(x[i], cents[static_cast<size_t>(assign[row]) * dim + j]);
}

// ProductQuantizer::encode (src/product_quantizer.cc:165-171): per sub-space the first index of
// the minimum of sum_t (r_t - cb_t)^2 (CentroidTable::l2 + argmin_n). grid.y = sub-space.
// kD = the sub-space width when it is a compile-time constant (the thread's residual slice then
// stays in registers for all 256 sub-centroids), 0 for any other width.
template <int kD>
__global__ void pq_encode_kernel(const float* __restrict__ resid, size_t n, int dim, int m,
                                 int dsub_rt, const float* __restrict__ cb,
                                 uint8_t* __restrict__ codes) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sc = reinterpret_cast<float*>(smem_raw);  // 256 x dsub
  const int dsub = kD > 0 ? kD : dsub_rt;
  const int j = blockIdx.y;
  for (int i = threadIdx.x; i < kSubCentroids * dsub; i += blockDim.x)
    sc[i] = cb[static_cast<size_t>(j) * kSubCentroids * dsub + i];
  __syncthreads();
  const size_t row = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (row >= n) return;
  const float* r = resid + row * dim + static_cast<size_t>(j) * dsub;
  float rr[kD > 0 ? kD : 1];  // the residual slice, read once (compile-time widths)
  if constexpr (kD > 0) {
#pragma unroll
    for (int t = 0; t < kD; ++t) rr[t] = r[t];
  }
  // The squared distance to sub-centroid c, sequential in t, separately rounded.
  auto dist = [&](int c) {
    float s = 0.0f;
    if constexpr (kD > 0) {
#pragma unroll
      for (int t = 0; t < kD; ++t) {
        const float d = __fsub_rn(rr[t], sc[c * kD + t]);
        s = __fadd_rn(s, __fmul_rn(d, d));
      }
    } else {
      for (int t = 0; t < dsub; ++t) {
        const float d = __fsub_rn(r[t], sc[c * dsub + t]);
        s = __fadd_rn(s, __fmul_rn(d, d));
      }
    }
    return s;
  };
  // argmin_n: the minimum m (NaN never wins), then the first index holding m. A strict-< scan
  // finds that index whenever m is finite; only when m = +inf is a second pass needed.
  float best = kInf;
  int code = 0;
#pragma unroll 4
  for (int c = 0; c < kSubCentroids; ++c) {
    const float s = dist(c);
    if (s < best) {
      best = s;
      code = c;
    }
  }
  if (best == kInf) {
    for (int c = 0; c < kSubCentroids; ++c) {
      if (dist(c) == kInf) {
        code = c;
        break;
      }
    }
  }
  codes[row * m + j] = static_cast<uint8_t>(code);
}

// ---- scan ------------------------------------------------------------------------------------------

struct ScanArgs {
  const float* q;           // nq x dim (normalized for cosine)
  int dim, m, dsub;
  bool ip, use_pre;
  const float* cents;
  const float* cb;
  const float* pre;
  const uint64_t* offsets;
  const uint32_t* global_base;
  const uint8_t* codes;
  const uint64_t* labels;
  const float* vectors;
  const uint64_t* bitmap;   // positions
  const uint32_t* probes;   // nq x nprobe
  const float* probe_d;
  int nprobe;
  int keep, k, cap;
  bool refine;
  // outputs (final mode): labels/dists nq x k. candidate mode: dists/keys/labels nq x keep
  bool candidate_mode;
  // Inner-product metrics with at most kSeqLists probes: the probed lists are scanned as one
  // sequence (per-list data in dynamic shared memory after the survivor buffer).
  bool seq;
  uint64_t* out_labels;
  float* out_d;
  uint64_t* out_keys;
};

// When the buffer holds more than 2 x keep entries (and at most 4 per thread), the keep-th
// smallest distance t is found first by a radix select over the distances' ordered bits (-0
// counted as +0, as the (distance, key) order treats them), and only the entries at or below t
// (keep of them plus ties at t) are moved to the front and sorted: every entry left out has a
// larger distance than all of them, so the keep best by (distance, key) are among them.
constexpr int kSelectPerThread = 4;  // the select path serves up to this many entries per thread

__device__ __forceinline__ uint32_t select_bits(float d) { return dev::ordered_bits(d + 0.0f); }

// Returns the number of entries moved to the front of bd / bk / bp (at least keep).
__device__ int select_front(float* bd, uint64_t* bk, uint64_t* bp, int n, int keep) {
  __shared__ unsigned hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_need, s_moved;
  uint32_t prefix = 0;
  int need = keep;  // rank (1-based) of the target among the entries matching the prefix
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t above = pass == 0 ? 0u : ~0u << (shift + 8);
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t u = select_bits(bd[i]);
      if ((u & above) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      unsigned h[8], sum = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        h[b] = hist[lane * 8 + b];
        sum += h[b];
      }
      unsigned incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      unsigned cum = incl - sum;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (cum < static_cast<unsigned>(need) && static_cast<unsigned>(need) <= cum + h[b]) {
          s_prefix = prefix | (static_cast<uint32_t>(lane * 8 + b) << shift);
          s_need = need - static_cast<int>(cum);
        }
        cum += h[b];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
  }
  // prefix: the ordered bits of the keep-th smallest distance. Entries at or below it move to
  // the front, one block-wide round of blockDim entries at a time: a round writes only below the
  // count of entries selected so far, i.e. into positions already read (this round's included).
  if (threadIdx.x == 0) s_moved = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool in = i < n && select_bits(bd[i]) <= prefix;
    const float d = in ? bd[i] : 0.0f;
    const uint64_t k = in ? bk[i] : 0, p = in ? bp[i] : 0;
    __syncthreads();  // every entry of this round has been read (and s_moved set)
    if (in) {
      const int slot = atomicAdd(&s_moved, 1);
      bd[slot] = d;
      bk[slot] = k;
      bp[slot] = p;
    }
    __syncthreads();
  }
  return s_moved;
}

// Compacts the block buffer to its best `keep` (distance, key) entries; updates the threshold.
// Sorts only the filled part (or the selected front), rounded up to a power of two (at least
// `keep`'s).
__device__ void scan_compact(float* bd, uint64_t* bk, uint64_t* bp, int cap, int keep, int* cnt,
                             float* thr) {
  if (*cnt > 2 * keep && *cnt <= kSelectPerThread * static_cast<int>(blockDim.x)) {
    const int moved = select_front(bd, bk, bp, *cnt, keep);
    if (threadIdx.x == 0) *cnt = moved;
    __syncthreads();
  }
  int n2 = 1;
  while (n2 < *cnt || n2 < keep) n2 <<= 1;
  n2 = min(n2, cap);
  for (int i = *cnt + threadIdx.x; i < n2; i += blockDim.x) {
    bd[i] = kInf;
    bk[i] = ~0ull;
    bp[i] = ~0ull;
  }
  dev::block_bitonic_sort<true>(bd, bk, bp, n2);
  if (threadIdx.x == 0) {
    if (*cnt >= keep) {
      *cnt = keep;
      *thr = fminf(*thr, bd[keep - 1]);
    }
  }
  __syncthreads();
}

// Code bytes of one entry held in registers: words[i] holds bytes 4i..4i+3 of the code.
// M = 0: the code width is only known at run time; bytes are then read from global memory.
template <int M>
struct CodeWords;

template <>
struct CodeWords<0> {
  const uint8_t* p;
  __device__ __forceinline__ void load(const uint8_t* codes, uint64_t pos, int m) {
    p = codes + pos * static_cast<uint64_t>(m);
  }
  __device__ __forceinline__ uint32_t byte(int j) const { return __ldg(p + j); }
};

template <int M>
struct CodeWords {
  static constexpr int kWords = (M + 3) / 4;
  uint32_t w[kWords];
  // Loads entry `pos` of a code array with M bytes per entry (16 bytes of slack after the array).
  __device__ __forceinline__ void load(const uint8_t* codes, uint64_t pos, int /*m*/) {
    const uint64_t start = pos * M;
    if constexpr (M % 16 == 0) {
      const uint4* src = reinterpret_cast<const uint4*>(codes + start);
#pragma unroll
      for (int i = 0; i < M / 16; ++i) {
        const uint4 v = __ldg(src + i);
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
      }
    } else {
      // Aligned 4-byte loads covering [start, start + M), then a funnel shift per word.
      const uint32_t* src = reinterpret_cast<const uint32_t*>(codes + (start & ~uint64_t{3}));
      const uint32_t sh = static_cast<uint32_t>(start & 3) * 8;
      uint32_t raw[kWords + 1];
#pragma unroll
      for (int i = 0; i <= kWords; ++i) raw[i] = __ldg(src + i);
#pragma unroll
      for (int i = 0; i < kWords; ++i) w[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
    }
  }
  __device__ __forceinline__ uint32_t byte(int j) const { return (w[j >> 2] >> ((j & 3) * 8)) & 0xffu; }
};

// ADC sums of two codes at once (two independent dependency chains): each in ascending j from
// 0.0f with one rounding per addition, as ProductQuantizer::adc (src/product_quantizer.cc:188-217).
template <int M>
__device__ __forceinline__ void adc2(const float* table, const CodeWords<M>& c0,
                                     const CodeWords<M>& c1, int m, float& s0, float& s1) {
  s0 = 0.0f;
  s1 = 0.0f;
  if constexpr (M > 0) {
#pragma unroll
    for (int j = 0; j < M; ++j) {
      s0 = __fadd_rn(s0, table[j * kSubCentroids + c0.byte(j)]);
      s1 = __fadd_rn(s1, table[j * kSubCentroids + c1.byte(j)]);
    }
  } else {
    for (int j = 0; j < m; ++j) {
      s0 = __fadd_rn(s0, table[j * kSubCentroids + c0.byte(j)]);
      s1 = __fadd_rn(s1, table[j * kSubCentroids + c1.byte(j)]);
    }
  }
}

// One block per query: lookup tables in shared memory, then every probed list in probe order.
// Each thread takes two codes per pass, loaded straight from global memory into registers
// (M = code bytes, a compile-time constant), and sums their m table entries in ascending j from
// 0.0f (ProductQuantizer::adc, src/product_quantizer.cc:188-217); dist = ip ? 1-(base+s) : base+s
// (src/ivfpq_index.cc:346). Survivors of the running threshold and the position bitmap go to a
// block buffer that is compacted to the best `keep` after every pass of 2 x kScanThreads codes.
// kRegQ (code width 32, L2 with precomputed terms, several probed lists): the query term is kept
// in registers instead of shared memory (thread tid owns entries tid + i * kScanThreads, the same
// entries it adds into each list's table). It costs registers (2 resident blocks per SM instead
// of 4), which the single-list case, whose table needs no query term, does not pay.
template <int M, bool kRegQ = false>
__global__ void __launch_bounds__(kScanThreads, kRegQ ? 3 : (M <= 32 ? 4 : 2))
    ivf_scan_kernel(ScanArgs a) {
  static_assert(!kRegQ || M > 0, "the register query term needs a compile-time code width");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int ts = (M > 0 ? M : a.m) * kSubCentroids;
  // One probed list with the L2 precomputed terms: the query term goes straight into that list's
  // table (the same rounded sum pre + (-2 * ip)), so no separate query table is kept.
  const bool fused = a.use_pre && !a.ip && a.nprobe == 1;
  float qreg[kRegQ ? M : 1];
  float* table = reinterpret_cast<float*>(smem_raw);
  float* qtab = table + ts;                                // L2 precomputed, in shared memory
  float* qv = qtab + (a.use_pre && !fused && !kRegQ ? ts : 0);  // dim (residual scratch for L2)
  float* bd = qv + ((a.dim + 3) & ~3);
  uint64_t* bk = reinterpret_cast<uint64_t*>(bd + a.cap);
  uint64_t* bp = bk + a.cap;
  // seq: per probed list its first index in the sequence (nprobe + 1 entries), first code
  // position, list id, global base and coarse term.
  int64_t* s_start = reinterpret_cast<int64_t*>(bp + a.cap);
  uint64_t* s_off = reinterpret_cast<uint64_t*>(s_start + a.nprobe + 1);
  uint32_t* s_list = reinterpret_cast<uint32_t*>(s_off + a.nprobe);
  uint32_t* s_gb = s_list + a.nprobe;
  float* s_base = reinterpret_cast<float*>(s_gb + a.nprobe);
  __shared__ int s_cnt;
  __shared__ float s_thr;

  const size_t q = blockIdx.x;
  const float* qrow = a.q + q * a.dim;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_cnt = 0;
    s_thr = kInf;
  }
  for (int i = tid; i < a.dim; i += blockDim.x) qv[i] = qrow[i];
  __syncthreads();
  // Query-side tables: ip_table (CentroidTable::dot over each sub-space, sequential in t).
  if (a.ip || a.use_pre) {
    float* dst = (a.ip || fused) ? table : qtab;
    const float* pre0 = fused ? a.pre + static_cast<size_t>(a.probes[q]) * ts : nullptr;
    if (a.dsub == 4) {
      // Sub-spaces of 4 (configs 2 and 3): one 16-byte load per entry, the loop unrolled so that
      // many entries' loads are in flight per thread (the codebook is read from L2 by every
      // query).
#pragma unroll
      for (int i = 0; i < (M > 0 ? M : ts / kScanThreads + 1); ++i) {
        const int e = tid + i * kScanThreads;
        if (M == 0 && e >= ts) break;
        const float4 c = __ldg(reinterpret_cast<const float4*>(a.cb) + e);
        const float* qs = qv + (e / kSubCentroids) * 4;
        float acc = __fadd_rn(0.0f, __fmul_rn(qs[0], c.x));
        acc = __fadd_rn(acc, __fmul_rn(qs[1], c.y));
        acc = __fadd_rn(acc, __fmul_rn(qs[2], c.z));
        acc = __fadd_rn(acc, __fmul_rn(qs[3], c.w));
        // query_table = -2 * ip_table (:316-317); fused: its list's table entry pre + that
        const float v = a.ip ? acc : __fmul_rn(acc, -2.0f);
        if constexpr (kRegQ) {
          if (!a.ip && !fused) {
            qreg[i] = v;
            continue;
          }
        }
        dst[e] = fused ? __fadd_rn(__ldg(pre0 + e), v) : v;
      }
    } else {
#pragma unroll
      for (int i = 0; i < (M > 0 ? M : ts / kScanThreads + 1); ++i) {
        const int e = tid + i * kScanThreads;
        if (M == 0 && e >= ts) break;
        const int j = e / kSubCentroids;
        const float* cbv = a.cb + static_cast<size_t>(e) * a.dsub;
        const float* qs = qv + j * a.dsub;
        float acc = 0.0f;
        for (int t = 0; t < a.dsub; ++t) acc = __fadd_rn(acc, __fmul_rn(qs[t], cbv[t]));
        const float v = a.ip ? acc : __fmul_rn(acc, -2.0f);
        if constexpr (kRegQ) {
          if (!a.ip && !fused) {
            qreg[i] = v;
            continue;
          }
        }
        dst[e] = fused ? __fadd_rn(__ldg(pre0 + e), v) : v;
      }
    }
  }
  __syncthreads();

  float thr = kInf;
  // With the L2 precomputed terms and a compile-time code width, each thread keeps its M
  // entries of the next probed list's precomputed slice in registers: they are loaded while the
  // current list is scanned and only added to the query's table after it. (kRegQ instead holds
  // the query term there and loads each slice when it builds the table: 3 blocks per SM.)
  constexpr bool kPrefetch = M > 0 && !kRegQ;
  float pf[kPrefetch ? M : 1];
  auto prefetch = [&](int pi) {
    if constexpr (kPrefetch) {
      const uint32_t l = a.probes[q * a.nprobe + pi];
      const float* pre = a.pre + static_cast<size_t>(l) * ts;
#pragma unroll
      for (int i = 0; i < M; ++i) pf[i] = __ldg(pre + tid + i * kScanThreads);
    }
  };
  if (a.use_pre && !a.ip && !fused) prefetch(0);
  if (a.seq) {
    // Inner product: one table serves every list (only the coarse term differs), so the lists'
    // codes form one sequence and a pass of 2 x kScanThreads codes may span list boundaries
    // instead of ending with each list. Each code's arithmetic, key and position are the ones
    // the per-list loop below gives it.
    for (int pi = tid; pi < a.nprobe; pi += blockDim.x) {
      const uint32_t l = a.probes[q * a.nprobe + pi];
      s_list[pi] = l;
      s_off[pi] = a.offsets[l];
      s_gb[pi] = a.global_base[l];
      s_base[pi] = -a.probe_d[q * a.nprobe + pi];
    }
    __syncthreads();
    if (tid == 0) {
      int64_t acc = 0;
      for (int pi = 0; pi < a.nprobe; ++pi) {
        s_start[pi] = acc;
        acc += static_cast<int64_t>(a.offsets[s_list[pi] + 1] - s_off[pi]);
      }
      s_start[a.nprobe] = acc;
    }
    __syncthreads();
    const int64_t total = s_start[a.nprobe];
    int cur[2] = {0, 0};  // the list holding this thread's next code of each half
    for (int64_t r0 = 0; r0 < total; r0 += 2 * kScanThreads) {
      int64_t g[2];
      bool v[2];
      uint64_t pos[2];
      CodeWords<M> c[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        g[h] = r0 + h * kScanThreads + tid;
        v[h] = g[h] < total;
        while (v[h] && s_start[cur[h] + 1] <= g[h]) ++cur[h];
        pos[h] = v[h] ? s_off[cur[h]] + static_cast<uint64_t>(g[h] - s_start[cur[h]]) : 0;
        c[h].load(a.codes, pos[h], a.m);
      }
      float sum[2];
      adc2<M>(table, c[0], c[1], a.m, sum[0], sum[1]);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int pi = cur[h];
        float dist = __fsub_rn(1.0f, __fadd_rn(s_base[pi], sum[h]));
        dist = dev::nan_to_inf(dist);
        if (v[h] && dist <= thr && dev::bitmap_test(a.bitmap, pos[h])) {
          const uint64_t i = pos[h] - s_off[pi];
          const int slot = atomicAdd(&s_cnt, 1);
          bd[slot] = dist;
          bk[slot] = (static_cast<uint64_t>(s_list[pi]) << 32) | (s_gb[pi] + i);
          bp[slot] = pos[h];
        }
      }
      __syncthreads();
      const int filled = s_cnt;
      __syncthreads();
      if (filled > a.cap - 2 * kScanThreads || (thr == kInf && filled >= 8 * a.keep))
        scan_compact(bd, bk, bp, a.cap, a.keep, &s_cnt, &s_thr);
      thr = s_thr;
    }
  }
  for (int pi = 0; pi < (a.seq ? 0 : a.nprobe); ++pi) {
    const uint32_t l = a.probes[q * a.nprobe + pi];
    const uint64_t off = a.offsets[l];
    const int64_t len = static_cast<int64_t>(a.offsets[l + 1] - off);
    if (len == 0) {
      if (kPrefetch && a.use_pre && !a.ip && pi + 1 < a.nprobe) prefetch(pi + 1);
      continue;
    }
    float base;
    if (a.ip) {
      base = -a.probe_d[q * a.nprobe + pi];
    } else if (fused) {
      base = a.probe_d[q];  // the table was built with the query term
    } else if (a.use_pre) {
      base = a.probe_d[q * a.nprobe + pi];
      __syncthreads();
      if constexpr (kPrefetch) {
#pragma unroll
        for (int i = 0; i < M; ++i) {
          const int e = tid + i * kScanThreads;
          table[e] = __fadd_rn(pf[i], qtab[e]);
        }
      } else if constexpr (kRegQ) {
        const float* pre = a.pre + static_cast<size_t>(l) * ts;
#pragma unroll
        for (int i = 0; i < M; ++i) {
          const int e = tid + i * kScanThreads;
          table[e] = __fadd_rn(__ldg(pre + e), qreg[i]);
        }
      } else {
        const float* pre = a.pre + static_cast<size_t>(l) * ts;
        for (int e = tid; e < ts; e += blockDim.x) table[e] = __fadd_rn(__ldg(pre + e), qtab[e]);
      }
      __syncthreads();
      if (pi + 1 < a.nprobe) prefetch(pi + 1);
    } else {
      // Residual L2 table (src/ivfpq_index.cc:339-341 with compute_l2_table).
      base = 0.0f;
      const float* c = a.cents + static_cast<size_t>(l) * a.dim;
      __syncthreads();
      for (int e = tid; e < ts; e += blockDim.x) {
        const int j = e / kSubCentroids;
        const float* cbv = a.cb + static_cast<size_t>(e) * a.dsub;
        float acc = 0.0f;
        for (int t = 0; t < a.dsub; ++t) {
          const int col = j * a.dsub + t;
          const float r = __fsub_rn(qv[col], c[col]);
          const float d = __fsub_rn(r, cbv[t]);
          acc = __fadd_rn(acc, __fmul_rn(d, d));
        }
        table[e] = acc;
      }
      __syncthreads();
    }
    const uint64_t gbase = static_cast<uint64_t>(a.global_base[l]);
    for (int64_t r0 = 0; r0 < len; r0 += 2 * kScanThreads) {
      const int64_t i0 = r0 + tid, i1 = r0 + kScanThreads + tid;
      const bool v0 = i0 < len, v1 = i1 < len;
      CodeWords<M> c0, c1;
      c0.load(a.codes, off + (v0 ? i0 : 0), a.m);
      c1.load(a.codes, off + (v1 ? i1 : 0), a.m);
      float s0, s1;
      adc2<M>(table, c0, c1, a.m, s0, s1);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const bool valid = h == 0 ? v0 : v1;
        const int64_t i = h == 0 ? i0 : i1;
        const float sum = h == 0 ? s0 : s1;
        float dist = a.ip ? __fsub_rn(1.0f, __fadd_rn(base, sum)) : __fadd_rn(base, sum);
        dist = dev::nan_to_inf(dist);
        const uint64_t pos = off + static_cast<uint64_t>(i);
        if (valid && dist <= thr && dev::bitmap_test(a.bitmap, pos)) {
          const int slot = atomicAdd(&s_cnt, 1);
          bd[slot] = dist;
          bk[slot] = (static_cast<uint64_t>(l) << 32) | (gbase + static_cast<uint64_t>(i));
          bp[slot] = pos;
        }
      }
      // Every thread reads the count between two barriers, so no thread appends for the next
      // pass before all have decided (together) whether to compact. The first compaction comes
      // as soon as 8 x `keep` entries are held (the keep-th best of those is already a useful
      // threshold), which gives small-keep scans a finite threshold after their first pass.
      __syncthreads();
      const int filled = s_cnt;
      __syncthreads();
      if (filled > a.cap - 2 * kScanThreads || (thr == kInf && filled >= 8 * a.keep))
        scan_compact(bd, bk, bp, a.cap, a.keep, &s_cnt, &s_thr);
      thr = s_thr;
    }
  }
  __syncthreads();
  scan_compact(bd, bk, bp, a.cap, a.keep, &s_cnt, &s_thr);
  const int n = min(s_cnt, a.keep);
  if (a.candidate_mode) {
    for (int j = tid; j < a.keep; j += blockDim.x) {
      const size_t o = q * a.keep + j;
      a.out_d[o] = j < n ? bd[j] : kInf;
      a.out_keys[o] = j < n ? bk[j] : ~0ull;
      a.out_labels[o] = j < n ? a.labels[bp[j]] : kInvalidLabel;
    }
    return;
  }
  int nres = n;
  if (a.refine && n > 0) {
    // Exact re-rank (src/ivfpq_index.cc:362-373), one warp per candidate.
    const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    for (int i = warp; i < n; i += nwarps) {
      const float e = dev::nan_to_inf(
          dev::warp_exact_distance(qv, a.vectors + bp[i] * a.dim, a.dim, !a.ip, lane));
      if (lane == 0) bd[i] = e;
    }
    __syncthreads();
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = n + tid; i < np2; i += blockDim.x) {
      bd[i] = kInf;
      bk[i] = ~0ull;
      bp[i] = ~0ull;
    }
    dev::block_bitonic_sort<true>(bd, bk, bp, np2);
  }
  nres = min(nres, a.k);
  for (int j = tid; j < a.k; j += blockDim.x) {
    const size_t o = q * a.k + j;
    a.out_d[o] = j < nres ? bd[j] : kInf;
    a.out_labels[o] = j < nres ? a.labels[bp[j]] : kInvalidLabel;
  }
}

// Exact distance of each candidate this shard stores, +inf for the others.
__global__ void ivf_refine_kernel(const float* __restrict__ qn, size_t nq, int dim, int keep,
                                  const uint64_t* __restrict__ keys, const uint64_t* offsets,
                                  const uint32_t* global_base, size_t nlist, const float* vectors,
                                  bool l2, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const size_t w = blockIdx.x * static_cast<size_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= nq * keep) return;
  const size_t q = w / keep;
  const uint64_t key = keys[w];
  float e = kInf;
  if (key != ~0ull) {
    const uint64_t l = key >> 32;
    const uint64_t g = key & 0xffffffffull;
    if (l < nlist) {
      const uint64_t b = global_base[l];
      const uint64_t len = offsets[l + 1] - offsets[l];
      if (g >= b && g - b < len) {
        const uint64_t pos = offsets[l] + (g - b);
        e = dev::nan_to_inf(dev::warp_exact_distance(qn + q * dim, vectors + pos * dim, dim, l2, lane));
      }
    }
  }
  if (lane == 0) out[w] = e;
}

// Total length of the probed lists over all (query, probe) pairs: the number of codes a scan
// reads, for the timing statistics' algorithmic bytes.
__global__ void probed_codes_kernel(const uint32_t* __restrict__ probes, size_t total,
                                    const uint64_t* __restrict__ offsets,
                                    unsigned long long* __restrict__ out) {
  unsigned long long acc = 0;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t l = probes[i];
    acc += offsets[l + 1] - offsets[l];
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0 && acc != 0) atomicAdd(out, acc);
}

__global__ void copy_queries_kernel(const float* q, size_t total, float* out) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = q[i];
}

struct Prepared {
  DeviceBuffer qn, coarse, probes, probe_d;
  int nprobe = 1;
};

// Centroid tables: k centroids (device rows) as Flat rows labelled 0..k-1, scored with
// CentroidTable's arithmetic, so that an exact Flat search of a table (tensor-core screen, exact
// re-rank in that arithmetic, certificate) returns what CentroidTable's full scan returns:
//   kProbeL2  sum_j (q_j - c_j)^2, sequential (CentroidTable::l2: the L2 coarse probe);
//   kNegIp    -(sum_j q_j c_j), sequential (CentroidTable::dot: the IP and cosine probes, and the
//             inner-product assignment);
//   kAssignL2 ||c||^2 - 2<x,c>, both sequential (CentroidTable::nearest_batch: the L2 and cosine
//             assignment), its screens leaving out the constant ||x||^2.
enum class TableKind { kProbeL2, kNegIp, kAssignL2 };
std::unique_ptr<FlatState> centroid_table(const float* d_cents, size_t k, size_t dim, int device,
                                          TableKind kind, cudaStream_t st) {
  auto t = std::make_unique<FlatState>();
  t->device = device;
  t->dim = dim;
  t->metric = kind == TableKind::kNegIp ? QV_METRIC_IP : QV_METRIC_L2;
  t->sum_order = kind == TableKind::kAssignL2 ? kSumOrderNormDot : kSumOrderSeq;
  t->neg_ip = kind == TableKind::kNegIp;
  t->drop_qnorm = kind == TableKind::kAssignL2;
  DeviceBuffer ids(k * sizeof(uint64_t), st);
  sequential_labels(ids.get<uint64_t>(), k, 0, st);
  flat_append(*t, d_cents, ids.get<uint64_t>(), k, st, /*normalize=*/false);  // waits on st
  return t;
}

// Probe lists from a centroid table's Flat search: labels are list ids. A query without results
// (one holding NaN or infinity, which the host entry points reject before searching) gets lists
// 0..k-1, as the selection over its all-NaN distances would.
__global__ void probes_from_labels_kernel(const uint64_t* __restrict__ labels, size_t total,
                                          int k, size_t nlist, uint32_t* __restrict__ probes) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t l = labels[i];
    probes[i] = static_cast<uint32_t>(l < nlist ? l : i % static_cast<size_t>(k));
  }
}

// A centroid table is searched on the tensor cores where that screen applies and k stays within
// its narrow best lists; QV_IVF_COARSE=simt keeps the float32 CUDA-core kernels (distance table
// plus radix selection for the probe, the register-tiled scan for the assignment) everywhere.
// Both give the same lists and distances: the same sums, ordered by (distance, list id).
constexpr size_t kTableMaxK = 24;
constexpr size_t kTableMinRows = 128;
bool table_on_tensor_cores(const FlatState* t, size_t k) {
  if (t == nullptr || t->n < kTableMinRows || k > kTableMaxK) return false;
  const char* e = std::getenv("QV_IVF_COARSE");
  if (e != nullptr && std::strcmp(e, "simt") == 0) return false;
  return flat_tc_eligible(*t, k) && !flat_tc_is_wide(*t, k);
}

// The k nearest table rows of n device rows: ids (n x k, u32) and, when d_dist is not null, their
// distances.
void table_nearest(const FlatState& t, const float* d_x, size_t n, size_t k, uint32_t* d_ids,
                   float* d_dist, cudaStream_t st) {
  const size_t total = n * k;
  DeviceBuffer labels(total * sizeof(uint64_t), st);
  DeviceBuffer dist(d_dist == nullptr ? total * sizeof(float) : 0, st);
  DeviceBuffer flags(kSearchFlagWords * sizeof(int), st);
  QV_CUDA(cudaMemsetAsync(flags.get(), 0, kSearchFlagWords * sizeof(int), st));
  flat_search(t, d_x, n, k, nullptr, labels.get<uint64_t>(),
              d_dist != nullptr ? d_dist : dist.get<float>(), nullptr, flags.get<int>(), st);
  probes_from_labels_kernel<<<static_cast<unsigned>(std::min<size_t>(ceil_div(total, 256), 4096)),
                              256, 0, st>>>(labels.get<uint64_t>(), total, static_cast<int>(k),
                                            t.n, d_ids);
  check_launch("probes_from_labels_kernel");
}

Prepared prepare_search(const IvfState& s, const float* d_queries, size_t nq, size_t nprobe,
                        cudaStream_t st) {
  Prepared p;
  p.nprobe = static_cast<int>(std::min(std::max<size_t>(nprobe, 1), s.nlist));  // :286
  p.qn.allocate(nq * s.dim * sizeof(float), st);
  copy_queries_kernel<<<std::min<size_t>(ceil_div(nq * s.dim, 256), 4096), 256, 0, st>>>(
      d_queries, nq * s.dim, p.qn.get<float>());
  check_launch("copy_queries_kernel");
  if (s.metric == QV_METRIC_COSINE) normalize_rows_device(p.qn.get<float>(), nq, s.dim, st);
  p.probes.allocate(nq * p.nprobe * sizeof(uint32_t), st);
  p.probe_d.allocate(nq * p.nprobe * sizeof(float), st);
  if (table_on_tensor_cores(s.coarse_table.get(), static_cast<size_t>(p.nprobe))) {
    table_nearest(*s.coarse_table, p.qn.get<float>(), nq, static_cast<size_t>(p.nprobe),
                  p.probes.get<uint32_t>(), p.probe_d.get<float>(), st);
    return p;
  }
  p.coarse.allocate(nq * s.nlist * sizeof(float), st);
  dim3 grid(static_cast<unsigned>(ceil_div(nq, kTileP4)),
            static_cast<unsigned>(ceil_div(s.nlist, kTileC4)));
  coarse_dist_kernel4<<<grid, 256, 0, st>>>(p.qn.get<float>(), nq, s.centroids.get<float>(),
                                            s.nlist, static_cast<int>(s.dim), s.ip(),
                                            p.coarse.get<float>());
  check_launch("coarse_dist_kernel4");
  const int pool = static_cast<int>(next_pow2(s.nlist));
  if (p.nprobe <= kRadixProbeMax) {
    int id_passes = 1;
    while (id_passes < 4 && (s.nlist - 1) >> (8 * id_passes) != 0) ++id_passes;
    const int sort_n = static_cast<int>(next_pow2(static_cast<size_t>(p.nprobe)));
    const bool shared = s.nlist * sizeof(uint64_t) <= kRadixSharedMax;
    const size_t smem = (sort_n + (shared ? s.nlist : 0)) * sizeof(uint64_t);
    auto kernel = shared ? select_probes_radix_kernel<true> : select_probes_radix_kernel<false>;
    QV_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kernel<<<static_cast<unsigned>(nq), kRadixThreads, smem, st>>>(
        p.coarse.get<float>(), s.nlist, p.nprobe, id_passes, sort_n, p.probes.get<uint32_t>(),
        p.probe_d.get<float>());
    check_launch("select_probes_radix_kernel");
    return p;
  }
  const size_t smem = pool * (sizeof(float) + sizeof(uint64_t));
  QV_REQUIRE(smem <= 227 * 1024, "IVF-PQ search: nprobe above 1024 needs nlist <= 16384");
  QV_CUDA(cudaFuncSetAttribute(select_probes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  select_probes_kernel<<<static_cast<unsigned>(nq), 512, smem, st>>>(
      p.coarse.get<float>(), s.nlist, pool, p.nprobe, p.probes.get<uint32_t>(),
      p.probe_d.get<float>());
  check_launch("select_probes_kernel");
  return p;
}

void run_scan(const IvfState& s, const Prepared& p, size_t nq, size_t keep, size_t k, bool refine,
              const uint64_t* d_bitmap, bool candidate_mode, uint64_t* out_labels, float* out_d,
              uint64_t* out_keys, cudaStream_t st) {
  ScanArgs a{};
  a.q = p.qn.get<float>();
  a.dim = static_cast<int>(s.dim);
  a.m = static_cast<int>(s.m);
  a.dsub = static_cast<int>(s.dsub);
  a.ip = s.ip();
  a.use_pre = !s.ip() && s.use_precomputed();
  a.cents = s.centroids.get<float>();
  a.cb = s.codebooks.get<float>();
  a.pre = s.precomputed.get<float>();
  a.offsets = s.offsets.get<uint64_t>();
  a.global_base = s.global_base.get<uint32_t>();
  a.codes = s.codes.get<uint8_t>();
  a.labels = s.labels.get<uint64_t>();
  a.vectors = s.vectors.get<float>();
  a.bitmap = d_bitmap;
  a.probes = p.probes.get<uint32_t>();
  a.probe_d = p.probe_d.get<float>();
  a.nprobe = p.nprobe;
  a.keep = static_cast<int>(keep);
  a.k = static_cast<int>(k);
  a.cap = static_cast<int>(std::max<size_t>(1024, next_pow2(keep + 2 * kScanThreads)));
  a.refine = refine;
  a.candidate_mode = candidate_mode;
  a.seq = a.ip && p.nprobe <= kSeqLists;
  a.out_labels = out_labels;
  a.out_d = out_d;
  a.out_keys = out_keys;
  const size_t ts = s.m * kSubCentroids * sizeof(float);
  const bool fused = a.use_pre && p.nprobe == 1;  // no separate query table (see the kernel)
  // Several probed lists with the precomputed terms and code width 32: the query term in registers.
  const bool reg_q = s.m == 32 && a.use_pre && !fused;
  const size_t seq_bytes =
      a.seq ? (p.nprobe + 1) * sizeof(int64_t) + p.nprobe * (sizeof(uint64_t) + 3 * sizeof(uint32_t))
            : 0;
  const size_t smem = ts * (a.use_pre && !fused && !reg_q ? 2 : 1) +
                      ((s.dim + 3) & ~size_t{3}) * sizeof(float) +
                      a.cap * (sizeof(float) + 2 * sizeof(uint64_t)) + seq_bytes;
  if (smem > 227 * 1024) {
    fail(QV_ERR_UNSUPPORTED,
         "IVF-PQ search: m=" + std::to_string(s.m) + " with keep=" + std::to_string(keep) +
             " needs " + std::to_string(smem) + " bytes of shared memory per query (max 232448)");
  }
  // Code widths with a specialized kernel (codes held in registers); others read code bytes from
  // global memory.
  void (*kernel)(ScanArgs) = ivf_scan_kernel<0>;
  switch (s.m) {
    case 8: kernel = ivf_scan_kernel<8>; break;
    case 10: kernel = ivf_scan_kernel<10>; break;
    case 16: kernel = ivf_scan_kernel<16>; break;
    case 25: kernel = ivf_scan_kernel<25>; break;
    case 32: kernel = reg_q ? ivf_scan_kernel<32, true> : ivf_scan_kernel<32>; break;
    case 48: kernel = ivf_scan_kernel<48>; break;
    case 64: kernel = ivf_scan_kernel<64>; break;
    default: break;
  }
  QV_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // With timing on: the scan's algorithmic bytes are the codes of the probed lists (m bytes
  // each), the lookup-table source per probe (the precomputed slice for L2 with precomputed
  // terms; the codebooks once per query otherwise), the query, and the stored vectors the
  // refine gathers.
  const double lut = static_cast<double>(ts) * (a.use_pre ? p.nprobe : 1);
  const double per_query = lut + s.dim * sizeof(float) +
                           (refine ? static_cast<double>(keep) * s.dim * sizeof(float) : 0.0);
  unsigned long long* slot = nullptr;
  if (thread_timing()) {
    // The codes of the probed lists are counted on the device and copied to a pinned slot that
    // is read when the timer is resolved; the search itself does not wait.
    DeviceBuffer codes_read(sizeof(unsigned long long), st);
    QV_CUDA(cudaMemsetAsync(codes_read.get(), 0, sizeof(unsigned long long), st));
    const size_t pairs = nq * static_cast<size_t>(p.nprobe);
    probed_codes_kernel<<<static_cast<unsigned>(std::min<size_t>(ceil_div(pairs, 256), 1024)), 256,
                          0, st>>>(p.probes.get<uint32_t>(), pairs, a.offsets,
                                   codes_read.get<unsigned long long>());
    check_launch("probed_codes_kernel");
    slot = timing_count_slot();
    QV_CUDA(cudaMemcpyAsync(slot, codes_read.get(), sizeof(*slot), cudaMemcpyDeviceToHost, st));
  }
  KernelTimer timer(st, "ivf_scan_kernel", per_query * static_cast<double>(nq), true);
  if (slot != nullptr) timer.set_device_count(slot, static_cast<double>(s.m));
  kernel<<<static_cast<unsigned>(nq), kScanThreads, smem, st>>>(a);
  timer.stop();
  check_launch("ivf_scan_kernel");
}

}  // namespace

// ---- host entry points ---------------------------------------------------------------------------------

void ivf_set_trained(IvfState& s, const float* h_centroids, const float* h_codebooks,
                     cudaStream_t st) {
  const size_t cn = s.nlist * s.dim, bn = s.m * kSubCentroids * s.dsub;
  s.host_centroids.assign(h_centroids, h_centroids + cn);
  s.host_codebooks.assign(h_codebooks, h_codebooks + bn);
  s.centroids.allocate(cn * sizeof(float));
  s.codebooks.allocate(bn * sizeof(float));
  s.cnorm2.allocate(s.nlist * sizeof(float));
  QV_CUDA(cudaMemcpyAsync(s.centroids.get(), h_centroids, cn * sizeof(float),
                          cudaMemcpyHostToDevice, st));
  QV_CUDA(cudaMemcpyAsync(s.codebooks.get(), h_codebooks, bn * sizeof(float),
                          cudaMemcpyHostToDevice, st));
  centroid_norms_kernel<<<ceil_div(s.nlist, 256), 256, 0, st>>>(
      s.centroids.get<float>(), s.nlist, static_cast<int>(s.dim), s.cnorm2.get<float>());
  check_launch("centroid_norms_kernel");
  s.precomputed.release();
  const size_t pre_bytes = s.nlist * s.m * kSubCentroids * sizeof(float);
  if (!s.ip() && pre_bytes <= kMaxPrecomputedBytes) {  // src/ivfpq_index.cc:114
    s.precomputed.allocate(pre_bytes);
    const size_t total = s.nlist * s.m * kSubCentroids;
    precompute_kernel<<<ceil_div(total, 256), 256, 0, st>>>(
        s.centroids.get<float>(), s.nlist, s.codebooks.get<float>(), static_cast<int>(s.m),
        static_cast<int>(s.dsub), s.precomputed.get<float>());
    check_launch("precompute_kernel");
  }
  // The centroid tables of the coarse probe and of add()'s assignment.
  s.coarse_table = centroid_table(s.centroids.get<float>(), s.nlist, s.dim, s.device,
                                  s.ip() ? TableKind::kNegIp : TableKind::kProbeL2, st);
  s.l2_assign_table.reset();
  if (s.metric != QV_METRIC_IP)
    s.l2_assign_table = centroid_table(s.centroids.get<float>(), s.nlist, s.dim, s.device,
                                       TableKind::kAssignL2, st);
  QV_CUDA(cudaStreamSynchronize(st));
  s.trained = true;
}

void nearest_centroids_device(const float* d_x, size_t n, const float* d_cents, size_t k,
                              size_t dim, bool by_ip, float* d_cnorm2, uint32_t* d_assign,
                              cudaStream_t st) {
  if (n == 0) return;
  if (k >= kTableMinRows) {
    int device = 0;
    QV_CUDA(cudaGetDevice(&device));
    const std::unique_ptr<FlatState> t = centroid_table(
        d_cents, k, dim, device, by_ip ? TableKind::kNegIp : TableKind::kAssignL2, st);
    if (table_on_tensor_cores(t.get(), 1)) {
      table_nearest(*t, d_x, n, 1, d_assign, nullptr, st);
      return;
    }
  }
  centroid_norms_kernel<<<ceil_div(k, 256), 256, 0, st>>>(d_cents, k, static_cast<int>(dim),
                                                          d_cnorm2);
  check_launch("centroid_norms_kernel");
  coarse_assign_kernel4<<<ceil_div(n, kTileP4), 256, 0, st>>>(d_x, n, d_cents, d_cnorm2, k,
                                                              static_cast<int>(dim), by_ip,
                                                              d_assign);
  check_launch("coarse_assign_kernel4");
}

void ivf_encode_device(const IvfState& s, const float* d_x, size_t n, uint32_t* d_assign,
                       uint8_t* d_codes, cudaStream_t st) {
  if (n == 0) return;
  // assign_by_ip for the inner-product metric (src/ivfpq_index.cc:107)
  if (table_on_tensor_cores(s.assign_table(), 1)) {
    table_nearest(*s.assign_table(), d_x, n, 1, d_assign, nullptr, st);
  } else {
    coarse_assign_kernel4<<<ceil_div(n, kTileP4), 256, 0, st>>>(
        d_x, n, s.centroids.get<float>(), s.cnorm2.get<float>(), s.nlist,
        static_cast<int>(s.dim), s.metric == QV_METRIC_IP, d_assign);
    check_launch("coarse_assign_kernel4");
  }
  DeviceBuffer resid(n * s.dim * sizeof(float), st);
  residual_kernel<<<ceil_div(n * s.dim, 256), 256, 0, st>>>(
      d_x, n, static_cast<int>(s.dim), s.centroids.get<float>(), d_assign, resid.get<float>());
  check_launch("residual_kernel");
  const size_t smem = kSubCentroids * s.dsub * sizeof(float);
  QV_REQUIRE(smem <= 227 * 1024, "PQ sub-space too wide for the GPU encoder");
  void (*encode)(const float*, size_t, int, int, int, const float*, uint8_t*) =
      pq_encode_kernel<0>;
  switch (s.dsub) {
    case 1: encode = pq_encode_kernel<1>; break;
    case 2: encode = pq_encode_kernel<2>; break;
    case 4: encode = pq_encode_kernel<4>; break;
    case 8: encode = pq_encode_kernel<8>; break;
    case 16: encode = pq_encode_kernel<16>; break;
    default: break;
  }
  QV_CUDA(cudaFuncSetAttribute(encode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(static_cast<unsigned>(ceil_div(n, 256)), static_cast<unsigned>(s.m));
  encode<<<grid, 256, smem, st>>>(resid.get<float>(), n, static_cast<int>(s.dim),
                                  static_cast<int>(s.m), static_cast<int>(s.dsub),
                                  s.codebooks.get<float>(), d_codes);
  check_launch("pq_encode_kernel");
}

void ivf_upload_lists(IvfState& s, cudaStream_t st) {
  s.offsets.allocate((s.nlist + 1) * sizeof(uint64_t));
  s.global_base.allocate(s.nlist * sizeof(uint32_t));
  QV_CUDA(cudaMemcpyAsync(s.offsets.get(), s.host_offsets.data(), (s.nlist + 1) * sizeof(uint64_t),
                          cudaMemcpyHostToDevice, st));
  QV_CUDA(cudaMemcpyAsync(s.global_base.get(), s.host_global_base.data(),
                          s.nlist * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
  // 16 bytes of slack: the scan reads each code with aligned 4- or 16-byte loads that may extend
  // up to 15 bytes past the last code.
  s.codes.allocate(s.count * s.m + 16);
  s.labels.allocate(std::max<size_t>(1, s.count) * sizeof(uint64_t));
  if (s.count > 0) {
    QV_CUDA(cudaMemcpyAsync(s.codes.get(), s.host_codes.data(), s.count * s.m,
                            cudaMemcpyHostToDevice, st));
    QV_CUDA(cudaMemcpyAsync(s.labels.get(), s.host_labels.data(), s.count * sizeof(uint64_t),
                            cudaMemcpyHostToDevice, st));
  }
  QV_CUDA(cudaStreamSynchronize(st));
}

static size_t keep_for(size_t count, size_t k, size_t refine_factor, bool store_vectors,
                       bool* refine) {
  // src/ivfpq_index.cc:303-307, saturating.
  *refine = refine_factor > 0 && store_vectors;
  const size_t factor = *refine ? refine_factor : 1;
  const size_t kk = std::max<size_t>(k, 1);
  return std::min(count, factor > count / kk ? count : k * factor);
}

void ivf_search(const IvfState& s, const float* d_queries, size_t nq, size_t k, size_t nprobe,
                size_t refine_factor, const uint64_t* d_bitmap, uint64_t* d_labels,
                float* d_dists, cudaStream_t st) {
  if (nq == 0 || k == 0) return;
  bool refine = false;
  const size_t keep = keep_for(s.count, k, refine_factor, s.store_vectors, &refine);
  if (keep == 0 || !s.trained) {  // src/ivfpq_index.cc:277-279, :308
    std::vector<float> inf(nq * k, INFINITY);
    std::vector<uint64_t> inv(nq * k, kInvalidLabel);
    QV_CUDA(cudaMemcpyAsync(d_dists, inf.data(), nq * k * sizeof(float), cudaMemcpyHostToDevice, st));
    QV_CUDA(cudaMemcpyAsync(d_labels, inv.data(), nq * k * sizeof(uint64_t), cudaMemcpyHostToDevice, st));
    QV_CUDA(cudaStreamSynchronize(st));
    return;
  }
  QV_REQUIRE(keep <= 3840, "IVF-PQ search: k * refine_factor above 3840 candidates per query is "
                           "not supported on the GPU");
  Prepared p = prepare_search(s, d_queries, nq, nprobe, st);
  run_scan(s, p, nq, keep, k, refine, d_bitmap, false, d_labels, d_dists, nullptr, st);
}

void ivf_candidates(const IvfState& s, const float* d_queries, size_t nq, size_t keep,
                    size_t nprobe, const uint64_t* d_bitmap, float* d_dists, uint64_t* d_keys,
                    uint64_t* d_labels, cudaStream_t st) {
  if (nq == 0 || keep == 0) return;
  QV_REQUIRE(s.trained, "IVF-PQ index must be trained before search");
  QV_REQUIRE(keep <= 3840, "IVF-PQ candidates: keep above 3840 is not supported on the GPU");
  Prepared p = prepare_search(s, d_queries, nq, nprobe, st);
  run_scan(s, p, nq, keep, keep, false, d_bitmap, true, d_labels, d_dists, d_keys, st);
}

void ivf_refine(const IvfState& s, const float* d_queries, size_t nq, size_t keep,
                const uint64_t* d_keys, float* d_exact, cudaStream_t st) {
  if (nq == 0 || keep == 0) return;
  QV_REQUIRE(s.store_vectors, "refine needs store_vectors");
  DeviceBuffer qn(nq * s.dim * sizeof(float), st);
  copy_queries_kernel<<<std::min<size_t>(ceil_div(nq * s.dim, 256), 4096), 256, 0, st>>>(
      d_queries, nq * s.dim, qn.get<float>());
  check_launch("copy_queries_kernel");
  if (s.metric == QV_METRIC_COSINE) normalize_rows_device(qn.get<float>(), nq, s.dim, st);
  const size_t warps = nq * keep;
  ivf_refine_kernel<<<ceil_div(warps, 8), 256, 0, st>>>(
      qn.get<float>(), nq, static_cast<int>(s.dim), static_cast<int>(keep), d_keys,
      s.offsets.get<uint64_t>(), s.global_base.get<uint32_t>(), s.nlist, s.vectors.get<float>(),
      s.metric == QV_METRIC_L2, d_exact);
  check_launch("ivf_refine_kernel");
}

}  // namespace qv
