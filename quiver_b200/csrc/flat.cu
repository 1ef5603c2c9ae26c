// Exact FlatIndex search on the GPU (src/flat_index.cc:69-140 of the reference).
//
// Pipeline per batch:
//   1. prep:     copy queries into a zero-padded row-major buffer, normalizing cosine queries with
//                simd::normalize's exact arithmetic; per-query squared norm and norm for the screen.
//   2. screen:   a fast approximate pass over all rows. Each work unit is (query tile, row chunk);
//                one thread owns one query and keeps its KK best approximate candidates in a
//                private max-heap in shared memory. Units publish their KK-th value as a per-query
//                threshold that later units start from.
//   3. finalize: per query, merge the units' candidates, keep the KK best, recompute those
//                exactly in the reference's AVX2 summation order, sort by (distance, row) and emit
//                the top k. A certificate proves no other row can enter the top k: every row left
//                out has screen distance >= T (the KK-th candidate's), and |screen - exact| <= eps
//                (a rigorous float error bound), so T - eps >= D_k (the k-th exact distance)
//                suffices. Queries that fail it are listed for step 4.
//   4. rescan:   failed queries are answered by an exact scan of every row (reference arithmetic),
//                so results never depend on the screen's precision.
// Distances returned are bit-identical to the reference's; ties are broken by row id.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "qv_state.h"

namespace qv {
namespace {

using dev::kFull;

constexpr int kScreenRows = 32;   // rows per shared-memory tile of the SIMT screen
constexpr int kScreenDChunk = 256;  // columns per shared-memory tile
constexpr int kFinalizeThreads = 256;
constexpr int kMaxCandidatesPerQuery = 1024;  // n_chunks * KK, merged in one block
constexpr size_t kTcMinChunkRows = 2048;      // rows per tensor-core work unit, at least
constexpr float kInf = __builtin_huge_valf();

// ---- normalization and per-row statistics ---------------------------------------------------------

// simd::normalize (src/simd/dispatch.cc:119-135) of a row held in memory, by one warp.
__device__ void warp_normalize(float* v, int dim, int lane) {
  const float ns = dev::warp_dot_avx2(v, v, dim, lane);
  __syncwarp();
  if (!isfinite(ns)) {
    double acc = 0.0;
    if (lane == 0) {
      for (int i = 0; i < dim; ++i) {
        const double x = static_cast<double>(v[i]);
        acc = __dadd_rn(acc, __dmul_rn(x, x));
      }
    }
    acc = __shfl_sync(kFull, acc, 0);
    const double inv = (acc > 0.0 && isfinite(acc)) ? __ddiv_rn(1.0, __dsqrt_rn(acc)) : 0.0;
    if (inv == 0.0) return;
    for (int i = lane; i < dim; i += 32) v[i] = __double2float_rn(__dmul_rn(static_cast<double>(v[i]), inv));
    __syncwarp();
    return;
  }
  if (ns <= 0.0f) return;
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ns));
  for (int i = lane; i < dim; i += 32) v[i] = __fmul_rn(v[i], inv);
  __syncwarp();
}

__global__ void normalize_rows_kernel(float* x, size_t n, int dim) {
  const int lane = threadIdx.x & 31;
  const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  warp_normalize(x + row * dim, dim, lane);
}

// Squared norm of each row (screen only; any summation order) and the max row norm.
__global__ void row_stats_kernel(const float* x, size_t n, int dim, float* norm2,
                                 unsigned* max_norm_bits) {
  const int lane = threadIdx.x & 31;
  const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  const float* v = x + row * dim;
  float s = 0.0f;
  for (int i = lane; i < dim; i += 32) s = fmaf(v[i], v[i], s);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (lane == 0) {
    norm2[row] = s;
    atomicMax(max_norm_bits, __float_as_uint(sqrtf(s) * 1.0001f));
  }
}

// Error model of the float32 SIMT screen against the reference's float32 result: both sums carry
// at most gamma_d = d*u/(1-d*u) relative error of sum|q_i x_i| <= ||q|| ||x|| (u = 2^-24), plus the
// rounding of the final 1 - dot or norm combination; doubled for margin.
struct EpsModel {
  float c_l2;   // multiplies (||q|| + max||x||)^2
  float c_ip;   // multiplies ||q|| * max||x||
  float c_abs;  // multiplies (1 + ||q|| * max||x||)
};

// Queries -> zero-padded rows (dpad columns), normalized for cosine; squared norm, and the SIMT
// screen's error bound eps[q] (the tensor-core screen overwrites eps with its own bound).
// A query holding NaN or infinity is marked in qbad[q] and counted in *nonfinite: the reference
// rejects such queries (src/flat_index.cc:131). Checking here, where the queries are read anyway,
// keeps the host from scanning the batch before each search; the finalize gives such a query
// no results (QV_INVALID_LABEL with a NaN distance) and the host-buffer entry point raises.
__global__ void prep_queries_kernel(const float* q, size_t nq, int dim, int dpad, bool cosine,
                                    bool l2, bool drop_qnorm, EpsModel em, float xmax, float* qp,
                                    float* qnorm2, float* eps, int* qbad, int* nonfinite) {
  const int lane = threadIdx.x & 31;
  const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= nq) return;
  float* out = qp + row * dpad;
  bool bad = false;
  for (int i = lane; i < dpad; i += 32) {
    const float v = i < dim ? q[row * dim + i] : 0.0f;
    bad |= (__float_as_uint(v) & 0x7f800000u) == 0x7f800000u;
    out[i] = v;
  }
  bad = __any_sync(kFull, bad);
  if (lane == 0) {
    qbad[row] = bad ? 1 : 0;
    if (bad) atomicAdd(nonfinite, 1);
  }
  __syncwarp();
  if (cosine) warp_normalize(out, dim, lane);
  float s = 0.0f;
  for (int i = lane; i < dim; i += 32) s = fmaf(out[i], out[i], s);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (lane == 0) {
    qnorm2[row] = drop_qnorm ? 0.0f : s;
    const float qn = sqrtf(s) * 1.0001f;
    if (l2) {
      const float t = qn + xmax;
      eps[row] = em.c_l2 * t * t;
    } else {
      eps[row] = em.c_ip * qn * xmax + em.c_abs * (1.0f + qn * xmax);
    }
  }
}

// The result slot of a query that holds NaN or infinity: no label, NaN distance.
__device__ __forceinline__ void write_invalid(uint64_t* labels, float* dists, uint64_t* keys,
                                              size_t o) {
  labels[o] = kInvalidLabel;
  dists[o] = __int_as_float(0x7fc00000);
  if (keys) keys[o] = ~0ull;
}

// Results of a search over an empty index: every slot unfilled (QV_INVALID_LABEL, +inf), or
// invalid (NaN distance) for a query holding NaN or infinity, which is also counted. One warp
// per query.
__global__ void empty_results_kernel(const float* q, size_t nq, int dim, int k, uint64_t* labels,
                                     float* dists, uint64_t* keys, int* nonfinite) {
  const int lane = threadIdx.x & 31;
  const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= nq) return;
  bool bad = false;
  for (int i = lane; i < dim; i += 32)
    bad |= (__float_as_uint(q[row * dim + i]) & 0x7f800000u) == 0x7f800000u;
  bad = __any_sync(kFull, bad);
  if (bad && lane == 0) atomicAdd(nonfinite, 1);
  for (int j = lane; j < k; j += 32) {
    const size_t o = row * k + j;
    labels[o] = kInvalidLabel;
    dists[o] = bad ? __int_as_float(0x7fc00000) : kInf;
    if (keys) keys[o] = ~0ull;
  }
}

// ---- per-thread bounded max-heap in shared memory (interleaved: element i of thread t at i*stride+t)

struct ThreadHeap {
  float* d;
  uint32_t* r;
  int stride;
  int n;
  int cap;
  __device__ float top_d() const { return d[0]; }
  __device__ void push(float dist, uint32_t row) {
    if (n < cap) {  // sift up
      int i = n++;
      while (i > 0) {
        const int p = (i - 1) >> 1;
        const float pd = d[p * stride];
        const uint32_t pr = r[p * stride];
        if (!dev::key_less(pd, pr, dist, row)) break;
        d[i * stride] = pd;
        r[i * stride] = pr;
        i = p;
      }
      d[i * stride] = dist;
      r[i * stride] = row;
      return;
    }
    if (!dev::key_less(dist, row, d[0], r[0])) return;
    int i = 0;  // replace the root and sift down
    for (;;) {
      const int l = 2 * i + 1;
      if (l >= n) break;
      int w = l;
      float wd = d[l * stride];
      uint32_t wr = r[l * stride];
      if (l + 1 < n) {
        const float rd = d[(l + 1) * stride];
        const uint32_t rr = r[(l + 1) * stride];
        if (dev::key_less(wd, wr, rd, rr)) {
          w = l + 1;
          wd = rd;
          wr = rr;
        }
      }
      if (!dev::key_less(dist, row, wd, wr)) break;
      d[i * stride] = wd;
      r[i * stride] = wr;
      i = w;
    }
    d[i * stride] = dist;
    r[i * stride] = row;
  }
};

// ---- SIMT screen ---------------------------------------------------------------------------------
// Unit u: chunk = u / n_qtiles, query tile = u % n_qtiles (chunk-major, so concurrently running
// units share row chunks in L2). Thread t owns query qtile*qpb + t. Screen distance:
//   L2: ||q||^2 + ||x||^2 - 2<q,x>,  IP/cosine: ip_one - <q,x> (ip_one 1, or 0 for -<q,x>),
//   float32 with FMA.
template <bool kL2>
__global__ void __launch_bounds__(128) flat_screen_simt_kernel(
    const float* __restrict__ qp, int dpad, const float* __restrict__ qnorm2, int nq, int qpb,
    const float* __restrict__ x, int dim, const float* __restrict__ xnorm2, int64_t nrows,
    const uint64_t* __restrict__ bitmap, int64_t chunk_rows, int n_qtiles, int n_chunks, int kk,
    float* __restrict__ cand_d, uint32_t* __restrict__ cand_r, int* __restrict__ cand_n,
    unsigned* __restrict__ thr_bits, float ip_one) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);  // kScreenRows x kScreenDChunk
  float* hd = xs + kScreenRows * kScreenDChunk;     // kk x qpb
  uint32_t* hr = reinterpret_cast<uint32_t*>(hd + static_cast<size_t>(kk) * qpb);

  const int chunk = blockIdx.x / n_qtiles;
  const int qtile = blockIdx.x - chunk * n_qtiles;
  const int t = threadIdx.x;
  const int q = qtile * qpb + t;
  const bool active = t < qpb && q < nq;
  const int64_t r0 = static_cast<int64_t>(chunk) * chunk_rows;
  const int64_t r1 = min(nrows, r0 + chunk_rows);

  ThreadHeap heap{hd + (active ? t : 0), hr + (active ? t : 0), qpb, 0, kk};
  float thr = active ? dev::from_ordered_bits(thr_bits[q]) : -kInf;
  const float qn = (active && kL2) ? qnorm2[q] : 0.0f;
  const float* qrow = qp + static_cast<size_t>(active ? q : 0) * dpad;
  const int warp = t >> 5, lane = t & 31, nwarps = blockDim.x >> 5;

  for (int64_t rb = r0; rb < r1; rb += kScreenRows) {
    const int nr = static_cast<int>((r1 - rb < kScreenRows ? r1 - rb : kScreenRows));
    float acc[kScreenRows];
#pragma unroll
    for (int r = 0; r < kScreenRows; ++r) acc[r] = 0.0f;
    for (int c0 = 0; c0 < dim; c0 += kScreenDChunk) {
      const int dc = min(kScreenDChunk, dpad - c0);
      __syncthreads();
      for (int rr = warp; rr < kScreenRows; rr += nwarps) {
        const float* src = x + (rb + rr) * static_cast<int64_t>(dim);
        for (int c = lane; c < dc; c += 32) {
          const int col = c0 + c;
          xs[rr * kScreenDChunk + c] = (rr < nr && col < dim) ? src[col] : 0.0f;
        }
      }
      __syncthreads();
      if (active) {
        for (int cc = 0; cc < dc; cc += 32) {
          float qv[32];
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(qrow + c0 + cc + j);
            qv[j] = v.x;
            qv[j + 1] = v.y;
            qv[j + 2] = v.z;
            qv[j + 3] = v.w;
          }
#pragma unroll
          for (int r = 0; r < kScreenRows; ++r) {
            const float4* xr = reinterpret_cast<const float4*>(xs + r * kScreenDChunk + cc);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 v = xr[j];
              acc[r] = fmaf(qv[4 * j], v.x, acc[r]);
              acc[r] = fmaf(qv[4 * j + 1], v.y, acc[r]);
              acc[r] = fmaf(qv[4 * j + 2], v.z, acc[r]);
              acc[r] = fmaf(qv[4 * j + 3], v.w, acc[r]);
            }
          }
        }
      }
    }
    if (!active) continue;
#pragma unroll
    for (int r = 0; r < kScreenRows; ++r) {
      if (r < nr) {
        const int64_t row = rb + r;
        float dist = kL2 ? fmaf(-2.0f, acc[r], qn + xnorm2[row]) : ip_one - acc[r];
        dist = dev::nan_to_inf(dist);
        if (dist <= thr && dev::bitmap_test(bitmap, static_cast<uint64_t>(row))) {
          heap.push(dist, static_cast<uint32_t>(row));
          if (heap.n == kk) thr = fminf(thr, heap.top_d());
        }
      }
    }
  }
  if (!active) return;
  const size_t base = (static_cast<size_t>(q) * n_chunks + chunk) * kk;
  for (int i = 0; i < heap.n; ++i) {
    cand_d[base + i] = hd[i * qpb + t];
    cand_r[base + i] = hr[i * qpb + t];
  }
  cand_n[static_cast<size_t>(q) * n_chunks + chunk] = heap.n;
  if (heap.n == kk) atomicMin(thr_bits + q, dev::ordered_bits(heap.top_d()));
}

// ---- finalize: merge, exact rerank, certificate ------------------------------------------------------

// Candidates are rows (group_rows == 1, the SIMT screen) or groups of group_rows consecutive rows
// (the tensor-core screen), each with the best screen distance among its admitted rows. The kk
// best candidates are kept (their kk-th screen value is T); group candidates are expanded into
// their admitted rows, and every kept row is recomputed exactly in the reference's order. Any row
// left out has screen distance >= T, so T - eps >= (k-th exact distance) certifies the result.
__global__ void __launch_bounds__(kFinalizeThreads) flat_finalize_kernel(
    const float* __restrict__ qp, int dpad, const float* __restrict__ eps_q, int nq,
    const float* __restrict__ x, int dim, int64_t nrows, const uint64_t* __restrict__ bitmap,
    const uint64_t* __restrict__ labels, uint64_t row_offset,
    bool l2, int kind, const float* __restrict__ cand_d,
    const uint32_t* __restrict__ cand_r, const int* __restrict__ cand_n, int n_chunks, int kk,
    int group_rows, int pool, int k, uint64_t* __restrict__ out_labels, float* __restrict__ out_d,
    uint64_t* __restrict__ out_keys, const int* __restrict__ qbad, int* __restrict__ fail_count,
    int* __restrict__ fail_q, float* __restrict__ fail_dk, int* __restrict__ flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sd = reinterpret_cast<float*>(smem_raw);               // pool
  uint64_t* sk = reinterpret_cast<uint64_t*>(sd + pool);        // pool (8-byte aligned: pool%2==0)
  __shared__ int s_total;
  const int q = blockIdx.x;
  if (q >= nq) return;
  if (qbad[q]) {  // NaN or infinity in the query: no results
    for (int j = threadIdx.x; j < k; j += blockDim.x)
      write_invalid(out_labels, out_d, out_keys, static_cast<size_t>(q) * k + j);
    return;
  }
  if (threadIdx.x == 0) {
    int tot = 0;
    for (int c = 0; c < n_chunks; ++c) tot += cand_n[static_cast<size_t>(q) * n_chunks + c];
    s_total = tot;
  }
  for (int i = threadIdx.x; i < pool; i += blockDim.x) {
    sd[i] = kInf;
    sk[i] = ~0ull;
  }
  __syncthreads();
  // Gather: chunk c's candidates land at [c*kk, c*kk + n_c).
  for (int i = threadIdx.x; i < n_chunks * kk; i += blockDim.x) {
    const int c = i / kk, j = i - c * kk;
    const size_t slot = static_cast<size_t>(q) * n_chunks + c;
    if (j < cand_n[slot]) {
      sd[i] = cand_d[slot * kk + j];
      sk[i] = cand_r[slot * kk + j];
    }
  }
  dev::block_bitonic_sort<false>(sd, sk, nullptr, pool);
  const int total = s_total;
  const float T = total >= kk ? sd[kk - 1] : kInf;
  int m = min(total, kk);
  __syncthreads();
  if (group_rows > 1) {
    // Expand the m best groups into their rows; rows past the index or rejected by the filter
    // become (+inf, ~0). The group ids move to registers first (m <= kk <= blockDim.x).
    const uint64_t gid = threadIdx.x < m ? sk[threadIdx.x] : 0;
    __syncthreads();
    if (threadIdx.x < m) {
      for (int j = 0; j < group_rows; ++j) {
        const uint64_t row = gid * static_cast<uint64_t>(group_rows) + j;
        const bool in = row < static_cast<uint64_t>(nrows) && dev::bitmap_test(bitmap, row);
        sd[threadIdx.x * group_rows + j] = in ? 0.0f : kInf;
        sk[threadIdx.x * group_rows + j] = in ? row : ~0ull;
      }
    }
    m *= group_rows;
    __syncthreads();
  }
  // Exact rerank of the m best (reference AVX2 order), one warp per candidate.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const float* qrow = qp + static_cast<size_t>(q) * dpad;
  // Four rows per warp at a time, so that their loads overlap; a slot without an admitted row
  // (row ~0) keeps +inf.
  for (int i0 = warp * 4; i0 < m; i0 += nwarps * 4) {
    uint64_t row[4];
    const float* xr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      row[r] = i0 + r < m ? sk[i0 + r] : ~0ull;
      xr[r] = x + (row[r] == ~0ull ? 0 : row[r]) * dim;
    }
    float e[4];
    dev::warp_exact_distance_x4(qrow, xr, dim, l2, lane, e, kind);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < 4; ++r)
        if (row[r] != ~0ull) sd[i0 + r] = dev::nan_to_inf(e[r]);
    }
  }
  __syncthreads();
  // Re-sort the first m' = next_pow2(m) entries (the tail beyond m holds screen values; mask them).
  int mp = 1;
  while (mp < m) mp <<= 1;
  for (int i = m + threadIdx.x; i < mp; i += blockDim.x) {
    sd[i] = kInf;
    sk[i] = ~0ull;
  }
  dev::block_bitonic_sort<false>(sd, sk, nullptr, mp);
  if (threadIdx.x == 0) {
    const float dk = m >= k ? sd[k - 1] : kInf;
    bool ok = true;
    if (total >= kk && m >= k) ok = (T - eps_q[q]) >= dk;
    if (!ok) {
      const int slot = atomicAdd(fail_count, 1);
      fail_q[slot] = q;
      fail_dk[slot] = dk;
      atomicAdd(flags + kFlagRescanned, 1);
    }
  }
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const size_t o = static_cast<size_t>(q) * k + j;
    if (j < m && sk[j] != ~0ull) {
      out_d[o] = sd[j];
      out_labels[o] = labels[sk[j]];
      if (out_keys) out_keys[o] = row_offset + sk[j];
    } else {
      out_d[o] = kInf;
      out_labels[o] = kInvalidLabel;
      if (out_keys) out_keys[o] = ~0ull;
    }
  }
}

// ---- finalize for group candidates: one warp per query -------------------------------------------

// simd::avx2::dot / l2sqr (src/simd/kernels_avx2.cc:35-83) evaluated by ONE thread, in exactly the
// order dev::warp_reduce_avx2 uses: accumulator s[a][l] takes elements i + 8a + l of every
// 32-element block, 8-element blocks go to s[0][l], then (s0+s1)+(s2+s3) per l, the hsum
// (t[l]+t[l+4]) and (lo0+lo1)+(lo2+lo3), then the scalar tail (the first 4 products rounded and
// added in order when 4 or more remain, FMAs after). q is in shared memory (all lanes read the same
// element: a broadcast), x is this thread's row. Bit-identical to the warp version.
template <bool kDiff>
__device__ __forceinline__ float lane_reduce_avx2(const float* __restrict__ q,
                                                  const float* __restrict__ x, int dim) {
  float s[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int l = 0; l < 8; ++l) s[a][l] = 0.0f;
  auto acc = [&](float& dst, float u, float v) {
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    dst = __fmaf_rn(u, v, dst);
  };
  int i = 0;
  const bool vec = (dim & 3) == 0;  // rows and q start on 16-byte boundaries
  for (; i + 32 <= dim; i += 32) {
    if (vec) {
#pragma unroll
      for (int f = 0; f < 8; ++f) {
        const float4 xv = __ldg(reinterpret_cast<const float4*>(x + i) + f);
        const float4 qv = reinterpret_cast<const float4*>(q + i)[f];
        const int e = 4 * f;
        acc(s[(e + 0) >> 3][(e + 0) & 7], qv.x, xv.x);
        acc(s[(e + 1) >> 3][(e + 1) & 7], qv.y, xv.y);
        acc(s[(e + 2) >> 3][(e + 2) & 7], qv.z, xv.z);
        acc(s[(e + 3) >> 3][(e + 3) & 7], qv.w, xv.w);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) acc(s[e >> 3][e & 7], q[i + e], __ldg(x + i + e));
    }
  }
  for (; i + 8 <= dim; i += 8) {
#pragma unroll
    for (int l = 0; l < 8; ++l) acc(s[0][l], q[i + l], __ldg(x + i + l));
  }
  float t[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) t[l] = __fadd_rn(__fadd_rn(s[0][l], s[1][l]), __fadd_rn(s[2][l], s[3][l]));
  float lo[4];
#pragma unroll
  for (int l = 0; l < 4; ++l) lo[l] = __fadd_rn(t[l], t[l + 4]);
  float sum = __fadd_rn(__fadd_rn(lo[0], lo[1]), __fadd_rn(lo[2], lo[3]));
  int j = i;
  if (dim - i >= 4) {
    for (; j < i + 4; ++j) {
      float u = q[j], v = __ldg(x + j);
      if (kDiff) {
        u = __fsub_rn(u, v);
        v = u;
      }
      sum = __fadd_rn(sum, __fmul_rn(u, v));
    }
  }
  for (; j < dim; ++j) {
    float u = q[j], v = __ldg(x + j);
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    sum = __fmaf_rn(u, v, sum);
  }
  return sum;
}

// simd::avx2::l2sqr_sq8 / dot_sq8 (src/simd/kernels_avx2.cc:85-129) on a decoded row x, evaluated
// by ONE thread in the order dev::warp_reduce_sq8 uses: accumulator s[a][l] takes elements
// i + 8a + l of every 16-element block, 8-element blocks go to s[0][l], then s0 + s1 per l, the
// hsum, and the scalar tail (one FMA per element). Bit-identical to the warp version.
template <bool kDiff>
__device__ __forceinline__ float lane_reduce_sq8(const float* __restrict__ q,
                                                 const float* __restrict__ x, int dim) {
  float s[2][8];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int l = 0; l < 8; ++l) s[a][l] = 0.0f;
  auto acc = [&](float& dst, float u, float v) {
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    dst = __fmaf_rn(u, v, dst);
  };
  int i = 0;
  const bool vec = (dim & 3) == 0;  // rows and q start on 16-byte boundaries
  for (; i + 16 <= dim; i += 16) {
    if (vec) {
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        const float4 xv = __ldg(reinterpret_cast<const float4*>(x + i) + f);
        const float4 qv = reinterpret_cast<const float4*>(q + i)[f];
        const int e = 4 * f;
        acc(s[(e + 0) >> 3][(e + 0) & 7], qv.x, xv.x);
        acc(s[(e + 1) >> 3][(e + 1) & 7], qv.y, xv.y);
        acc(s[(e + 2) >> 3][(e + 2) & 7], qv.z, xv.z);
        acc(s[(e + 3) >> 3][(e + 3) & 7], qv.w, xv.w);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) acc(s[e >> 3][e & 7], q[i + e], __ldg(x + i + e));
    }
  }
  for (; i + 8 <= dim; i += 8) {
#pragma unroll
    for (int l = 0; l < 8; ++l) acc(s[0][l], q[i + l], __ldg(x + i + l));
  }
  float t[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) t[l] = __fadd_rn(s[0][l], s[1][l]);
  float lo[4];
#pragma unroll
  for (int l = 0; l < 4; ++l) lo[l] = __fadd_rn(t[l], t[l + 4]);
  float sum = __fadd_rn(__fadd_rn(lo[0], lo[1]), __fadd_rn(lo[2], lo[3]));
  for (; i < dim; ++i) acc(sum, q[i], __ldg(x + i));
  return sum;
}

// CentroidTable's sequential sums (src/internal/centroid_table.h:65-144) evaluated by ONE thread:
// the same rounded operations in the same order as dev::seq_reduce / dev::seq_norm_minus_2dot,
// with the row read 16 bytes at a time when the rows allow it (q is in shared memory, where all
// lanes read the same element). kNorm: ||x||^2 - 2<q,x> (L2 only).
template <bool kDiff, bool kNorm>
__device__ __forceinline__ float lane_reduce_seq(const float* __restrict__ q,
                                                 const float* __restrict__ x, int dim) {
  float s = 0.0f, nn = 0.0f;
  auto acc = [&](float u, float v) {
    if (kNorm) nn = __fadd_rn(nn, __fmul_rn(v, v));
    if (kDiff) {
      u = __fsub_rn(u, v);
      v = u;
    }
    s = __fadd_rn(s, __fmul_rn(u, v));
  };
  int i = 0;
  if ((dim & 3) == 0) {  // rows and q start on 16-byte boundaries
    for (; i < dim; i += 4) {
      const float4 xv = __ldg(reinterpret_cast<const float4*>(x + i));
      const float4 qv = *reinterpret_cast<const float4*>(q + i);
      acc(qv.x, xv.x);
      acc(qv.y, xv.y);
      acc(qv.z, xv.z);
      acc(qv.w, xv.w);
    }
  }
  for (; i < dim; ++i) acc(q[i], __ldg(x + i));
  return kNorm ? __fsub_rn(nn, __fmul_rn(2.0f, s)) : s;
}

// The exact distance of the stored row x for an exact-distance kind (summation order |
// kKindNegIp): the float32 kernels' order (src/flat_index.cc:87), the SQ8 kernels'
// (src/hnsw_index.cc:202-218; x is then the decoded codes), CentroidTable's sequential sums
// (src/internal/centroid_table.h:65-85), or for L2 its ||x||^2 - 2<q,x> (:94-144); inner
// product as 1 - <q,x>, or -<q,x> with kKindNegIp.
__device__ __forceinline__ float lane_exact_distance(const float* q, const float* x, int dim,
                                                     bool l2, int kind) {
  const int order = kind & 3;
  float s;
  if (order == 3 && l2) return lane_reduce_seq<false, true>(q, x, dim);
  if (order == 1)
    s = l2 ? lane_reduce_sq8<true>(q, x, dim) : lane_reduce_sq8<false>(q, x, dim);
  else if (order >= 2)
    s = l2 ? lane_reduce_seq<true, false>(q, x, dim) : lane_reduce_seq<false, false>(q, x, dim);
  else
    s = l2 ? lane_reduce_avx2<true>(q, x, dim) : lane_reduce_avx2<false>(q, x, dim);
  if (l2) return s;
  return (kind & kKindNegIp) ? -s : __fsub_rn(1.0f, s);
}

// One warp per query, for the tensor-core screen's group candidates (kk <= 32 groups per unit,
// k <= kk). Each unit's list is sorted by (value, group). With few lists the rank of a candidate
// in the union is the sum over lists of how many entries precede it there (a binary search each);
// with more, a k-way merge takes the warp's minimum over the lists' heads kk times. Either way
// the kk best groups are selected and the kk-th gives T. The groups' admitted rows (8 * kk at
// most) are then recomputed exactly in batches, one row per lane, and the k best are picked by k
// rounds of a warp minimum over (distance, row). Same results and certificate as
// flat_finalize_kernel.
constexpr int kGroupFinalizeWarps = 4;
constexpr int kRankMergeChunks = 3;

// Shared memory of one warp of flat_finalize_groups_kernel (the layout the kernel carves).
__host__ __device__ inline size_t group_finalize_bytes_per_warp(int dpad, int n_chunks, int kk,
                                                                int group_rows) {
  const size_t nl = static_cast<size_t>(n_chunks) * kk, nx = static_cast<size_t>(kk) * group_rows;
  const size_t bytes = static_cast<size_t>(dpad) * 4 + nl * 8 + ((n_chunks + 1) & ~1) * 4 +
                       static_cast<size_t>(kk) * 8 + nx * 12;
  return (bytes + 15) / 16 * 16;
}

__global__ void __launch_bounds__(32 * kGroupFinalizeWarps, 6) flat_finalize_groups_kernel(
    const float* __restrict__ qp, int dpad, const float* __restrict__ eps_q, int nq,
    const float* __restrict__ x, int dim, int64_t nrows, const uint64_t* __restrict__ bitmap,
    const uint64_t* __restrict__ labels, uint64_t row_offset, bool l2, int kind,
    const float* __restrict__ cand_d, const uint32_t* __restrict__ cand_r,
    const int* __restrict__ cand_n, int n_chunks, int kk, int group_rows, int k, bool rank_merge,
    uint64_t* __restrict__ out_labels, float* __restrict__ out_d, uint64_t* __restrict__ out_keys,
    const int* __restrict__ qbad, const int* __restrict__ screen_err,
    int* __restrict__ fail_count, int* __restrict__ fail_q, float* __restrict__ fail_dk,
    int* __restrict__ flags) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = blockIdx.x * kGroupFinalizeWarps + warp;
  // Per warp: the query (dpad floats), the lists (n_chunks x kk values and groups), their
  // lengths, the selected groups (kk) and the expanded rows' exact distances (kk * group_rows).
  const int nl = n_chunks * kk, nx = kk * group_rows;
  const size_t per_warp = group_finalize_bytes_per_warp(dpad, n_chunks, kk, group_rows);
  unsigned char* base = smem_raw + per_warp * warp;
  float* sq = reinterpret_cast<float*>(base);
  float* ld = sq + dpad;
  uint32_t* lr = reinterpret_cast<uint32_t*>(ld + nl);
  int* ln = reinterpret_cast<int*>(lr + nl);
  uint32_t* sel = reinterpret_cast<uint32_t*>(ln + ((n_chunks + 1) & ~1));
  float* sv = reinterpret_cast<float*>(sel + kk);  // the selected groups' screen values
  float* ed = sv + kk;
  uint64_t* er = reinterpret_cast<uint64_t*>(ed + nx);  // 8-byte aligned: offsets are even words
  if (q >= nq) return;
  // A screen that gave up waiting on a pipeline barrier left its candidates incomplete: every
  // query then fails the certificate and is answered by the exact rescan.
  const bool aborted = *screen_err != 0;
  if (aborted && q == 0 && lane == 0) atomicAdd(flags + kFlagTimeout, 1);
  if (qbad[q]) {  // NaN or infinity in the query: no results
    for (int j = lane; j < k; j += 32)
      write_invalid(out_labels, out_d, out_keys, static_cast<size_t>(q) * k + j);
    return;
  }
  const float* qrow = qp + static_cast<size_t>(q) * dpad;
  for (int i = lane; i < dpad; i += 32) sq[i] = qrow[i];
  int total = 0;
  for (int c = lane; c < n_chunks; c += 32) ln[c] = cand_n[static_cast<size_t>(q) * n_chunks + c];
  __syncwarp();
  for (int c = 0; c < n_chunks; ++c) total += ln[c];
  for (int i = lane; i < nl; i += 32) {
    const int c = i / kk, j = i - c * kk;
    if (j < ln[c]) {
      const size_t slot = static_cast<size_t>(q) * n_chunks + c;
      ld[i] = cand_d[slot * kk + j];
      lr[i] = cand_r[slot * kk + j];
    }
  }
  __syncwarp();
  const int m = min(total, kk);
  float T = kInf;
  if (rank_merge) {
    // Few lists: each entry's rank in the union is its index in its own list plus, for every
    // other list, the number of entries there that precede it by (value, group) (a binary search;
    // groups are distinct across lists, so ranks are distinct). Ranks below kk are the kk best.
    for (int i = lane; i < nl; i += 32) {
      const int c = i / kk, j = i - c * kk;
      if (j >= ln[c]) continue;
      const float d = ld[i];
      const uint32_t g = lr[i];
      int rank = j;
      for (int c2 = 0; c2 < n_chunks && rank < m; ++c2) {
        if (c2 == c) continue;
        const float* L = ld + c2 * kk;
        const uint32_t* R = lr + c2 * kk;
        int lo = 0, hi = ln[c2];
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (dev::key_less(L[mid], R[mid], d, g))
            lo = mid + 1;
          else
            hi = mid;
        }
        rank += lo;
      }
      if (rank < m) {
        sel[rank] = g;
        sv[rank] = d;
      }
    }
    __syncwarp();
    if (m == kk) T = sv[kk - 1];
  } else {
  // k-way merge of the sorted unit lists: each round, the warp's minimum over the lists' heads
  // (lane l watches lists l and l + 32) is the next best candidate.
  int h0 = 0, h1 = 0;
  const int c0 = lane, c1 = lane + 32;
  for (int r = 0; r < m; ++r) {
    float bd = kInf;
    uint32_t bg = 0xffffffffu;
    int bl = -1;
    if (c0 < n_chunks && h0 < ln[c0]) {
      bd = ld[c0 * kk + h0];
      bg = lr[c0 * kk + h0];
      bl = c0;
    }
    if (c1 < n_chunks && h1 < ln[c1]) {
      const float d1 = ld[c1 * kk + h1];
      const uint32_t g1 = lr[c1 * kk + h1];
      if (dev::key_less(d1, g1, bd, bg)) {
        bd = d1;
        bg = g1;
        bl = c1;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float od = __shfl_xor_sync(kFull, bd, o);
      const uint32_t og = __shfl_xor_sync(kFull, bg, o);
      const int ol = __shfl_xor_sync(kFull, bl, o);
      if (dev::key_less(od, og, bd, bg)) {
        bd = od;
        bg = og;
        bl = ol;
      }
    }
    if (lane == 0) {
      sel[r] = bg;
      sv[r] = bd;
    }
    if (r == kk - 1) T = bd;
    h0 += bl == c0 ? 1 : 0;
    h1 += bl == c1 ? 1 : 0;
  }
  __syncwarp();
  }
  // Exact distances of the selected groups' admitted rows, one row per lane.
  auto exact_rows = [&](int g0, int g1) {
    for (int i = g0 * group_rows + lane; i < g1 * group_rows; i += 32) {
      const int g = i / group_rows, j = i - g * group_rows;
      const uint64_t row = static_cast<uint64_t>(sel[g]) * group_rows + j;
      const bool in = row < static_cast<uint64_t>(nrows) && dev::bitmap_test(bitmap, row);
      ed[i] = in ? dev::nan_to_inf(lane_exact_distance(sq, x + row * dim, dim, l2, kind)) : kInf;
      er[i] = in ? row : ~0ull;
    }
    __syncwarp();
  };
  // Groups come in ascending screen value, and every row of group g has an exact distance of at
  // least sv[g] - eps. So the groups are expanded in batches: after each, the k-th best exact
  // distance dk among the expanded rows is found, and the next group is expanded only when it
  // could still hold a row at or below dk; otherwise none of the remaining groups' rows can enter
  // the top k (their exact distances all exceed dk >= the final k-th distance). The first batch
  // holds one group for k <= 2 (the best group usually holds the answer), else about 2k groups
  // (at least 4, at most 16); later batches 8.
  int ng = m;
  const int first = k <= 2 ? 1 : min(16, max(4, (2 * k + 3) / 4 * 4));
  if (group_rows > 1 && m > first && k <= 32) {
    exact_rows(0, first);
    ng = first;
    // k-th smallest (distance, row) among the expanded rows: k rounds of a warp minimum with
    // removal (lane r keeps round r's winner), then the removed entries are put back.
    auto kth_best = [&]() {
      float win_d = kInf, kth = kInf;
      int win_i = -1;
      for (int r = 0; r < k; ++r) {
        float bd = kInf;
        uint64_t br = ~0ull;
        int bi = -1;
        for (int i = lane; i < ng * group_rows; i += 32) {
          if (dev::key_less(ed[i], er[i], bd, br)) {
            bd = ed[i];
            br = er[i];
            bi = i;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float od = __shfl_xor_sync(kFull, bd, o);
          const uint64_t orow = __shfl_xor_sync(kFull, br, o);
          const int oi = __shfl_xor_sync(kFull, bi, o);
          if (dev::key_less(od, orow, bd, br)) {
            bd = od;
            br = orow;
            bi = oi;
          }
        }
        if (lane == r) {
          win_d = bd;
          win_i = bi;
        }
        if (lane == 0 && bi >= 0) ed[bi] = kInf;
        if (r == k - 1) kth = bd;
        __syncwarp();
      }
      if (lane < k && win_i >= 0) ed[win_i] = win_d;
      __syncwarp();
      return kth;
    };
    while (ng < m) {
      const float dk1 = kth_best();
      if (dk1 < kInf && sv[ng] - eps_q[q] > dk1) break;
      const int next = min(m, ng + 8);
      exact_rows(ng, next);
      ng = next;
    }
  } else {
    exact_rows(0, m);
  }
  // The k best by (distance, row): k rounds of a warp minimum; each round's winner is removed.
  float dk = kInf;
  for (int r = 0; r < k; ++r) {
    float bd = kInf;
    uint64_t br = ~0ull;
    int bi = -1;
    for (int i = lane; i < ng * group_rows; i += 32) {
      if (dev::key_less(ed[i], er[i], bd, br)) {
        bd = ed[i];
        br = er[i];
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float od = __shfl_xor_sync(kFull, bd, o);
      const uint64_t orow = __shfl_xor_sync(kFull, br, o);
      const int oi = __shfl_xor_sync(kFull, bi, o);
      if (dev::key_less(od, orow, bd, br)) {
        bd = od;
        br = orow;
        bi = oi;
      }
    }
    const size_t o = static_cast<size_t>(q) * k + r;
    if (lane == 0) {
      const bool valid = br != ~0ull;
      out_d[o] = valid ? bd : kInf;
      out_labels[o] = valid ? labels[br] : kInvalidLabel;
      if (out_keys) out_keys[o] = valid ? row_offset + br : ~0ull;
      if (bi >= 0) {
        ed[bi] = kInf;
        er[bi] = ~0ull;
      }
    }
    if (r == k - 1) dk = br != ~0ull ? bd : kInf;
    __syncwarp();
  }
  if (lane == 0) {
    bool ok = !aborted;
    if (ok && total >= kk) ok = (T - eps_q[q]) >= dk;
    if (!ok) {
      const int slot = atomicAdd(fail_count, 1);
      fail_q[slot] = q;
      fail_dk[slot] = dk;
      atomicAdd(flags + kFlagRescanned, 1);
    }
  }
}

// ---- exact rescan of uncertified queries -------------------------------------------------------------
// A query that fails the certificate is rescanned over every row, split into `slices` row ranges
// taken by different blocks (one block alone would stream the rows at a single SM's bandwidth):
// the grid walks the (failed query, slice) pairs. A block keeps a threshold buffer: rows whose
// exact distance is <= the running threshold (first the k-th exact distance the finalize found,
// an upper bound of the true one) are appended; when the buffer might overflow it is sorted and
// cut to k, which tightens the threshold. One row per thread, exact distances in the row kind's
// order (lane_exact_distance, the query staged in shared memory). With one slice the k best go
// straight to the output; otherwise each slice's k best (sorted by (distance, row), padded with
// (+inf, ~0)) go to sl_d / sl_r and flat_rescan_merge_kernel merges them.
__global__ void __launch_bounds__(256) flat_rescan_kernel(
    const float* __restrict__ qp, int dpad, const float* __restrict__ x, int dim, int64_t nrows,
    const uint64_t* __restrict__ labels, const uint64_t* __restrict__ bitmap, uint64_t row_offset,
    bool l2, int kind, int k, int cap, int slices, const int* __restrict__ fail_count,
    const int* __restrict__ fail_q, const float* __restrict__ fail_dk,
    float* __restrict__ sl_d, uint64_t* __restrict__ sl_r, uint64_t* __restrict__ out_labels,
    float* __restrict__ out_d, uint64_t* __restrict__ out_keys) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sq = reinterpret_cast<float*>(smem_raw);  // dpad floats (16-byte multiple)
  float* bd = sq + dpad;
  uint64_t* bk = reinterpret_cast<uint64_t*>(bd + cap);
  __shared__ int s_cnt, s_strict;
  __shared__ float s_thr;
  const int nfail = *fail_count;
  const int64_t pairs = static_cast<int64_t>(nfail) * slices;
  for (int64_t p = blockIdx.x; p < pairs; p += gridDim.x) {
    const int f = static_cast<int>(p / slices), sl = static_cast<int>(p - static_cast<int64_t>(f) * slices);
    const int q = fail_q[f];
    const int64_t lo = nrows * sl / slices, hi = nrows * (sl + 1) / slices;
    __syncthreads();
    for (int i = threadIdx.x; i < dpad; i += blockDim.x) sq[i] = qp[static_cast<size_t>(q) * dpad + i];
    if (threadIdx.x == 0) {
      s_cnt = 0;
      s_thr = fail_dk[f];
      s_strict = 0;
    }
    __syncthreads();
    const int64_t per_round = blockDim.x;
    for (int64_t rb = lo; rb < hi; rb += per_round) {
      // Once a compaction has kept k rows, the k-th of them precedes every row still to come
      // (rows are scanned in ascending order), so a row at exactly the threshold loses the tie.
      const float thr = s_thr;
      const bool strict = s_strict != 0;
      const int64_t row = rb + threadIdx.x;
      if (row < hi && dev::bitmap_test(bitmap, static_cast<uint64_t>(row))) {
        const float e = dev::nan_to_inf(lane_exact_distance(sq, x + row * dim, dim, l2, kind));
        if (e < thr || (e == thr && !strict)) {
          const int slot = atomicAdd(&s_cnt, 1);
          bd[slot] = e;
          bk[slot] = static_cast<uint64_t>(row);
        }
      }
      __syncthreads();
      if (s_cnt > cap - per_round) {  // compact to the k best
        for (int i = s_cnt + threadIdx.x; i < cap; i += blockDim.x) {
          bd[i] = kInf;
          bk[i] = ~0ull;
        }
        dev::block_bitonic_sort<false>(bd, bk, nullptr, cap);
        if (threadIdx.x == 0) {
          s_cnt = min(s_cnt, k);
          if (s_cnt == k) {
            s_thr = fminf(s_thr, bd[k - 1]);
            s_strict = 1;
          }
        }
      }
      __syncthreads();
    }
    for (int i = s_cnt + threadIdx.x; i < cap; i += blockDim.x) {
      bd[i] = kInf;
      bk[i] = ~0ull;
    }
    dev::block_bitonic_sort<false>(bd, bk, nullptr, cap);
    const int m = min(s_cnt, k);
    if (slices > 1) {
      const size_t o = static_cast<size_t>(p) * k;
      for (int j = threadIdx.x; j < k; j += blockDim.x) {
        sl_d[o + j] = j < m ? bd[j] : kInf;
        sl_r[o + j] = j < m ? bk[j] : ~0ull;
      }
      continue;
    }
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      const size_t o = static_cast<size_t>(q) * k + j;
      if (j < m) {
        out_d[o] = bd[j];
        out_labels[o] = labels[bk[j]];
        if (out_keys) out_keys[o] = row_offset + bk[j];
      } else {
        out_d[o] = kInf;
        out_labels[o] = kInvalidLabel;
        if (out_keys) out_keys[o] = ~0ull;
      }
    }
  }
}

// The k best (distance, row) of a failed query's slices (slices * k entries, sorted per slice)
// into the output; pool = next_pow2(slices * k).
__global__ void __launch_bounds__(256) flat_rescan_merge_kernel(
    const int* __restrict__ fail_count, const int* __restrict__ fail_q, int slices, int k,
    int pool, const float* __restrict__ sl_d, const uint64_t* __restrict__ sl_r,
    const uint64_t* __restrict__ labels, uint64_t row_offset, uint64_t* __restrict__ out_labels,
    float* __restrict__ out_d, uint64_t* __restrict__ out_keys) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* bd = reinterpret_cast<float*>(smem_raw);
  uint64_t* bk = reinterpret_cast<uint64_t*>(bd + pool);  // pool is a power of two >= 2
  const int nfail = *fail_count;
  const int n = slices * k;
  for (int f = blockIdx.x; f < nfail; f += gridDim.x) {
    const int q = fail_q[f];
    __syncthreads();
    for (int i = threadIdx.x; i < pool; i += blockDim.x) {
      const size_t src = static_cast<size_t>(f) * n + i;
      bd[i] = i < n ? sl_d[src] : kInf;
      bk[i] = i < n ? sl_r[src] : ~0ull;
    }
    dev::block_bitonic_sort<false>(bd, bk, nullptr, pool);
    __syncthreads();
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      const size_t o = static_cast<size_t>(q) * k + j;
      if (bk[j] != ~0ull) {
        out_d[o] = bd[j];
        out_labels[o] = labels[bk[j]];
        if (out_keys) out_keys[o] = row_offset + bk[j];
      } else {
        out_d[o] = kInf;
        out_labels[o] = kInvalidLabel;
        if (out_keys) out_keys[o] = ~0ull;
      }
    }
  }
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v != nullptr && *v != '\0') ? std::atoi(v) : dflt;
}

}  // namespace

// ---- host launchers ----------------------------------------------------------------------------------

void normalize_rows_device(float* d_x, size_t n, size_t dim, cudaStream_t st) {
  if (n == 0) return;
  const int rows_per_block = 8;
  normalize_rows_kernel<<<ceil_div(n, rows_per_block), 32 * rows_per_block, 0, st>>>(
      d_x, n, static_cast<int>(dim));
  check_launch("normalize_rows_kernel");
}

namespace {
// flags[0] = some value is NaN or infinite; flags[1] = some label is the reserved 2^64-1.
__global__ void check_rows_kernel(const float* __restrict__ x, size_t count,
                                  const uint64_t* __restrict__ labels, size_t n, int* flags) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t i0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  bool bad = false;
  for (size_t i = i0; i < count; i += stride)
    bad |= (__float_as_uint(x[i]) & 0x7f800000u) == 0x7f800000u;
  if (__any_sync(kFull, bad) && (threadIdx.x & 31) == 0) atomicOr(flags, 1);
  bool bad_label = false;
  if (labels != nullptr)
    for (size_t i = i0; i < n; i += stride) bad_label |= labels[i] == kInvalidLabel;
  if (__any_sync(kFull, bad_label) && (threadIdx.x & 31) == 0) atomicOr(flags + 1, 1);
}

__global__ void sequential_labels_kernel(uint64_t* out, size_t n, uint64_t first) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    out[i] = first + i;
}
}  // namespace

void flat_check_rows(const float* d_x, size_t count, const uint64_t* d_labels, size_t n,
                     int* d_flags, cudaStream_t st) {
  const unsigned grid =
      static_cast<unsigned>(std::min<size_t>(ceil_div(std::max(count, n), 256), 16384));
  check_rows_kernel<<<std::max(grid, 1u), 256, 0, st>>>(d_x, count, d_labels, n, d_flags);
  check_launch("check_rows_kernel");
}

void sequential_labels(uint64_t* d_out, size_t n, uint64_t first, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>(std::min<size_t>(ceil_div(n, 256), 16384));
  sequential_labels_kernel<<<std::max(grid, 1u), 256, 0, st>>>(d_out, n, first);
  check_launch("sequential_labels_kernel");
}

void flat_reserve(FlatState& s, size_t rows, cudaStream_t st) {
  if (rows <= s.cap) return;
  size_t cap = std::max<size_t>(rows, s.cap + s.cap / 2);
  DeviceBuffer x(cap * s.dim * sizeof(float)), n2(cap * sizeof(float)),
      lab(cap * sizeof(uint64_t));
  if (s.n > 0) {
    QV_CUDA(cudaMemcpyAsync(x.get(), s.x.get(), s.n * s.dim * sizeof(float),
                            cudaMemcpyDeviceToDevice, st));
    QV_CUDA(cudaMemcpyAsync(n2.get(), s.xnorm2.get(), s.n * sizeof(float),
                            cudaMemcpyDeviceToDevice, st));
    QV_CUDA(cudaMemcpyAsync(lab.get(), s.labels.get(), s.n * sizeof(uint64_t),
                            cudaMemcpyDeviceToDevice, st));
  }
  QV_CUDA(cudaStreamSynchronize(st));
  s.x = std::move(x);
  s.xnorm2 = std::move(n2);
  s.labels = std::move(lab);
  s.cap = cap;
}

void flat_append(FlatState& s, const float* d_rows, const uint64_t* d_labels, size_t n,
                 cudaStream_t st, bool normalize) {
  if (n == 0) return;
  flat_reserve(s, s.n + n, st);
  float* dst = s.x.get<float>() + s.n * s.dim;
  if (d_rows != dst)
    QV_CUDA(cudaMemcpyAsync(dst, d_rows, n * s.dim * sizeof(float), cudaMemcpyDeviceToDevice, st));
  QV_CUDA(cudaMemcpyAsync(s.labels.get<uint64_t>() + s.n, d_labels, n * sizeof(uint64_t),
                          cudaMemcpyDeviceToDevice, st));
  if (normalize && s.metric == QV_METRIC_COSINE) normalize_rows_device(dst, n, s.dim, st);
  DeviceBuffer maxbits(sizeof(unsigned), st);
  QV_CUDA(cudaMemsetAsync(maxbits.get(), 0, sizeof(unsigned), st));
  row_stats_kernel<<<ceil_div(n, 8), 256, 0, st>>>(dst, n, static_cast<int>(s.dim),
                                                   s.xnorm2.get<float>() + s.n,
                                                   maxbits.get<unsigned>());
  check_launch("row_stats_kernel");
  unsigned bits = 0;
  QV_CUDA(cudaMemcpyAsync(&bits, maxbits.get(), sizeof(bits), cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaStreamSynchronize(st));
  float mx;
  memcpy(&mx, &bits, sizeof(mx));
  s.max_norm = std::max(s.max_norm, mx);
  s.n += n;
  s.x16_rows = 0;  // the fp16 copy is rebuilt by the next tensor-core search
}

// Chooses how many row chunks to split the database into: enough units (query tiles x chunks) to
// fill the GPU, at most `max_chunks` (the finalize merges n_chunks * KK candidates per query in
// one block), preferring counts that leave the last wave of a persistent grid nearly full.
static int choose_chunks(size_t nrows, int n_qtiles, int max_chunks, int grid, int64_t align,
                         int64_t* chunk_rows, size_t min_chunk_rows = 0) {
  const int limit = static_cast<int>(std::min<size_t>(
      max_chunks, ceil_div(nrows, std::max<size_t>(static_cast<size_t>(align), min_chunk_rows))));
  int best = 1;
  double best_eff = -1.0;
  for (int c = 1; c <= limit; ++c) {
    const double units = static_cast<double>(c) * n_qtiles;
    const double waves = std::ceil(units / grid);
    const double eff = units / (waves * grid);
    // The fewest chunks within 2 % of the best wave efficiency: every work unit has a fixed cost
    // (operand loads, its first rows screened against the query's looser threshold, its output).
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = c;
    }
  }
  *chunk_rows = static_cast<int64_t>(ceil_div(ceil_div(nrows, best), align)) * align;
  return static_cast<int>(ceil_div(nrows, static_cast<size_t>(*chunk_rows)));
}

// Sizes and layout of one search's temporaries, carved from one device block (offsets in bytes,
// each 256-byte aligned).
struct FlatPlan {
  bool tensor = false;
  int dim = 0, dpad = 0, kk = 0, n_qtiles = 0, n_chunks = 0, qpb = 0, group_rows = 1;
  int64_t chunk_rows = 0;
  size_t slots = 0;
  int rescan_slices = 1;  // row slices of an uncertified query's rescan
  size_t qp = 0, qn2 = 0, eps = 0, qbad = 0, fail = 0, cand_d = 0, cand_r = 0, cand_n = 0,
         thr = 0, tc = 0, flags = 0, rescan = 0, total = 0;
};

// Row slices of one uncertified query's rescan: enough for the rows to stream from many SMs, at
// least 4096 rows each, the per-slice results of every query within kRescanScratchBytes, and at
// most 4096 entries per query to merge.
constexpr size_t kRescanScratchBytes = size_t{32} << 20;
static int rescan_slices_for(size_t nrows, size_t nq, size_t k, int nsm) {
  const size_t per_slice = nq * k * (sizeof(float) + sizeof(uint64_t));
  size_t sl = std::min<size_t>(2 * static_cast<size_t>(nsm), ceil_div(nrows, 4096));
  sl = std::min(sl, kRescanScratchBytes / std::max<size_t>(per_slice, 1));
  sl = std::min(sl, 4096 / k);
  return static_cast<int>(std::max<size_t>(sl, 1));
}

static size_t align256(size_t x) { return (x + 255) & ~size_t{255}; }

// allow_tensor: the tensor-core screen may be used (the allocation-free entry point screens on
// the CUDA cores only); own_flags: the block also holds the kSearchFlagWords report words.
static FlatPlan plan_search(const FlatState& s, size_t nq, size_t k, bool allow_tensor,
                            bool own_flags) {
  FlatPlan P;
  P.dim = static_cast<int>(s.dim);
  P.dpad = static_cast<int>(ceil_div(s.dim, 32) * 32);
  const int nsm = sm_count(s.device);
  // QV_FLAT_KK overrides the candidate budget of the SIMT screen (any value >= k); small budgets
  // exercise the exact rescan. QV_FLAT_SCREEN=simt selects the SIMT screen.
  const int forced_kk = env_int("QV_FLAT_KK", 0);
  P.tensor = allow_tensor && forced_kk == 0 && flat_tc_eligible(s, k);
  const size_t nrows = std::max<size_t>(s.n, 1);
  if (P.tensor) {
    P.kk = flat_tc_kk(s, k);
    // Work units cover query groups of 2 x 128 (narrow screen), 4 x 128 (narrow screen in CTA
    // pairs) or one 128-query tile (wide).
    P.n_qtiles = static_cast<int>(ceil_div(nq, static_cast<size_t>(flat_tc_group_rows(s, k))));
    // At least kTcMinChunkRows rows per unit: every unit has a fixed candidate cost (each query's
    // list starts empty and takes most of its first groups), which small tables cannot amortize.
    P.n_chunks = choose_chunks(nrows, P.n_qtiles, std::max(1, kMaxCandidatesPerQuery / P.kk),
                               flat_tc_workers(s, k), 128, &P.chunk_rows, kTcMinChunkRows);
    P.group_rows = kTcGroupRows;
  } else {
    P.kk = static_cast<int>(next_pow2(k + std::max<size_t>(8, k / 4)));
    if (forced_kk > 0) P.kk = std::max<int>(static_cast<int>(k), forced_kk);
    const int heap_budget = 64 * 1024;
    P.qpb = std::min<int>(128, heap_budget / (P.kk * 8));
    if (P.qpb >= 32) P.qpb = P.qpb / 32 * 32;
    P.qpb = std::max(1, P.qpb);
    P.n_qtiles = static_cast<int>(ceil_div(nq, P.qpb));
    P.n_chunks = choose_chunks(nrows, P.n_qtiles, std::max(1, kMaxCandidatesPerQuery / P.kk),
                               3 * nsm, kScreenRows, &P.chunk_rows);
    P.group_rows = 1;
  }
  P.slots = nq * static_cast<size_t>(P.n_chunks);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  P.qp = take(nq * P.dpad * sizeof(float));
  P.qn2 = take(nq * sizeof(float));
  P.eps = take(nq * sizeof(float));
  P.qbad = take(nq * sizeof(int));
  P.fail = take(2 * sizeof(int) + nq * (sizeof(int) + sizeof(float)));
  P.cand_d = take(P.slots * P.kk * sizeof(float));
  P.cand_r = take(P.slots * P.kk * sizeof(uint32_t));
  P.cand_n = take(P.slots * sizeof(int));
  P.thr = take(nq * sizeof(unsigned));
  if (P.tensor) P.tc = take(flat_tc_scratch_bytes(s, nq, k, P.kk));
  if (own_flags) P.flags = take(kSearchFlagWords * sizeof(int));
  // The allocation-free entry point (own_flags) rescans each query in one block: no slice results.
  P.rescan_slices = own_flags ? 1 : rescan_slices_for(nrows, nq, k, nsm);
  if (P.rescan_slices > 1)
    P.rescan = take(nq * static_cast<size_t>(P.rescan_slices) * k *
                    (sizeof(float) + sizeof(uint64_t)));
  P.total = off;
  return P;
}

// Resets what every search's temporaries must start from: no candidates per (query, chunk),
// +inf thresholds, the rescan list's count and the screen's error word, and (when given) the
// report words.
__global__ void init_search_kernel(int* cand_n, size_t slots, unsigned* thr, size_t nq,
                                   int* fail_hdr, int* flags) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t i0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  for (size_t i = i0; i < slots; i += stride) cand_n[i] = 0;
  for (size_t i = i0; i < nq; i += stride) thr[i] = 0xff800000u;  // ordered bits of +inf
  if (i0 < 2) fail_hdr[i0] = 0;
  if (flags != nullptr && i0 < kSearchFlagWords) flags[i0] = 0;
}

// The whole search on stream `st`, temporaries at `base` (plan P). No host synchronization.
static void run_search(const FlatState& s, const FlatPlan& P, unsigned char* base,
                       const float* d_queries, size_t nq, size_t k, const uint64_t* d_bitmap,
                       uint64_t* d_labels, float* d_dists, uint64_t* d_keys, int* d_flags,
                       cudaStream_t st) {
  const int dim = P.dim, dpad = P.dpad, kk = P.kk;
  const bool l2 = s.metric == QV_METRIC_L2;
  const int kind = static_cast<int>(s.sum_order) | (s.neg_ip ? kKindNegIp : 0);
  const int nsm = sm_count(s.device);
  float* qp = reinterpret_cast<float*>(base + P.qp);
  float* qn2 = reinterpret_cast<float*>(base + P.qn2);
  float* eps = reinterpret_cast<float*>(base + P.eps);
  int* qbad = reinterpret_cast<int*>(base + P.qbad);
  int* fail_count = reinterpret_cast<int*>(base + P.fail);
  int* screen_err = fail_count + 1;
  int* fail_q = fail_count + 2;
  float* fail_dk = reinterpret_cast<float*>(fail_q + nq);
  float* cand_d = reinterpret_cast<float*>(base + P.cand_d);
  uint32_t* cand_r = reinterpret_cast<uint32_t*>(base + P.cand_r);
  int* cand_n = reinterpret_cast<int*>(base + P.cand_n);
  unsigned* thr = reinterpret_cast<unsigned*>(base + P.thr);

  init_search_kernel<<<static_cast<unsigned>(std::min<size_t>(
                           ceil_div(std::max(P.slots, nq), 256), 4 * static_cast<size_t>(nsm))),
                       256, 0, st>>>(cand_n, P.slots, thr, nq, fail_count,
                                     P.flags ? d_flags : nullptr);
  check_launch("init_search_kernel");
  const double u = std::ldexp(1.0, -24);
  const double gamma = (dim + 2) * u / (1.0 - (dim + 2) * u);
  EpsModel em;
  em.c_l2 = static_cast<float>(2.0 * (2.0 * gamma + 4.0 * u));
  em.c_ip = static_cast<float>(2.0 * (2.0 * gamma));
  em.c_abs = static_cast<float>(2.0 * (2.0 * u));
  prep_queries_kernel<<<ceil_div(nq, 8), 256, 0, st>>>(d_queries, nq, dim, dpad,
                                                       s.metric == QV_METRIC_COSINE, l2,
                                                       s.drop_qnorm, em,
                                                       s.max_norm, qp, qn2, eps, qbad,
                                                       d_flags + kFlagNonFinite);
  check_launch("prep_queries_kernel");

  if (P.tensor) {
    {
      FlatState& ms = const_cast<FlatState&>(s);  // the fp16 copy is a cache of the rows
      std::lock_guard<std::mutex> lock(ms.x16_mu);
      flat_tc_prepare(ms, st);
    }
    flat_screen_tc(s, qp, dpad, nq, k, d_bitmap, P.n_chunks, P.chunk_rows, kk, cand_d, cand_r,
                   cand_n, thr, eps, screen_err, base + P.tc, st);
  } else {
    const size_t smem = kScreenRows * kScreenDChunk * sizeof(float) +
                        static_cast<size_t>(kk) * P.qpb * (sizeof(float) + sizeof(uint32_t));
    const dim3 grid(static_cast<unsigned>(P.n_qtiles * P.n_chunks));
    KernelTimer timer(st, "flat_screen_simt_kernel", 2.0 * nq * static_cast<double>(s.n) * dim,
                      false);
    auto kernel = l2 ? flat_screen_simt_kernel<true> : flat_screen_simt_kernel<false>;
    QV_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kernel<<<grid, 128, smem, st>>>(qp, dpad, qn2, static_cast<int>(nq), P.qpb, s.x.get<float>(),
                                    dim, s.xnorm2.get<float>(), static_cast<int64_t>(s.n),
                                    d_bitmap, P.chunk_rows, P.n_qtiles, P.n_chunks, kk, cand_d,
                                    cand_r, cand_n, thr, s.neg_ip ? 0.0f : 1.0f);
    timer.stop();
    check_launch("flat_screen_simt_kernel");
  }

  if (P.tensor) {
    // The tensor-core screen keeps 8-row groups; the finalize expands the kk best into rows.
    QV_REQUIRE(P.n_chunks <= 64, "group finalize: more than 64 row chunks");
    // Up to kRankMergeChunks unit lists per query are merged by ranks, more by rounds of a warp
    // minimum (QV_FINALIZE_MERGE=rounds: always by rounds; both select the same groups).
    const char* merge_env = std::getenv("QV_FINALIZE_MERGE");
    const bool rank_merge = P.n_chunks <= kRankMergeChunks &&
                            !(merge_env != nullptr && std::strcmp(merge_env, "rounds") == 0);
    const size_t gsmem =
        kGroupFinalizeWarps * group_finalize_bytes_per_warp(dpad, P.n_chunks, kk, P.group_rows);
    QV_CUDA(cudaFuncSetAttribute(flat_finalize_groups_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsmem));
    flat_finalize_groups_kernel<<<static_cast<unsigned>(ceil_div(nq, kGroupFinalizeWarps)),
                                  32 * kGroupFinalizeWarps, gsmem, st>>>(
        qp, dpad, eps, static_cast<int>(nq), s.x.get<float>(), dim, static_cast<int64_t>(s.n),
        d_bitmap, s.labels.get<uint64_t>(), s.row_offset, l2, kind, cand_d, cand_r, cand_n,
        P.n_chunks, kk, P.group_rows, static_cast<int>(k), rank_merge, d_labels, d_dists, d_keys,
        qbad, screen_err,
        fail_count, fail_q, fail_dk, d_flags);
    check_launch("flat_finalize_groups_kernel");
  } else {
    const int pool = static_cast<int>(next_pow2(static_cast<size_t>(P.n_chunks) * kk));
    const size_t fsmem = pool * (sizeof(float) + sizeof(uint64_t));
    QV_CUDA(cudaFuncSetAttribute(flat_finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)fsmem));
    flat_finalize_kernel<<<static_cast<unsigned>(nq), kFinalizeThreads, fsmem, st>>>(
        qp, dpad, eps, static_cast<int>(nq), s.x.get<float>(), dim, static_cast<int64_t>(s.n),
        d_bitmap, s.labels.get<uint64_t>(), s.row_offset, l2, kind, cand_d, cand_r, cand_n,
        P.n_chunks, kk, 1, pool, static_cast<int>(k), d_labels, d_dists, d_keys, qbad, fail_count, fail_q,
        fail_dk, d_flags);
    check_launch("flat_finalize_kernel");
  }

  const int cap = static_cast<int>(next_pow2(k + 256));
  const int slices = P.rescan_slices;
  float* sl_d = slices > 1 ? reinterpret_cast<float*>(base + P.rescan) : nullptr;
  uint64_t* sl_r = slices > 1 ? reinterpret_cast<uint64_t*>(
                                    sl_d + nq * static_cast<size_t>(slices) * k)
                              : nullptr;
  const size_t rsmem = dpad * sizeof(float) + cap * (sizeof(float) + sizeof(uint64_t));
  QV_CUDA(cudaFuncSetAttribute(flat_rescan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)rsmem));
  flat_rescan_kernel<<<static_cast<unsigned>(std::min<size_t>(nq * slices, 2 * nsm)), 256, rsmem,
                       st>>>(
      qp, dpad, s.x.get<float>(), dim, static_cast<int64_t>(s.n), s.labels.get<uint64_t>(),
      d_bitmap, s.row_offset, l2, kind, static_cast<int>(k), cap, slices, fail_count, fail_q,
      fail_dk, sl_d, sl_r, d_labels, d_dists, d_keys);
  check_launch("flat_rescan_kernel");
  if (slices > 1) {
    const int pool = static_cast<int>(next_pow2(static_cast<size_t>(slices) * k));
    const size_t msmem = pool * (sizeof(float) + sizeof(uint64_t));
    QV_CUDA(cudaFuncSetAttribute(flat_rescan_merge_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
    flat_rescan_merge_kernel<<<static_cast<unsigned>(std::min<size_t>(nq, 2 * nsm)), 256, msmem,
                               st>>>(fail_count, fail_q, slices, static_cast<int>(k), pool, sl_d,
                                     sl_r, s.labels.get<uint64_t>(), s.row_offset, d_labels,
                                     d_dists, d_keys);
    check_launch("flat_rescan_merge_kernel");
  }
}

void flat_search(const FlatState& s, const float* d_queries, size_t nq, size_t k,
                 const uint64_t* d_bitmap, uint64_t* d_labels, float* d_dists, uint64_t* d_keys,
                 int* d_flags, cudaStream_t st) {
  if (nq == 0 || k == 0) return;
  QV_REQUIRE(k <= 1024, "k > 1024 is not supported by the GPU FlatIndex");
  if (s.n == 0) {  // nothing stored: every slot unfilled
    empty_results_kernel<<<ceil_div(nq, 8), 256, 0, st>>>(d_queries, nq, static_cast<int>(s.dim),
                                                          static_cast<int>(k), d_labels, d_dists,
                                                          d_keys, d_flags + kFlagNonFinite);
    check_launch("empty_results_kernel");
    return;
  }
  const FlatPlan P = plan_search(s, nq, k, /*allow_tensor=*/true, /*own_flags=*/false);
  // One stream-ordered block for every temporary (returned to the device's memory pool, which
  // keeps it for the next search, when the work queued before the free has run).
  DeviceBuffer arena(P.total, st);
  run_search(s, P, arena.get<unsigned char>(), d_queries, nq, k, d_bitmap, d_labels, d_dists,
             d_keys, d_flags, st);
}

// ---- allocation-free search ------------------------------------------------------------------------
//
// For callers that must not allocate device memory while they search (a serving loop with a fixed
// memory budget, code running in a driver callback or under an allocator lock, ...): the same
// Flat search, screened on the float32 CUDA cores and then certified and re-ranked exactly like
// flat_search, with every temporary carved from one file-scope device array. Results are
// identical to flat_search's.

constexpr size_t kNoAllocScratchBytes = size_t{64} << 20;  // per device, held until exit
constexpr int kNoAllocMaxDevices = 64;

}  // namespace qv

// The scratch itself. In host code this name is only a handle for cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_flat_noalloc_scratch[qv::kNoAllocScratchBytes];

namespace qv {

// Device address of the scratch on `device` (which must be current), resolved once per device.
// The address is cached for the life of the process: a device reset after the first call would
// leave it stale, so a process that uses this entry point must not reset that device.
static unsigned char* noalloc_scratch(int device) {
  static std::mutex mu;
  static void* addr[kNoAllocMaxDevices] = {};
  QV_REQUIRE(device >= 0 && device < kNoAllocMaxDevices, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_flat_noalloc_scratch);
    if (e != cudaSuccess)
      fail(QV_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    addr[device] = p;
  }
  return static_cast<unsigned char*>(addr[device]);
}

size_t flat_noalloc_max_bytes() { return kNoAllocScratchBytes; }

// The same search as flat_search, screened on the CUDA cores, with every temporary (the report
// words included) carved from the fixed scratch. Results equal flat_search's, also for queries
// holding NaN or infinity (QV_INVALID_LABEL with a NaN distance).
void flat_search_noalloc(const FlatState& s, const float* d_queries, size_t nq, size_t k,
                         const uint64_t* d_bitmap, uint64_t* d_labels, float* d_dists,
                         uint64_t* d_keys, cudaStream_t st) {
  if (nq == 0 || k == 0) return;
  QV_REQUIRE(k <= 1024, "k > 1024 is not supported by the GPU FlatIndex");
  const FlatPlan P = plan_search(s, nq, k, /*allow_tensor=*/false, /*own_flags=*/true);
  if (P.total > kNoAllocScratchBytes)
    fail(QV_ERR_INVALID, "allocation-free search needs " + std::to_string(P.total) +
                             " bytes of scratch for nq=" + std::to_string(nq) +
                             ", k=" + std::to_string(k) + "; its fixed scratch holds " +
                             std::to_string(kNoAllocScratchBytes) + " bytes (search fewer queries "
                             "per call)");
  unsigned char* base = noalloc_scratch(s.device);
  int* flags = reinterpret_cast<int*>(base + P.flags);
  if (s.n == 0) {
    empty_results_kernel<<<ceil_div(nq, 8), 256, 0, st>>>(d_queries, nq, static_cast<int>(s.dim),
                                                          static_cast<int>(k), d_labels, d_dists,
                                                          d_keys, flags + kFlagNonFinite);
    check_launch("empty_results_kernel");
    return;
  }
  // The scratch keeps the previous call's contents: run_search's first kernel resets what must
  // start empty (the report words included).
  run_search(s, P, base, d_queries, nq, k, d_bitmap, d_labels, d_dists, d_keys, flags, st);
}

}  // namespace qv
