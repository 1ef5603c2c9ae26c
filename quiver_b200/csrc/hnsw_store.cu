// HNSW's vector storage on the GPU and the exact scan HnswIndex::search falls back to when a filter
// admits few vectors (src/hnsw_index.cc:723-760 of the reference).
//
// The store keeps what the reference's HnswIndex keeps per node for distance computations:
//   * float32 storage: the prepared vector (normalized for cosine, src/hnsw_index.cc:334-339 and
//     :560-561);
//   * SQ8 storage: its 8-bit codes (ScalarQuantizer::encode, src/scalar_quantizer.cc:46-52) with
//     the per-dimension (vmin, vscale) trained on prepared vectors (:541-551), and, for the
//     scan, the decoded rows vmin + code * vscale rounded once (the FMA the reference's SQ8
//     kernels decode with, src/simd/kernels_avx2.cc:25-31), so that the scan reads float rows;
//   * labels, and a removed bit per node (soft deletes, src/hnsw_index.cc:1032-1040).
// The graph itself is not here: only the exact scan runs on the GPU. It is the Flat search
// (tensor-core screen, exact re-rank and certificate, flat.cu) over the admitted live nodes; for
// SQ8 the re-rank sums in the SQ8 kernels' order (FlatState::sum_order), so distances equal
// l2sqr_sq8 / 1 - dot_sq8 bit for bit. When the filter admits a small share of the nodes, their
// rows are first gathered into a compact block (in node order), so the scan's work follows the
// filter's cardinality as the reference's does.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "qv_state.h"

namespace qv {
namespace {

// The admitted nodes are gathered into a compact block when they are at most 1 / kGatherShare of
// the store; otherwise the scan reads the store in place and skips the rest by the bitmap.
constexpr size_t kGatherShare = 8;
constexpr unsigned kOrdPosInf = 0xff800000u;  // dev::ordered_bits(+inf)
constexpr unsigned kOrdNegInf = 0x007fffffu;  // dev::ordered_bits(-inf)

__global__ void fill_u32_kernel(unsigned* p, size_t n, unsigned v) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i < n) p[i] = v;
}

// Per-dimension minimum and maximum (ScalarQuantizer::train, src/scalar_quantizer.cc:15-21):
// thread = column, blockIdx.y strides over rows, one atomic per (thread, row slice).
__global__ void sq8_minmax_kernel(const float* __restrict__ x, size_t n, int dim, unsigned* lo,
                                  unsigned* hi) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= dim) return;
  float mn = __int_as_float(0x7f800000), mx = -mn;
  for (size_t r = blockIdx.y; r < n; r += gridDim.y) {
    const float v = x[r * dim + j];
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  atomicMin(lo + j, dev::ordered_bits(mn));
  atomicMax(hi + j, dev::ordered_bits(mx));
}

// vscale = range / 255 (1 for a constant dimension), src/scalar_quantizer.cc:23-31; *bad is set
// when a range is not finite.
__global__ void sq8_params_kernel(const unsigned* lo, const unsigned* hi, int dim, float* vmin,
                                  float* vscale, int* bad) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= dim) return;
  const float a = dev::from_ordered_bits(lo[j]), b = dev::from_ordered_bits(hi[j]);
  const float range = __fsub_rn(b, a);
  if (!isfinite(range)) atomicExch(bad, 1);
  vmin[j] = a;
  vscale[j] = range > 0.0f ? __fdiv_rn(range, 255.0f) : 1.0f;
}

// ScalarQuantizer::encode (src/scalar_quantizer.cc:46-52): nearest integer (ties to even) of
// (v - vmin) / vscale, clamped to 0..255; the row is overwritten with its decoded value
// vmin + code * vscale rounded once.
__global__ void sq8_encode_kernel(float* __restrict__ x, size_t total, int dim,
                                  const float* __restrict__ vmin, const float* __restrict__ vscale,
                                  uint8_t* __restrict__ codes) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += stride) {
    const int j = static_cast<int>(i % static_cast<size_t>(dim));
    const float lo = vmin[j], sc = vscale[j];
    const float t = rintf(__fdiv_rn(__fsub_rn(x[i], lo), sc));
    const float c = t >= 255.0f ? 255.0f : (t > 0.0f ? t : 0.0f);
    codes[i] = static_cast<uint8_t>(c);
    x[i] = __fmaf_rn(c, sc, lo);
  }
}

// bm[w] = (filter word, or all ones without a filter) & ~removed[w].
__global__ void live_bitmap_kernel(uint64_t* bm, const uint64_t* removed, size_t words,
                                   bool have_filter) {
  const size_t w = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (w >= words) return;
  bm[w] = (have_filter ? bm[w] : ~0ull) & ~removed[w];
}

// Set bits per block of 1024 bitmap words (the last word masked to n positions).
constexpr int kScanWords = 1024;
__global__ void bitmap_block_counts_kernel(const uint64_t* bm, size_t words, size_t n,
                                           unsigned* counts) {
  __shared__ unsigned s;
  if (threadIdx.x == 0) s = 0;
  __syncthreads();
  unsigned c = 0;
  for (size_t w = blockIdx.x * static_cast<size_t>(kScanWords) + threadIdx.x;
       w < words && w < (blockIdx.x + 1) * static_cast<size_t>(kScanWords); w += blockDim.x) {
    uint64_t b = bm[w];
    if (w == words - 1 && (n & 63)) b &= (1ull << (n & 63)) - 1;
    c += __popcll(b);
  }
  atomicAdd(&s, c);
  __syncthreads();
  if (threadIdx.x == 0) counts[blockIdx.x] = s;
}

// Positions of the set bits, in ascending order: block b writes from base[b]; inside a block,
// thread t owns words b*1024 + t*4 .. +3 and its offset is an exclusive scan over the block.
__global__ void __launch_bounds__(256) bitmap_positions_kernel(const uint64_t* bm, size_t words,
                                                               size_t n, const unsigned* base,
                                                               uint32_t* pos) {
  __shared__ unsigned warp_sums[8];
  const size_t w0 = blockIdx.x * static_cast<size_t>(kScanWords) + threadIdx.x * 4;
  uint64_t b[4];
  unsigned c = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const size_t w = w0 + i;
    b[i] = w < words ? bm[w] : 0ull;
    if (w == words - 1 && (n & 63)) b[i] &= (1ull << (n & 63)) - 1;
    c += __popcll(b[i]);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  unsigned before = 0;
  for (int i = 0; i < warp; ++i) before += warp_sums[i];
  unsigned out = base[blockIdx.x] + before + incl - c;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t bits = b[i];
    while (bits) {
      const int t = __ffsll(static_cast<long long>(bits)) - 1;
      pos[out++] = static_cast<uint32_t>((w0 + i) * 64 + t);
      bits &= bits - 1;
    }
  }
}

// Compact rows (and labels) of the listed node ids.
__global__ void gather_nodes_kernel(const float* __restrict__ x, const uint64_t* __restrict__ labels,
                                    const uint32_t* __restrict__ ids, size_t count, int dim,
                                    float* __restrict__ out, uint64_t* __restrict__ out_labels) {
  const size_t r = blockIdx.x * static_cast<size_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= count) return;
  const int lane = threadIdx.x & 31;
  const size_t id = ids[r];
  for (int c = lane; c < dim; c += 32) out[r * dim + c] = x[id * dim + c];
  if (lane == 0) out_labels[r] = labels[id];
}

// keys (positions in the gathered block) -> node ids.
__global__ void map_keys_kernel(uint64_t* keys, size_t total, const uint32_t* ids) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i < total && keys[i] != ~0ull) keys[i] = ids[keys[i]];
}

}  // namespace

void hnsw_sq8_train(HnswStoreState& s, const float* d_x, size_t n, cudaStream_t st) {
  const int dim = static_cast<int>(s.flat.dim);
  DeviceBuffer mm(2 * dim * sizeof(unsigned) + sizeof(int), st);
  unsigned* lo = mm.get<unsigned>();
  unsigned* hi = lo + dim;
  int* bad = reinterpret_cast<int*>(hi + dim);
  fill_u32_kernel<<<ceil_div(dim, 256), 256, 0, st>>>(lo, dim, kOrdPosInf);
  fill_u32_kernel<<<ceil_div(dim, 256), 256, 0, st>>>(hi, dim, kOrdNegInf);
  QV_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), st));
  const dim3 grid(static_cast<unsigned>(ceil_div(dim, 128)),
                  static_cast<unsigned>(std::min<size_t>(std::max<size_t>(1, n / 64), 512)));
  sq8_minmax_kernel<<<grid, 128, 0, st>>>(d_x, n, dim, lo, hi);
  check_launch("sq8_minmax_kernel");
  if (s.vmin.bytes() == 0) {
    s.vmin.allocate(dim * sizeof(float));
    s.vscale.allocate(dim * sizeof(float));
  }
  sq8_params_kernel<<<ceil_div(dim, 256), 256, 0, st>>>(lo, hi, dim, s.vmin.get<float>(),
                                                        s.vscale.get<float>(), bad);
  check_launch("sq8_params_kernel");
  int h_bad = 0;
  s.host_vmin.resize(dim);
  s.host_vscale.resize(dim);
  QV_CUDA(cudaMemcpyAsync(&h_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaMemcpyAsync(s.host_vmin.data(), s.vmin.get(), dim * sizeof(float),
                          cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaMemcpyAsync(s.host_vscale.data(), s.vscale.get(), dim * sizeof(float),
                          cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaStreamSynchronize(st));
  QV_REQUIRE(h_bad == 0, "ScalarQuantizer::train: value range overflows float");
  s.trained = true;
}

void hnsw_store_append(HnswStoreState& s, float* d_x, const uint64_t* d_labels, size_t n,
                       cudaStream_t st) {
  if (n == 0) return;
  const size_t dim = s.flat.dim, first = s.flat.n;
  if (s.storage == kStorageSq8) {
    const size_t need = (first + n) * dim;
    if (need > s.codes.bytes()) {
      DeviceBuffer grown(std::max(need, s.codes.bytes() + s.codes.bytes() / 2));
      if (first > 0)
        QV_CUDA(cudaMemcpyAsync(grown.get(), s.codes.get(), first * dim, cudaMemcpyDeviceToDevice,
                                st));
      QV_CUDA(cudaStreamSynchronize(st));
      s.codes = std::move(grown);
    }
    const size_t total = n * dim;
    sq8_encode_kernel<<<static_cast<unsigned>(std::min<size_t>(ceil_div(total, 256), 65536)), 256,
                        0, st>>>(d_x, total, static_cast<int>(dim), s.vmin.get<float>(),
                                 s.vscale.get<float>(), s.codes.get<uint8_t>() + first * dim);
    check_launch("sq8_encode_kernel");
  }
  // The rows are prepared already (normalized for cosine before training and encoding).
  flat_append(s.flat, d_x, d_labels, n, st, /*normalize=*/false);
  const size_t words = ceil_div(s.flat.n, 64);
  if (words > s.host_removed.size()) {
    s.host_removed.resize(words, 0);
    DeviceBuffer grown(std::max<size_t>(1, s.flat.cap / 64 + 1) * sizeof(uint64_t));
    QV_CUDA(cudaMemsetAsync(grown.get(), 0, grown.bytes(), st));
    if (s.removed.bytes() != 0)
      QV_CUDA(cudaMemcpyAsync(grown.get(), s.removed.get(),
                              std::min(s.removed.bytes(), grown.bytes()), cudaMemcpyDeviceToDevice,
                              st));
    QV_CUDA(cudaStreamSynchronize(st));
    s.removed = std::move(grown);
  }
}

void hnsw_store_mark_removed(HnswStoreState& s, uint32_t id, cudaStream_t st) {
  s.host_removed[id >> 6] |= 1ull << (id & 63);
  QV_CUDA(cudaMemcpyAsync(s.removed.get<uint64_t>() + (id >> 6), &s.host_removed[id >> 6],
                          sizeof(uint64_t), cudaMemcpyHostToDevice, st));
  QV_CUDA(cudaStreamSynchronize(st));
  ++s.removed_count;
}

void hnsw_store_search(const HnswStoreState& s, const float* d_queries, size_t nq, size_t k,
                       uint64_t* d_bitmap, bool have_filter, uint64_t* d_labels, float* d_dists,
                       uint64_t* d_keys, int* d_flags, cudaStream_t st) {
  const FlatState& f = s.flat;
  const size_t n = f.n, words = ceil_div(std::max<size_t>(n, 1), 64);
  const bool restrict_rows = have_filter || s.removed_count > 0;
  if (!restrict_rows || n == 0) {  // an empty store: every slot unfilled
    flat_search(f, d_queries, nq, k, nullptr, d_labels, d_dists, d_keys, d_flags, st);
    return;
  }
  live_bitmap_kernel<<<ceil_div(words, 256), 256, 0, st>>>(d_bitmap, s.removed.get<uint64_t>(),
                                                           words, have_filter);
  check_launch("live_bitmap_kernel");
  // How many nodes the scan admits (one small host round trip): a small share is gathered into a
  // compact block first, so that the scan's work follows the filter.
  const size_t blocks = ceil_div(words, kScanWords);
  DeviceBuffer counts((blocks + 1) * sizeof(unsigned), st);
  bitmap_block_counts_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      d_bitmap, words, n, counts.get<unsigned>());
  check_launch("bitmap_block_counts_kernel");
  std::vector<unsigned> h(blocks);
  QV_CUDA(cudaMemcpyAsync(h.data(), counts.get(), blocks * sizeof(unsigned),
                          cudaMemcpyDeviceToHost, st));
  QV_CUDA(cudaStreamSynchronize(st));
  std::vector<unsigned> base(blocks + 1, 0);
  for (size_t b = 0; b < blocks; ++b) base[b + 1] = base[b] + h[b];
  const size_t admitted = base[blocks];
  if (admitted * kGatherShare > n) {
    flat_search(f, d_queries, nq, k, d_bitmap, d_labels, d_dists, d_keys, d_flags, st);
    return;
  }
  FlatState g;
  g.device = f.device;
  g.dim = f.dim;
  g.metric = f.metric;
  g.sum_order = f.sum_order;
  if (admitted == 0) {  // nothing to scan: every slot unfilled (flat_search on an empty state)
    flat_search(g, d_queries, nq, k, nullptr, d_labels, d_dists, d_keys, d_flags, st);
    return;
  }
  DeviceBuffer dbase(blocks * sizeof(unsigned), st), ids(admitted * sizeof(uint32_t), st);
  QV_CUDA(cudaMemcpyAsync(dbase.get(), base.data(), blocks * sizeof(unsigned),
                          cudaMemcpyHostToDevice, st));
  bitmap_positions_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      d_bitmap, words, n, dbase.get<unsigned>(), ids.get<uint32_t>());
  check_launch("bitmap_positions_kernel");
  flat_reserve(g, admitted, st);
  DeviceBuffer glabels(admitted * sizeof(uint64_t), st);
  gather_nodes_kernel<<<ceil_div(admitted, 8), 256, 0, st>>>(
      f.x.get<float>(), f.labels.get<uint64_t>(), ids.get<uint32_t>(), admitted,
      static_cast<int>(f.dim), g.x.get<float>(), glabels.get<uint64_t>());
  check_launch("gather_nodes_kernel");
  flat_append(g, g.x.get<float>(), glabels.get<uint64_t>(), admitted, st, /*normalize=*/false);
  flat_search(g, d_queries, nq, k, nullptr, d_labels, d_dists, d_keys, d_flags, st);
  if (d_keys != nullptr) {
    const size_t total = nq * k;
    map_keys_kernel<<<ceil_div(total, 256), 256, 0, st>>>(d_keys, total, ids.get<uint32_t>());
    check_launch("map_keys_kernel");
  }
  // The gathered block is released only after the search that reads it has run.
  QV_CUDA(cudaStreamSynchronize(st));
}

}  // namespace qv
