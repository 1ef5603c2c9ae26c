// Shard merge / per-row top-k selection, and filter preparation (label bitmaps or label sets
// turned into one bit per stored position, which the scans test).
#include <algorithm>
#include <vector>

#include "qv_state.h"

namespace qv {
namespace {

constexpr float kInf = __builtin_huge_valf();

// Entry i of query q lives at part = i / per_part, j = i % per_part:
// index = part * part_stride + q * per_part + j. Sorted by (distance, key); the first k are kept.
__global__ void select_kernel(const float* __restrict__ d, const uint64_t* __restrict__ keys,
                              const uint64_t* __restrict__ labels, size_t nq, int parts,
                              int per_part, size_t part_stride, int pool, int k,
                              float* __restrict__ od, uint64_t* __restrict__ ok,
                              uint64_t* __restrict__ ol) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sd = reinterpret_cast<float*>(smem_raw);
  uint64_t* sk = reinterpret_cast<uint64_t*>(sd + pool);
  uint64_t* sl = sk + pool;
  const size_t q = blockIdx.x;
  const int n = parts * per_part;
  for (int i = threadIdx.x; i < pool; i += blockDim.x) {
    if (i < n) {
      const int part = i / per_part, j = i - part * per_part;
      const size_t idx = part * part_stride + q * per_part + j;
      sd[i] = d[idx];
      sk[i] = keys[idx];
      sl[i] = labels ? labels[idx] : kInvalidLabel;
    } else {
      sd[i] = kInf;
      sk[i] = ~0ull;
      sl[i] = kInvalidLabel;
    }
  }
  dev::block_bitonic_sort<true>(sd, sk, sl, pool);
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const size_t o = q * k + j;
    const bool valid = j < n && sk[j] != ~0ull;
    od[o] = valid ? sd[j] : kInf;
    if (ok) ok[o] = valid ? sk[j] : ~0ull;
    if (ol) ol[o] = valid ? sl[j] : kInvalidLabel;
  }
}

void launch_select(const float* d, const uint64_t* keys, const uint64_t* labels, size_t nq,
                   int parts, int per_part, size_t part_stride, int k, float* od, uint64_t* ok,
                   uint64_t* ol, cudaStream_t st) {
  if (nq == 0 || k == 0) return;
  const int pool = static_cast<int>(next_pow2(static_cast<size_t>(parts) * per_part));
  const size_t smem = pool * (sizeof(float) + 2 * sizeof(uint64_t));
  QV_REQUIRE(smem <= 227 * 1024, "top-k merge: parts * k is too large for one block");
  QV_CUDA(cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  select_kernel<<<static_cast<unsigned>(nq), 256, smem, st>>>(d, keys, labels, nq, parts,
                                                              per_part, part_stride, pool, k, od,
                                                              ok, ol);
  check_launch("select_kernel");
}

// One thread per 64 positions: bit = filter admits labels[pos].
__global__ void bitmap_from_label_bitmap_kernel(const uint64_t* __restrict__ labels, size_t count,
                                                const uint64_t* __restrict__ words,
                                                uint64_t universe, uint64_t* __restrict__ out) {
  const size_t w = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t nwords = (count + 63) / 64;
  if (w >= nwords) return;
  uint64_t bits = 0;
  for (int b = 0; b < 64; ++b) {
    const size_t pos = w * 64 + b;
    if (pos >= count) break;
    const uint64_t label = labels[pos];
    if (label < universe && ((words[label >> 6] >> (label & 63)) & 1ull)) bits |= 1ull << b;
  }
  out[w] = bits;
}

__global__ void bitmap_from_label_set_kernel(const uint64_t* __restrict__ labels, size_t count,
                                             const uint64_t* __restrict__ sorted, size_t n,
                                             uint64_t* __restrict__ out) {
  const size_t w = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t nwords = (count + 63) / 64;
  if (w >= nwords) return;
  uint64_t bits = 0;
  for (int b = 0; b < 64; ++b) {
    const size_t pos = w * 64 + b;
    if (pos >= count) break;
    const uint64_t label = labels[pos];
    size_t lo = 0, hi = n;
    while (lo < hi) {
      const size_t mid = (lo + hi) / 2;
      if (sorted[mid] < label) lo = mid + 1; else hi = mid;
    }
    if (lo < n && sorted[lo] == label) bits |= 1ull << b;
  }
  out[w] = bits;
}

}  // namespace

void merge_topk(size_t parts, size_t nq, size_t k, const float* d, const uint64_t* keys,
                const uint64_t* labels, float* od, uint64_t* ok, uint64_t* ol, cudaStream_t st) {
  launch_select(d, keys, labels, nq, static_cast<int>(parts), static_cast<int>(k), nq * k,
                static_cast<int>(k), od, ok, ol, st);
}

void select_topk(size_t nq, size_t n, size_t k, const float* d, const uint64_t* keys,
                 const uint64_t* labels, float* od, uint64_t* ok, uint64_t* ol, cudaStream_t st) {
  launch_select(d, keys, labels, nq, 1, static_cast<int>(n), 0, static_cast<int>(k), od, ok, ol,
                st);
}

void build_position_bitmap(const uint64_t* d_labels, size_t count, const qv_filter& f,
                           uint64_t* d_bitmap, cudaStream_t st) {
  const size_t nwords = std::max<size_t>(1, (count + 63) / 64);
  if (count == 0) {
    QV_CUDA(cudaMemsetAsync(d_bitmap, 0, nwords * sizeof(uint64_t), st));
    return;
  }
  switch (f.kind) {
    case QV_FILTER_POSITION_BITMAP: {
      QV_REQUIRE(f.data != nullptr || count == 0, "filter: null position bitmap");
      QV_REQUIRE(f.size >= count, "filter: position bitmap shorter than the index");
      QV_CUDA(cudaMemcpyAsync(d_bitmap, f.data, nwords * sizeof(uint64_t), cudaMemcpyHostToDevice,
                              st));
      // bits past `count` in the last word are never read
      return;
    }
    case QV_FILTER_LABEL_BITMAP: {
      const size_t words = (f.size + 63) / 64;
      DeviceBuffer dw(std::max<size_t>(1, words) * sizeof(uint64_t), st);
      if (words > 0) {
        QV_REQUIRE(f.data != nullptr, "filter: null label bitmap");
        QV_CUDA(cudaMemcpyAsync(dw.get(), f.data, words * sizeof(uint64_t), cudaMemcpyHostToDevice, st));
      }
      bitmap_from_label_bitmap_kernel<<<ceil_div(nwords, 256), 256, 0, st>>>(
          d_labels, count, dw.get<uint64_t>(), f.size, d_bitmap);
      check_launch("bitmap_from_label_bitmap_kernel");
      QV_CUDA(cudaStreamSynchronize(st));
      return;
    }
    case QV_FILTER_LABEL_SET: {
      std::vector<uint64_t> sorted(f.data, f.data + f.size);
      std::sort(sorted.begin(), sorted.end());
      sorted.erase(std::unique(sorted.begin(), sorted.end()), sorted.end());
      DeviceBuffer ds(std::max<size_t>(1, sorted.size()) * sizeof(uint64_t), st);
      if (!sorted.empty())
        QV_CUDA(cudaMemcpyAsync(ds.get(), sorted.data(), sorted.size() * sizeof(uint64_t),
                                cudaMemcpyHostToDevice, st));
      bitmap_from_label_set_kernel<<<ceil_div(nwords, 256), 256, 0, st>>>(
          d_labels, count, ds.get<uint64_t>(), sorted.size(), d_bitmap);
      check_launch("bitmap_from_label_set_kernel");
      QV_CUDA(cudaStreamSynchronize(st));
      return;
    }
    default:
      fail(QV_ERR_INVALID, "filter: unknown kind " + std::to_string(f.kind));
  }
}

}  // namespace qv
