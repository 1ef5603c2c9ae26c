// Host-side state of the GPU indexes behind the C ABI handles, and the launcher entry points the
// kernels' translation units export to capi.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "qv_internal.cuh"

namespace qv {

// ---- Flat --------------------------------------------------------------------------------------
// Rows live in HBM row-major as float32 exactly as the reference stores them (normalized for
// cosine), with their labels, a squared norm per row for the L2 screen, and a scaled fp16 copy
// padded to at least 64 columns for the tensor-core screen.
// Summation order of the exact distances of a FlatState's rows: the reference's float32 kernels
// (FlatIndex), its SQ8 kernels (an HNSW SQ8 store, whose rows are the decoded codes), or plain
// sequential sums with every multiply and add rounded (CentroidTable::l2 / ::dot: the IVF-PQ
// coarse probe over the centroids), or, for L2, ||x||^2 - 2<q,x> from two such sums
// (CentroidTable::nearest_batch: the coarse assignment of rows to lists).
enum : uint32_t { kSumOrderF32 = 0, kSumOrderSq8 = 1, kSumOrderSeq = 2, kSumOrderNormDot = 3 };
// The exact-distance kind the re-rank kernels take: the summation order, plus kKindNegIp when an
// inner-product distance is -<q,x> (the coarse probe's) instead of 1 - <q,x>.
constexpr int kKindNegIp = 4;

struct FlatState {
  int device = 0;
  size_t dim = 0;
  uint32_t metric = 0;
  uint32_t sum_order = kSumOrderF32;
  bool neg_ip = false;  // inner-product distances are -<q,x> (screens score them the same way)
  // L2 screens leave out ||q||^2 (distances are ||x||^2 - 2<q,x>, kSumOrderNormDot).
  bool drop_qnorm = false;
  uint64_t row_offset = 0;
  size_t n = 0, cap = 0;
  DeviceBuffer x;         // cap x dim f32
  DeviceBuffer xnorm2;    // cap f32, sum of squares (screen only)
  DeviceBuffer labels;    // cap u64
  float max_norm = 0.0f;  // max ||x|| over stored rows (screen error bound)
  std::vector<uint64_t> host_labels;
  // fp16 copy for the tensor-core screen (n x kpad, kpad = dim rounded up to 16), built on the
  // first search after rows change; x16_err = max ||x - x16/scale|| over rows.
  DeviceBuffer x16;
  size_t kpad = 0, x16_rows = 0;
  // Device words of the fp16 copy: [0] bits of max |x| (the copy's power-of-two scale follows
  // from it), [1] bits of max ||x - x16 / scale||. Read by the kernels only, so building the copy
  // needs no host round trip.
  DeviceBuffer x16_stats;
  // Recorded after the copy's kernels; searches on other streams wait for it.
  cudaEvent_t x16_ready = nullptr;
  std::mutex x16_mu;
  FlatState() = default;
  FlatState(const FlatState&) = delete;
  FlatState& operator=(const FlatState&) = delete;
  ~FlatState() {
    if (x16_ready != nullptr) cudaEventDestroy(x16_ready);
  }
};

// Words a search's kernels report into (device int array, accumulated with atomics):
// [0] queries the certificate rejected and the exact rescan answered, [1] queries holding NaN or
// infinity (their results are QV_INVALID_LABEL with a NaN distance), [2] tensor-core screen
// launches that gave up waiting on a pipeline barrier (their queries were all rescanned exactly).
constexpr int kSearchFlagWords = 4;
enum { kFlagRescanned = 0, kFlagNonFinite = 1, kFlagTimeout = 2 };
struct SearchFlags {
  int* dev = nullptr;        // kSearchFlagWords device ints for _device searches
  int* host = nullptr;       // their pinned host copy, queued after each _device search
  cudaEvent_t done = nullptr;  // recorded after that copy
  int* sync_dev = nullptr;   // the same for the host-buffer entry points (which wait)
  int* sync_host = nullptr;
};
// This thread's report words on `device` (allocated on first use).
SearchFlags& thread_search_flags(int device);

void flat_search_noalloc(const FlatState& s, const float* d_queries, size_t nq, size_t k,
                         const uint64_t* d_bitmap, uint64_t* d_labels, float* d_dists,
                         uint64_t* d_keys, cudaStream_t st);
size_t flat_noalloc_max_bytes();
// The tensor-core screen's candidates are groups of this many consecutive rows.
constexpr int kTcGroupRows = 8;
// The tensor-core screen applies (flat_tc_eligible); the wide variant (dim > 128 or k > 24)
// handles it (flat_tc_is_wide); best-list length in 8-row groups (flat_tc_kk).
bool flat_tc_eligible(const FlatState& s, size_t k);
bool flat_tc_is_wide(const FlatState& s, size_t k);
int flat_tc_kk(const FlatState& s, size_t k);
bool flat_tc_wide_fits(const FlatState& s, size_t k);
int flat_tc_wide_kk(size_t k);
size_t flat_tc_wide_list_bytes(const FlatState& s, int kk);
void flat_tc_prepare(FlatState& s, cudaStream_t st);
// Work units cover query groups of flat_tc_group_rows queries; flat_tc_workers of them (CTAs, or
// CTA pairs) run at once.
int flat_tc_group_rows(const FlatState& s, size_t k);
int flat_tc_workers(const FlatState& s, size_t k);
// Device scratch the tensor-core screen needs for nq queries, k results, best lists of kk.
size_t flat_tc_scratch_bytes(const FlatState& s, size_t nq, size_t k, int kk);
void flat_screen_tc(const FlatState& s, const float* qp, int dpad, size_t nq, size_t k,
                    const uint64_t* d_bitmap, int n_chunks, int64_t chunk_rows, int kk,
                    float* cand_d, uint32_t* cand_r, int* cand_n, unsigned* thr_bits, float* eps,
                    int* err, void* scratch, cudaStream_t st);

void flat_reserve(FlatState& s, size_t rows, cudaStream_t st);
// Device-side input checks for an add from device memory: d_flags[0] is set when a value is NaN
// or infinite, d_flags[1] when a label is 2^64-1 (d_labels may be null).
void flat_check_rows(const float* d_x, size_t count, const uint64_t* d_labels, size_t n,
                     int* d_flags, cudaStream_t st);
// d_out[i] = first + i.
void sequential_labels(uint64_t* d_out, size_t n, uint64_t first, cudaStream_t st);
// Appends n rows (device pointer, row-major) with labels (device pointer); cosine rows are
// normalized unless `normalize` is false (rows that are already prepared).
void flat_append(FlatState& s, const float* d_rows, const uint64_t* d_labels, size_t n,
                 cudaStream_t st, bool normalize = true);
// Enqueues an exact search on `st` and returns without waiting for it. The kernels add their
// reports into d_flags (kSearchFlagWords device ints, see kFlag*).
void flat_search(const FlatState& s, const float* d_queries, size_t nq, size_t k,
                 const uint64_t* d_bitmap, uint64_t* d_labels, float* d_dists, uint64_t* d_keys,
                 int* d_flags, cudaStream_t st);

// ---- HNSW vector storage and its filtered exact scan (hnsw_store.cu) ---------------------------
enum : uint32_t { kStorageF32 = 0, kStorageSq8 = 1 };  // quiver::Storage
struct HnswStoreState {
  FlatState flat;            // rows the scan reads: prepared float32, or decoded SQ8; labels
  uint32_t storage = kStorageF32;
  bool trained = false;      // SQ8 parameters set (once)
  DeviceBuffer vmin, vscale;  // dim f32 each (SQ8)
  std::vector<float> host_vmin, host_vscale;
  DeviceBuffer codes;        // n x dim u8 (SQ8), node order
  DeviceBuffer removed;      // one bit per node: soft-deleted
  std::vector<uint64_t> host_removed;
  size_t removed_count = 0;
  std::unordered_map<uint64_t, uint32_t> label_to_id;  // a label's current node
};
// ScalarQuantizer::train on n prepared device rows: sets vmin / vscale (device and host copies).
void hnsw_sq8_train(HnswStoreState& s, const float* d_x, size_t n, cudaStream_t st);
// Appends n prepared device rows (SQ8: encoded, and d_x overwritten with the decoded rows).
void hnsw_store_append(HnswStoreState& s, float* d_x, const uint64_t* d_labels, size_t n,
                       cudaStream_t st);
void hnsw_store_mark_removed(HnswStoreState& s, uint32_t id, cudaStream_t st);
// The exact scan over the live nodes the position bitmap admits (d_bitmap: ceil(n / 64) words,
// the filter's when have_filter, else scratch; overwritten). d_keys (optional) get node ids.
void hnsw_store_search(const HnswStoreState& s, const float* d_queries, size_t nq, size_t k,
                       uint64_t* d_bitmap, bool have_filter, uint64_t* d_labels, float* d_dists,
                       uint64_t* d_keys, int* d_flags, cudaStream_t st);

// ---- IVF-PQ ------------------------------------------------------------------------------------
// Inverted lists are stored list-major and contiguous in HBM (codes count x m bytes, labels,
// optional float32 vectors) with offsets[nlist+1]; global_base[l] is the offset of this index's
// first entry of list l inside the full (unsharded) list, which makes candidate keys comparable
// across shards.
struct IvfState {
  int device = 0;
  size_t dim = 0, nlist = 0, m = 0, dsub = 0;
  uint32_t metric = 0;
  size_t train_iterations = 20;
  bool store_vectors = false;
  uint64_t seed = 1234;
  bool trained = false;
  size_t count = 0;
  DeviceBuffer centroids;    // nlist x dim f32
  DeviceBuffer cnorm2;       // nlist f32, ||c||^2 sequential (CentroidTable::reset)
  DeviceBuffer codebooks;    // m x 256 x dsub f32
  DeviceBuffer precomputed;  // nlist x m x 256 f32 (L2 and within budget) or empty
  DeviceBuffer offsets;      // nlist + 1 u64
  DeviceBuffer global_base;  // nlist u32
  DeviceBuffer codes;        // count x m u8
  DeviceBuffer labels;       // count u64
  DeviceBuffer vectors;      // count x dim f32 (store_vectors)
  std::vector<float> host_centroids, host_codebooks;
  std::vector<uint64_t> host_offsets;
  std::vector<uint32_t> host_global_base;
  std::vector<uint8_t> host_codes;
  std::vector<uint64_t> host_labels;
  // The centroids as a Flat table (labels 0..nlist-1, CentroidTable's sequential summation,
  // inner products scored -<q,c>): the coarse probe's tensor-core path searches it.
  std::unique_ptr<FlatState> coarse_table;
  // The same rows scored as add() assigns them (||c||^2 - 2<x,c>) for the L2 and cosine metrics;
  // the inner-product metric assigns by -<x,c>, as coarse_table scores.
  std::unique_ptr<FlatState> l2_assign_table;
  const FlatState* assign_table() const {
    return metric == QV_METRIC_IP ? coarse_table.get() : l2_assign_table.get();
  }
  bool ip() const { return metric != 0; }
  bool use_precomputed() const { return precomputed.bytes() != 0; }
};

void ivf_set_trained(IvfState& s, const float* h_centroids, const float* h_codebooks,
                     cudaStream_t st);
// Coarse assignment + PQ encode of n device rows (already normalized for cosine when needed).
void ivf_encode_device(const IvfState& s, const float* d_x, size_t n, uint32_t* d_assign,
                       uint8_t* d_codes, cudaStream_t st);
// CentroidTable::nearest_batch (src/internal/centroid_table.h:94-144) of n device rows against k
// device centroids, bit-identical: ||c||^2 - 2<x,c> (or -<x,c> by_ip), first minimum. d_cnorm2:
// k floats of scratch.
void nearest_centroids_device(const float* d_x, size_t n, const float* d_cents, size_t k,
                              size_t dim, bool by_ip, float* d_cnorm2, uint32_t* d_assign,
                              cudaStream_t st);
// IvfPqIndex::train (src/ivfpq_index.cc:144-206) with the assignments on the GPU; installs the
// trained state. h_in: n x dim host rows.
void ivf_train(IvfState& s, const float* h_in, size_t n, cudaStream_t st);
// Normalizes n rows in place with simd::normalize semantics (cosine).
void normalize_rows_device(float* d_x, size_t n, size_t dim, cudaStream_t st);
// Rebuilds device list arrays from the host mirrors (+ optional device vectors in storage order).
void ivf_upload_lists(IvfState& s, cudaStream_t st);
void ivf_search(const IvfState& s, const float* d_queries, size_t nq, size_t k, size_t nprobe,
                size_t refine_factor, const uint64_t* d_bitmap, uint64_t* d_labels,
                float* d_dists, cudaStream_t st);
void ivf_candidates(const IvfState& s, const float* d_queries, size_t nq, size_t keep,
                    size_t nprobe, const uint64_t* d_bitmap, float* d_dists, uint64_t* d_keys,
                    uint64_t* d_labels, cudaStream_t st);
void ivf_refine(const IvfState& s, const float* d_queries, size_t nq, size_t keep,
                const uint64_t* d_keys, float* d_exact, cudaStream_t st);

// ---- selection / merge -------------------------------------------------------------------------
void merge_topk(size_t parts, size_t nq, size_t k, const float* d, const uint64_t* keys,
                const uint64_t* labels, float* od, uint64_t* ok, uint64_t* ol, cudaStream_t st);
void select_topk(size_t nq, size_t n, size_t k, const float* d, const uint64_t* keys,
                 const uint64_t* labels, float* od, uint64_t* ok, uint64_t* ol, cudaStream_t st);

// Position bitmap on device from a label bitmap/set, for `count` stored labels (device pointer).
void build_position_bitmap(const uint64_t* d_labels, size_t count, const qv_filter& f,
                           uint64_t* d_bitmap, cudaStream_t st);

}  // namespace qv
