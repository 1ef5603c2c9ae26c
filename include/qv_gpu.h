/* quiver-b200 C ABI: the drop-in boundary between Quiver's host-side API and the sm_100a kernels.
 *
 * Every entry point is extern "C", takes plain pointers and sizes, never throws, and returns a
 * qv_status. On failure qv_last_error() returns a thread-local message whose text matches what the
 * reference's quiver::Error would carry for the same mistake (e.g. "vectors must not contain NaN
 * or infinity"), so the C++ wrapper can rethrow quiver::Error and the Python layer ValueError.
 *
 * Citations name the reference interface each entry point replaces, as file:line of the reference
 * Quiver project. The reference reaches that interface from Python through its nanobind module
 * (python/quiver_ext.cc); these functions are what that binding's lambdas would call instead.
 *
 * Host-buffer entry points (no "_device" suffix) take caller-owned host memory that is valid only
 * for the call; they copy inputs to the index's GPU, run there, and copy results back before
 * returning. "_device" entry points take device pointers on the index's GPU plus a cudaStream_t
 * passed as void* and return once the work is enqueued, without waiting for the GPU: results are
 * ordered like work queued on that stream. NULL means CUDA's default stream (PyTorch's default
 * stream too); the library then runs the work on the calling thread's own stream between two
 * event waits, so it is still ordered after earlier and before later default-stream work (NULL
 * calls from different host threads therefore run on different streams and may overlap).
 * Conditions a _device search can only detect on the GPU do not fail the call: a query holding
 * NaN or infinity gets no results (QV_INVALID_LABEL with a NaN distance) where the host-buffer
 * entry point fails with the reference's error. Index state is read-only during searches, so
 * concurrent searches on one index are safe; add() must not run concurrently with other calls on
 * the same index (the C++ wrapper serializes it with a shared mutex, as the reference does), and
 * with _device searches it must also not start before their GPU work has finished (synchronize
 * their streams first).
 *
 * Distances follow quiver::Metric (include/quiver/common.h:25-29): squared L2, 1 - <q,x> for inner
 * product, 1 - cos for cosine; smaller is closer. Unfilled result slots get label
 * QV_INVALID_LABEL (2^64-1) and distance +inf.
 */
#ifndef QV_GPU_H_
#define QV_GPU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum qv_status {
  QV_OK = 0,
  QV_ERR_INVALID = 1,     /* bad argument: quiver::Error in the reference */
  QV_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  QV_ERR_OOM = 3,         /* device or host allocation failed */
  QV_ERR_IO = 4,          /* file could not be read or written, or is corrupt */
  QV_ERR_STATE = 5,       /* e.g. add() before the index holds trained centroids */
  QV_ERR_UNSUPPORTED = 6, /* outside the GPU path's limits */
  QV_ERR_DEVICE = 7       /* a kernel reported an error through its status word */
} qv_status;

#define QV_INVALID_LABEL UINT64_MAX

enum { QV_METRIC_L2 = 0, QV_METRIC_IP = 1, QV_METRIC_COSINE = 2 };

/* Thread-local text of the last failure on this thread ("" if none). */
const char* qv_last_error(void);
/* Library version string. */
const char* qv_version(void);
/* Number of CUDA devices this process can use. */
qv_status qv_device_count(int* count);

/* ---- filters ----------------------------------------------------------------------------------
 * Replaces quiver::Filter (include/quiver/filter.h:24-102) at the boundary. The binding's
 * make_filter (python/quiver_ext.cc:40-51) builds a BitsetFilter or LabelSetFilter from the allowed
 * labels; here the same information crosses as one of:
 *   QV_FILTER_LABEL_SET:       data = allowed labels (size entries, any order, duplicates allowed)
 *   QV_FILTER_LABEL_BITMAP:    data = BitsetFilter words: label L is admitted iff L < size and
 *                              bit (L & 63) of data[L >> 6] is set
 *   QV_FILTER_POSITION_BITMAP: data = one bit per stored row, in the order qv_flat_rows /
 *                              qv_ivfpq_labels report (how an arbitrary PredicateFilter is passed:
 *                              the caller evaluates contains(label) per stored label)
 * A NULL qv_filter* means no filter. */
enum { QV_FILTER_LABEL_SET = 1, QV_FILTER_LABEL_BITMAP = 2, QV_FILTER_POSITION_BITMAP = 3 };
typedef struct qv_filter {
  uint32_t kind;
  const uint64_t* data;
  uint64_t size;
} qv_filter;

/* ---- FlatIndex --------------------------------------------------------------------------------- */
typedef struct qv_flat qv_flat;

/* FlatIndex(dim, metric): include/quiver/flat_index.h:21 (src/flat_index.cc:41-47). */
qv_status qv_flat_create(int device, size_t dim, uint32_t metric, qv_flat** out);
qv_status qv_flat_destroy(qv_flat* index);
/* add(vectors, n, labels): include/quiver/flat_index.h:25 (src/flat_index.cc:49-67). labels may be
 * NULL (row i gets label size()+i). Cosine rows are normalized on the GPU exactly as
 * simd::normalize does it. */
qv_status qv_flat_add(qv_flat* index, const float* vectors, size_t n, const uint64_t* labels);
/* Large collections (no counterpart in the reference, whose rows live in a growing std::vector):
 * qv_flat_reserve sizes the row storage for n rows at once (an add past the capacity otherwise
 * grows it by half and copies, which needs both copies on the GPU at once), and
 * qv_flat_add_device appends n rows that are already in device memory on the index's GPU
 * (vectors row-major, labels NULL or n device labels), with add()'s checks done on the device,
 * so a collection larger than host memory can be built chunk by chunk. It returns with the rows
 * resident, like add(). */
qv_status qv_flat_reserve(qv_flat* index, size_t n);
qv_status qv_flat_add_device(qv_flat* index, const float* vectors, size_t n,
                             const uint64_t* labels, void* stream);
/* search_batch(queries, nq, k, labels, distances, filter, pool): include/quiver/flat_index.h:34-36
 * (src/flat_index.cc:126-140). Writes nq*k results, closest first. */
qv_status qv_flat_search(const qv_flat* index, const float* queries, size_t nq, size_t k,
                         const qv_filter* filter, uint64_t* labels, float* distances);
/* size(), dim(), metric(): include/quiver/flat_index.h:38-40. */
qv_status qv_flat_info(const qv_flat* index, size_t* size, size_t* dim, uint32_t* metric);
/* vector(i) / label(i) host views: include/quiver/flat_index.h:43-44. Copies rows [first,
 * first+count) as stored (normalized for cosine) and/or their labels; either output may be NULL. */
qv_status qv_flat_rows(const qv_flat* index, size_t first, size_t count, float* vectors,
                       uint64_t* labels);
/* save/load: include/quiver/flat_index.h:46-47 (src/flat_index.cc:147-176), same .qvr format. */
qv_status qv_flat_save(const qv_flat* index, const char* path);
qv_status qv_flat_load(int device, const char* path, int verify_checksums, qv_flat** out);

/* Device-resident search for composing kernels and for multi-GPU sharding. Queries, outputs and
 * the optional position bitmap are device pointers on the index's GPU. keys (may be NULL) receive
 * row_offset + local row of each result, the canonical tie-break key used to merge shards. */
qv_status qv_flat_search_device(const qv_flat* index, const float* queries, size_t nq, size_t k,
                                const uint64_t* position_bitmap, uint64_t* labels, float* distances,
                                uint64_t* keys, void* stream);
/* Global id of this index's row 0 when it is one id-range shard of a larger collection. */
qv_status qv_flat_set_row_offset(qv_flat* index, uint64_t row_offset);

/* Allocation-free variant of qv_flat_search_device. It has no counterpart in the reference; it
 * exists for callers that must not allocate device memory while they search (a serving loop with
 * a fixed device-memory budget, or code running where cudaMalloc/cudaFree are not allowed, e.g.
 * from a driver callback or while another thread holds the allocator). Same arguments and the same
 * results as qv_flat_search_device, queries holding NaN or infinity included (it screens on the
 * CUDA cores and re-ranks and certifies exactly the same way), and it calls no cudaMalloc,
 * cudaFree or other allocating routine: every temporary lives in one fixed scratch array of
 * qv_flat_noalloc_max_bytes() bytes (64 MiB) that each GPU loading the library holds until the
 * process exits. A call whose temporaries would not fit (roughly nq * (dim + n_chunks * KK * 8)
 * bytes) fails with QV_ERR_INVALID; split the queries. It does not feed qv_last_search_stats.
 * The first call on a device looks up the scratch's device address (cudaGetSymbolAddress) and
 * caches it for the life of the process, so make that first call before any stream capture and
 * do not reset that device afterwards. All calls share the scratch and it keeps the last call's
 * contents: calls whose work overlaps on the GPU (different streams, another index on the same
 * device, or NULL-stream calls from different host threads, which run on different streams) race;
 * serialize them by passing one explicit stream, or call from one thread. */
qv_status qv_flat_search_device_noalloc(const qv_flat* index, const float* queries, size_t nq,
                                        size_t k, const uint64_t* position_bitmap,
                                        uint64_t* labels, float* distances, uint64_t* keys,
                                        void* stream);
size_t qv_flat_noalloc_max_bytes(void);

/* ---- HNSW vector storage and its filtered exact scan -------------------------------------------
 * The part of quiver::HnswIndex (include/quiver/hnsw_index.h:53-121) that the GPU serves: the
 * stored vectors (float32, or 8-bit scalar-quantized) and the exact scan HnswIndex::search takes
 * when a filter admits at most exact_scan_threshold of the live vectors (search_exact,
 * src/hnsw_index.cc:723-760). The graph walk stays with the host index. Nodes are numbered in
 * insertion order (HNSW's NodeId). storage: QV_STORAGE_FLOAT32 or QV_STORAGE_SQ8
 * (quiver::Storage, include/quiver/hnsw_index.h:25-28). */
enum { QV_STORAGE_FLOAT32 = 0, QV_STORAGE_SQ8 = 1 };
typedef struct qv_hnsw_store qv_hnsw_store;

/* HnswIndex(params) storage part: include/quiver/hnsw_index.h:55 (src/hnsw_index.cc:791-812). */
qv_status qv_hnsw_store_create(int device, size_t dim, uint32_t metric, uint32_t storage,
                               qv_hnsw_store** out);
qv_status qv_hnsw_store_destroy(qv_hnsw_store* store);
/* train(vectors, n): include/quiver/hnsw_index.h:63 (src/hnsw_index.cc:1018-1028, :541-551,
 * src/scalar_quantizer.cc:9-34): SQ8 only, once; the per-dimension ranges of the prepared
 * (cosine: normalized) vectors, computed on the GPU. */
qv_status qv_hnsw_store_train(qv_hnsw_store* store, const float* vectors, size_t n);
qv_status qv_hnsw_store_is_trained(const qv_hnsw_store* store, int* trained);
/* add(vectors, n, labels) storage part: include/quiver/hnsw_index.h:71-72 (src/hnsw_index.cc:
 * 644-694, :553-564, :582-596): the reference's checks (finite values, the reserved label,
 * duplicates in the call, labels already present and not removed), an untrained SQ8 store trains
 * on a first batch of at least 256 vectors, then each vector is prepared (normalized for cosine)
 * and stored or SQ8-encoded (src/scalar_quantizer.cc:46-52) on the GPU. labels NULL: node i of
 * all ever inserted gets label i. */
qv_status qv_hnsw_store_add(qv_hnsw_store* store, const float* vectors, size_t n,
                            const uint64_t* labels);
/* remove(label): include/quiver/hnsw_index.h:76 (src/hnsw_index.cc:1030-1042): soft delete;
 * *removed = 1 when the label was present and live. */
qv_status qv_hnsw_store_remove(qv_hnsw_store* store, uint64_t label, int* removed);
/* size() (live vectors), number of nodes (removed included), dim(), metric(), storage(). */
qv_status qv_hnsw_store_info(const qv_hnsw_store* store, size_t* live, size_t* nodes, size_t* dim,
                             uint32_t* metric, uint32_t* storage);
/* get_vector(label): include/quiver/hnsw_index.h:79-80: the stored vector (decoded for SQ8,
 * normalized for cosine). */
qv_status qv_hnsw_store_vector(const qv_hnsw_store* store, uint64_t label, float* vector);
/* The stored SQ8 codes of nodes [first, first+count) (dim bytes each), and the trained
 * (vmin, vscale) (dim floats each; either may be NULL). */
qv_status qv_hnsw_store_codes(const qv_hnsw_store* store, size_t first, size_t count,
                              uint8_t* codes);
qv_status qv_hnsw_store_sq8_params(const qv_hnsw_store* store, float* vmin, float* vscale);
/* The exact scan of HnswIndex::search_batch with a filter (src/hnsw_index.cc:723-760, :743-768):
 * for each query (normalized for cosine) the k closest live nodes among those whose label the
 * filter admits, with the storage's distance (l2sqr / 1 - dot, or l2sqr_sq8 / 1 - dot_sq8 for SQ8:
 * the same bits), closest first, unfilled slots QV_INVALID_LABEL / +inf. A NULL filter scans every
 * live node. The label set crosses as in qv_flat_search (QV_FILTER_POSITION_BITMAP: one bit per
 * node). */
qv_status qv_hnsw_store_search(const qv_hnsw_store* store, const float* queries, size_t nq,
                               size_t k, const qv_filter* filter, uint64_t* labels,
                               float* distances);
/* The same with device buffers on the store's GPU; position_bitmap (one bit per node, may be
 * NULL) is read, not modified; node_ids (may be NULL) receive each result's node id (UINT64_MAX
 * when unfilled). It returns after a short host round trip that counts the admitted nodes. */
qv_status qv_hnsw_store_search_device(const qv_hnsw_store* store, const float* queries, size_t nq,
                                      size_t k, const uint64_t* position_bitmap, uint64_t* labels,
                                      float* distances, uint64_t* node_ids, void* stream);

/* ---- IvfPqIndex -------------------------------------------------------------------------------- */
typedef struct qv_ivfpq qv_ivfpq;

/* IvfPqParams: include/quiver/ivfpq_index.h:26-35. */
typedef struct qv_ivfpq_params {
  size_t dim;
  uint32_t metric;
  size_t nlist;
  size_t m;
  size_t train_iterations;
  int store_vectors;
  uint64_t seed;
} qv_ivfpq_params;

/* IvfPqIndex(params): include/quiver/ivfpq_index.h:46 (src/ivfpq_index.cc:95-103). */
qv_status qv_ivfpq_create(int device, const qv_ivfpq_params* params, qv_ivfpq** out);
qv_status qv_ivfpq_destroy(qv_ivfpq* index);
/* train(vectors, n, pool): include/quiver/ivfpq_index.h:53 (src/ivfpq_index.cc:144-206,
 * src/product_quantizer.cc:29-153). The coarse k-means and the PQ sub-space k-means run with their
 * assignment steps on the GPU and the reference's random draws, double-precision cluster sums and
 * empty-cluster splitting on the host, so the centroids and codebooks are bit-identical to the
 * reference's for the same rows and parameters. Trained state can also come from qv_ivfpq_load or
 * qv_ivfpq_set_trained. */
qv_status qv_ivfpq_train(qv_ivfpq* index, const float* vectors, size_t n);
/* Installs trained state (nlist x dim centroids, m x 256 x dsub codebooks), as load() does
 * (src/ivfpq_index.cc:531-543), including the L2 precomputed term table. */
qv_status qv_ivfpq_set_trained(qv_ivfpq* index, const float* centroids, const float* codebooks);
qv_status qv_ivfpq_is_trained(const qv_ivfpq* index, int* trained);
/* add(vectors, n, labels, pool): include/quiver/ivfpq_index.h:57-58 (src/ivfpq_index.cc:208-271):
 * coarse assignment and PQ encode on the GPU, appended per list in input order. */
qv_status qv_ivfpq_add(qv_ivfpq* index, const float* vectors, size_t n, const uint64_t* labels);
/* The assign + encode half of add() without appending: cell ids and m-byte codes per vector,
 * bit-identical to src/ivfpq_index.cc:235-246. */
qv_status qv_ivfpq_encode(const qv_ivfpq* index, const float* vectors, size_t n, uint32_t* assign,
                          uint8_t* codes);
/* search_batch(queries, nq, k, labels, distances, {nprobe, refine_factor, filter}, pool):
 * include/quiver/ivfpq_index.h:62-64 (src/ivfpq_index.cc:421-437, :275-381). */
qv_status qv_ivfpq_search(const qv_ivfpq* index, const float* queries, size_t nq, size_t k,
                          size_t nprobe, size_t refine_factor, const qv_filter* filter,
                          uint64_t* labels, float* distances);
/* size(), memory_bytes(), list_sizes(): include/quiver/ivfpq_index.h:69-75. */
qv_status qv_ivfpq_info(const qv_ivfpq* index, qv_ivfpq_params* params, size_t* size,
                        size_t* memory_bytes);
qv_status qv_ivfpq_list_sizes(const qv_ivfpq* index, uint64_t* sizes /* nlist */);
/* Stored labels in storage (list-major) order; `labels` holds size() entries. */
qv_status qv_ivfpq_labels(const qv_ivfpq* index, uint64_t* labels);
/* save/load: include/quiver/ivfpq_index.h:66-67 (src/ivfpq_index.cc:465-576), same .qvr format.
 * load recomputes the precomputed table as the reference does (:542). */
qv_status qv_ivfpq_save(const qv_ivfpq* index, const char* path);
qv_status qv_ivfpq_load(int device, const char* path, int verify_checksums, qv_ivfpq** out);
/* One id-range shard of a .qvr: keeps the entries whose label lies in [label_begin, label_end)
 * (list order preserved) and remembers each list's global offset so that candidate keys
 * (list << 32 | offset-in-full-list) match the unsharded index. */
qv_status qv_ivfpq_load_shard(int device, const char* path, int verify_checksums,
                              uint64_t label_begin, uint64_t label_end, qv_ivfpq** out);
/* For a shard built by add() instead of load_shard: base[l] (nlist entries) = number of entries
 * of list l held by the shards before this one, so that candidate keys match the unsharded
 * index. No counterpart in the reference (which has no sharding). */
qv_status qv_ivfpq_set_list_base(qv_ivfpq* index, const uint32_t* base);

/* Device-resident stages for composing and for multi-GPU sharding (all pointers on the index's
 * GPU). qv_ivfpq_search_device runs the whole search. qv_ivfpq_candidates_device stops after the
 * ADC scan and returns each query's best `keep` (distance, key, label), sorted, padded with
 * (+inf, UINT64_MAX, QV_INVALID_LABEL); keys are list << 32 | offset-in-full-list.
 * qv_ivfpq_refine_device writes the exact distance of every candidate this index stores and +inf
 * for the others (keys not held here), so shards' outputs can be min-reduced. */
qv_status qv_ivfpq_search_device(const qv_ivfpq* index, const float* queries, size_t nq, size_t k,
                                 size_t nprobe, size_t refine_factor,
                                 const uint64_t* position_bitmap, uint64_t* labels,
                                 float* distances, void* stream);
qv_status qv_ivfpq_candidates_device(const qv_ivfpq* index, const float* queries, size_t nq,
                                     size_t keep, size_t nprobe, const uint64_t* position_bitmap,
                                     float* distances, uint64_t* keys, uint64_t* labels,
                                     void* stream);
qv_status qv_ivfpq_refine_device(const qv_ivfpq* index, const float* queries, size_t nq,
                                 size_t keep, const uint64_t* keys, float* exact, void* stream);
/* Builds the per-position bitmap a _device search takes from a host filter (uploaded once). The
 * bitmap is allocated on the index's GPU; release it with qv_device_free. */
qv_status qv_flat_filter_bitmap(const qv_flat* index, const qv_filter* filter,
                                uint64_t** device_bitmap);
qv_status qv_ivfpq_filter_bitmap(const qv_ivfpq* index, const qv_filter* filter,
                                 uint64_t** device_bitmap);
qv_status qv_device_free(int device, void* ptr);

/* ---- shard merge ---------------------------------------------------------------------------------
 * k-way merge of per-shard results: parts x nq x k (distance, key, label) triples, each row sorted
 * by (distance, key), into nq x k sorted by (distance, key). Device pointers on `device`. Replaces
 * nothing in the reference (which has no sharding); it is the final step of a sharded search. */
qv_status qv_merge_topk_device(int device, size_t parts, size_t nq, size_t k,
                               const float* distances, const uint64_t* keys,
                               const uint64_t* labels, float* out_distances, uint64_t* out_keys,
                               uint64_t* out_labels, void* stream);
/* Per-row top-k of candidate lists: nq x n (distance, key, label) -> nq x k sorted by
 * (distance, key). Used after min-reducing shard refine outputs. */
qv_status qv_select_topk_device(int device, size_t nq, size_t n, size_t k, const float* distances,
                                const uint64_t* keys, const uint64_t* labels,
                                float* out_distances, uint64_t* out_keys, uint64_t* out_labels,
                                void* stream);

/* Counters of the calling thread's searches (for the bench and tests): kernel launches issued,
 * queries whose screen could not be certified and were rescanned exactly, and, when timing is
 * enabled, the device time of the searches' dominant kernel (CUDA events recorded on the stream
 * it runs on), its name and its algorithmic work (FLOPs for the distance screen, bytes for scans)
 * so callers can compute a roofline fraction. With timing disabled they describe the last search;
 * with timing enabled they accumulate over every search since timing was enabled or since the
 * previous call, which resolves the recorded events (waiting for them) and starts again. The
 * rescan count of a _device Flat search is read after waiting for that search to finish. */
typedef struct qv_search_stats {
  uint64_t kernel_launches;
  uint64_t rescanned_queries;
  double dominant_kernel_ms;
  double dominant_kernel_work;
  uint32_t dominant_work_is_bytes;
  char dominant_kernel[64];
} qv_search_stats;
qv_status qv_last_search_stats(qv_search_stats* stats);
/* Enables (1) or disables (0) the per-search kernel timing above for the calling thread. */
qv_status qv_set_timing(int enable);

#ifdef __cplusplus
}
#endif
#endif /* QV_GPU_H_ */
