/* Test infrastructure only: a plain-C restatement of the reference Quiver nearest-neighbour hot
 * path, used by tests/ and bench.py's CPU-baseline leg to check the CUDA library. Nothing in the
 * product links or calls it.
 *
 * Metric codes follow quiver::Metric (include/quiver/common.h:29 of the reference):
 *   0 = L2 (squared), 1 = inner product (1 - <q,x>), 2 = cosine (1 - cos).
 * Reduction-order codes select which reference kernel a float reduction follows:
 *   0 = the portable scalar loop (src/simd/kernels_scalar.cc),
 *   2 = the AVX2 kernel (src/simd/kernels_avx2.cc), the one the reference picks on x86-64 hosts.
 * Filters are dense bitmaps over labels with BitsetFilter semantics (include/quiver/filter.h:39-71):
 * label L is admitted iff L < universe and bit (L & 63) of word (L >> 6) is set.
 */
#ifndef QV_ORACLE_H_
#define QV_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float qvo_dot(const float* a, const float* b, size_t dim, int order);
float qvo_l2sqr(const float* a, const float* b, size_t dim, int order);
void qvo_normalize_rows(float* v, size_t n, size_t dim, int order);

int qvo_flat_search(const float* base, const uint64_t* labels, size_t n, size_t dim, int metric,
                    int order, const float* queries, size_t nq, size_t k, const uint64_t* bitmap,
                    uint64_t universe, uint64_t* out_labels, float* out_dists);

float qvo_l2sqr_sq8(const float* q, const uint8_t* code, const float* vmin, const float* vscale,
                    size_t dim);
float qvo_dot_sq8(const float* q, const uint8_t* code, const float* vmin, const float* vscale,
                  size_t dim);
int qvo_sq8_train(const float* x, size_t n, size_t dim, float* vmin, float* vscale);
void qvo_sq8_encode(const float* vmin, const float* vscale, size_t dim, const float* x, size_t n,
                    uint8_t* codes);
int qvo_exact_scan(int storage, const void* data, const float* vmin, const float* vscale,
                   size_t dim, int metric, const uint32_t* ids, size_t n_ids,
                   const float* queries, size_t nq, size_t k, uint32_t* out_ids,
                   float* out_dists);

void qvo_centroid_norms(const float* cents, size_t k, size_t dim, float* norms);
void qvo_coarse_assign(const float* cents, size_t nlist, size_t dim, const float* x, size_t n,
                       int by_ip, uint32_t* out);
void qvo_pq_encode(const float* codebooks, size_t m, size_t dsub, const float* x, size_t n,
                   uint8_t* codes);
void qvo_ivf_encode(const float* cents, size_t nlist, const float* codebooks, size_t m,
                    size_t dim, int metric, int order, const float* x, size_t n,
                    uint32_t* assign, uint8_t* codes);
void qvo_precompute(const float* cents, size_t nlist, const float* codebooks, size_t m,
                    size_t dsub, float* pre);
void qvo_ip_table(const float* codebooks, size_t m, size_t dsub, const float* q, float* table);
void qvo_l2_table(const float* codebooks, size_t m, size_t dsub, const float* q, float* table);

typedef struct {
  size_t dim, nlist, m;
  int metric;
  const float* centroids;   /* nlist x dim */
  const float* codebooks;   /* m x 256 x dsub */
  const uint64_t* offsets;  /* nlist + 1, list-major */
  const uint8_t* codes;     /* count x m */
  const uint64_t* labels;   /* count */
  const float* vectors;     /* count x dim, or NULL when vectors are not stored */
  const float* precomputed; /* nlist x m x 256, or NULL when the reference would not build it */
} qvo_ivf_index;

int qvo_ivf_search(const qvo_ivf_index* ix, const float* queries, size_t nq, size_t k,
                   size_t nprobe, size_t refine_factor, const uint64_t* bitmap, uint64_t universe,
                   int order, uint64_t* out_labels, float* out_dists);

#ifdef __cplusplus
}
#endif
#endif
