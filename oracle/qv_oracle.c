/* Test infrastructure only (see qv_oracle.h): a CPU restatement of the reference's hot path.
 * Every function names the reference file:line it restates (paths relative to the reference
 * project root). Compiled with -ffp-contract=off so each '*' and '+' rounds separately; fmaf()
 * appears only where the reference uses an FMA intrinsic.
 *
 * Ties: the reference's bounded heaps leave the order of equal distances unspecified
 * (src/flat_index.cc:89-95, src/ivfpq_index.cc:348-358). This restatement breaks them
 * canonically by (distance, row id) for Flat and (distance, list<<32 | offset) for IVF-PQ.
 */
#include "qv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define KS 256

/* ---- reductions: src/simd/kernels_scalar.cc:7-22 and src/simd/kernels_avx2.cc:17-83 ---------- */

/* hsum of an 8-lane vector, src/simd/kernels_avx2.cc:17-23: lanes l and l+4 are added first, then
 * (l0+l1) + (l2+l3). */
static float hsum8(const float v[8]) {
  float lo[4];
  for (int l = 0; l < 4; ++l) lo[l] = v[l] + v[l + 4];
  return (lo[0] + lo[1]) + (lo[2] + lo[3]);
}

/* Tail of dot_avx2/l2sqr_avx2 from element i: x[j] holds a[j]*b[j]'s factors (diff=0) or the
 * differences (diff=1). */
static float tail_products(const float* a, const float* b, size_t i, size_t dim, float sum,
                           int diff) {
  size_t j = i;
  if (dim - i >= 4) {
    for (; j < i + 4; ++j) {
      const float u = diff ? a[j] - b[j] : a[j];
      const float v = diff ? u : b[j];
      sum = sum + u * v;
    }
  }
  for (; j < dim; ++j) {
    const float u = diff ? a[j] - b[j] : a[j];
    const float v = diff ? u : b[j];
    sum = fmaf(u, v, sum);
  }
  return sum;
}

/* src/simd/kernels_avx2.cc:63-83: four 8-lane FMA accumulators over 32-element blocks, then
 * 8-element blocks into the first, lane-wise (s0+s1)+(s2+s3), hsum, then the scalar tail.
 *
 * The tail (dim % 8 elements) is what GCC 13 makes of `sum += a[i] * b[i]` in a function with
 * target("avx2,fma") under the reference's flags (-O3, GCC's default -ffp-contract=fast): when 4
 * or more elements remain, the first 4 products are formed by one vector multiply (rounded) and
 * added to the sum in order; every remaining element is one FMA. tail_products() restates that;
 * it was checked bit for bit against the compiled reference for every dim in 1..79. */
static float dot_avx2(const float* a, const float* b, size_t dim) {
  float s[4][8];
  memset(s, 0, sizeof(s));
  size_t i = 0;
  for (; i + 32 <= dim; i += 32)
    for (int r = 0; r < 4; ++r)
      for (int l = 0; l < 8; ++l) s[r][l] = fmaf(a[i + 8 * r + l], b[i + 8 * r + l], s[r][l]);
  for (; i + 8 <= dim; i += 8)
    for (int l = 0; l < 8; ++l) s[0][l] = fmaf(a[i + l], b[i + l], s[0][l]);
  float t[8];
  for (int l = 0; l < 8; ++l) t[l] = (s[0][l] + s[1][l]) + (s[2][l] + s[3][l]);
  return tail_products(a, b, i, dim, hsum8(t), 0);
}

/* src/simd/kernels_avx2.cc:35-61: as dot_avx2 on the differences a-b, tail included. */
static float l2sqr_avx2(const float* a, const float* b, size_t dim) {
  float s[4][8];
  memset(s, 0, sizeof(s));
  size_t i = 0;
  for (; i + 32 <= dim; i += 32)
    for (int r = 0; r < 4; ++r)
      for (int l = 0; l < 8; ++l) {
        const float d = a[i + 8 * r + l] - b[i + 8 * r + l];
        s[r][l] = fmaf(d, d, s[r][l]);
      }
  for (; i + 8 <= dim; i += 8)
    for (int l = 0; l < 8; ++l) {
      const float d = a[i + l] - b[i + l];
      s[0][l] = fmaf(d, d, s[0][l]);
    }
  float t[8];
  for (int l = 0; l < 8; ++l) t[l] = (s[0][l] + s[1][l]) + (s[2][l] + s[3][l]);
  return tail_products(a, b, i, dim, hsum8(t), 1);
}

float qvo_dot(const float* a, const float* b, size_t dim, int order) {
  if (order == 2) return dot_avx2(a, b, dim);
  float sum = 0.0f; /* src/simd/kernels_scalar.cc:16-22 */
  for (size_t i = 0; i < dim; ++i) sum += a[i] * b[i];
  return sum;
}

float qvo_l2sqr(const float* a, const float* b, size_t dim, int order) {
  if (order == 2) return l2sqr_avx2(a, b, dim);
  float sum = 0.0f; /* src/simd/kernels_scalar.cc:7-14 */
  for (size_t i = 0; i < dim; ++i) {
    const float d = a[i] - b[i];
    sum += d * d;
  }
  return sum;
}

/* src/simd/dispatch.cc:119-135 */
static void normalize(float* v, size_t dim, int order) {
  const float norm_sq = qvo_dot(v, v, dim, order);
  if (!isfinite(norm_sq)) {
    double acc = 0.0;
    for (size_t i = 0; i < dim; ++i) acc += (double)v[i] * (double)v[i];
    const double inv = acc > 0.0 && isfinite(acc) ? 1.0 / sqrt(acc) : 0.0;
    if (inv == 0.0) return;
    for (size_t i = 0; i < dim; ++i) v[i] = (float)((double)v[i] * inv);
    return;
  }
  if (norm_sq <= 0.0f) return;
  const float inv = 1.0f / sqrtf(norm_sq);
  for (size_t i = 0; i < dim; ++i) v[i] *= inv;
}

void qvo_normalize_rows(float* v, size_t n, size_t dim, int order) {
  for (size_t i = 0; i < n; ++i) normalize(v + i * dim, dim, order);
}

/* ---- bounded top-k with a canonical (distance, id) order -------------------------------------- */

typedef struct {
  float d;
  uint64_t id;
} cand;

static int worse(cand a, cand b) { return a.d > b.d || (a.d == b.d && a.id > b.id); }

typedef struct {
  cand* h;
  size_t n, cap;
} topk;

static void topk_push(topk* t, cand c) {
  if (t->cap == 0) return;
  if (t->n == t->cap) {
    if (!worse(t->h[0], c)) return;
    size_t i = 0; /* replace the root and sift down (max-heap on worse()) */
    for (;;) {
      size_t l = 2 * i + 1, r = l + 1, w = i;
      cand cw = c;
      if (l < t->n && worse(t->h[l], cw)) { w = l; cw = t->h[l]; }
      if (r < t->n && worse(t->h[r], cw)) { w = r; cw = t->h[r]; }
      if (w == i) break;
      t->h[i] = t->h[w];
      i = w;
    }
    t->h[i] = c;
    return;
  }
  size_t i = t->n++;
  while (i > 0) {
    size_t p = (i - 1) / 2;
    if (!worse(c, t->h[p])) break;
    t->h[i] = t->h[p];
    i = p;
  }
  t->h[i] = c;
}

static int cand_cmp(const void* x, const void* y) {
  const cand a = *(const cand*)x, b = *(const cand*)y;
  if (worse(a, b)) return 1;
  if (worse(b, a)) return -1;
  return 0;
}

static int admitted(const uint64_t* bitmap, uint64_t universe, uint64_t label) {
  if (bitmap == NULL) return 1;
  return label < universe && ((bitmap[label >> 6] >> (label & 63)) & 1u) != 0;
}

/* ---- FlatIndex: src/flat_index.cc:69-107 (search_one) and :126-140 (search_batch) ------------- */

int qvo_flat_search(const float* base, const uint64_t* labels, size_t n, size_t dim, int metric,
                    int order, const float* queries, size_t nq, size_t k, const uint64_t* bitmap,
                    uint64_t universe, uint64_t* out_labels, float* out_dists) {
  if (nq == 0 || k == 0) return 0;
  float* q = (float*)malloc(dim * sizeof(float));
  cand* heap = (cand*)malloc((k < n ? k : n) * sizeof(cand) + sizeof(cand));
  if (!q || !heap) { free(q); free(heap); return -1; }
  for (size_t qi = 0; qi < nq; ++qi) {
    memcpy(q, queries + qi * dim, dim * sizeof(float));
    if (metric == 2) normalize(q, dim, order); /* :74-78 */
    topk t = {heap, 0, k < n ? k : n};
    for (size_t i = 0; i < n; ++i) {
      if (!admitted(bitmap, universe, labels[i])) continue; /* :85 */
      const float* x = base + i * dim;
      float d = metric == 0 ? qvo_l2sqr(q, x, dim, order) : 1.0f - qvo_dot(q, x, dim, order);
      if (d != d) d = INFINITY; /* :88 */
      cand c = {d, i};
      topk_push(&t, c);
    }
    qsort(t.h, t.n, sizeof(cand), cand_cmp); /* :97 sort_heap */
    for (size_t j = 0; j < k; ++j) { /* :98-106 */
      if (j < t.n) {
        out_labels[qi * k + j] = labels[t.h[j].id];
        out_dists[qi * k + j] = t.h[j].d;
      } else {
        out_labels[qi * k + j] = UINT64_MAX;
        out_dists[qi * k + j] = INFINITY;
      }
    }
  }
  free(q);
  free(heap);
  return 0;
}

/* ---- SQ8 storage and HNSW's filtered exact scan ------------------------------------------------
 * src/scalar_quantizer.cc (train/encode/decode), src/simd/kernels_avx2.cc:25-31 (sq8_decode8),
 * :85-129 (l2sqr_sq8, dot_sq8), src/hnsw_index.cc:541-551 (train on prepared vectors),
 * :553-564 (init_node stores or encodes the prepared vector), :723-741 (search_exact). */

/* One decoded component, vmin + code * vscale as one FMA (sq8_decode8's _mm256_fmadd_ps; GCC also
 * contracts the scalar tail's decode into an FMA under the reference's flags). */
static float sq8_dec(uint8_t c, float vmin, float vscale) { return fmaf((float)c, vscale, vmin); }

/* src/simd/kernels_avx2.cc:85-106: two 8-lane FMA accumulators over 16-element blocks, then
 * 8-element blocks into the first, lane-wise s0+s1, hsum, then the scalar tail, every element of
 * which is (decode FMA, subtract, FMA into the sum): checked bit for bit against the compiled
 * reference for every dim in 1..200. */
float qvo_l2sqr_sq8(const float* q, const uint8_t* code, const float* vmin, const float* vscale,
                    size_t dim) {
  float s0[8], s1[8];
  memset(s0, 0, sizeof(s0));
  memset(s1, 0, sizeof(s1));
  size_t i = 0;
  for (; i + 16 <= dim; i += 16)
    for (int l = 0; l < 8; ++l) {
      const float d0 = q[i + l] - sq8_dec(code[i + l], vmin[i + l], vscale[i + l]);
      const float d1 = q[i + 8 + l] - sq8_dec(code[i + 8 + l], vmin[i + 8 + l], vscale[i + 8 + l]);
      s0[l] = fmaf(d0, d0, s0[l]);
      s1[l] = fmaf(d1, d1, s1[l]);
    }
  for (; i + 8 <= dim; i += 8)
    for (int l = 0; l < 8; ++l) {
      const float d0 = q[i + l] - sq8_dec(code[i + l], vmin[i + l], vscale[i + l]);
      s0[l] = fmaf(d0, d0, s0[l]);
    }
  float t[8];
  for (int l = 0; l < 8; ++l) t[l] = s0[l] + s1[l];
  float sum = hsum8(t);
  for (; i < dim; ++i) {
    const float d = q[i] - sq8_dec(code[i], vmin[i], vscale[i]);
    sum = fmaf(d, d, sum);
  }
  return sum;
}

/* src/simd/kernels_avx2.cc:108-129, the same structure with q * decoded products. */
float qvo_dot_sq8(const float* q, const uint8_t* code, const float* vmin, const float* vscale,
                  size_t dim) {
  float s0[8], s1[8];
  memset(s0, 0, sizeof(s0));
  memset(s1, 0, sizeof(s1));
  size_t i = 0;
  for (; i + 16 <= dim; i += 16)
    for (int l = 0; l < 8; ++l) {
      s0[l] = fmaf(q[i + l], sq8_dec(code[i + l], vmin[i + l], vscale[i + l]), s0[l]);
      s1[l] = fmaf(q[i + 8 + l], sq8_dec(code[i + 8 + l], vmin[i + 8 + l], vscale[i + 8 + l]),
                   s1[l]);
    }
  for (; i + 8 <= dim; i += 8)
    for (int l = 0; l < 8; ++l)
      s0[l] = fmaf(q[i + l], sq8_dec(code[i + l], vmin[i + l], vscale[i + l]), s0[l]);
  float t[8];
  for (int l = 0; l < 8; ++l) t[l] = s0[l] + s1[l];
  float sum = hsum8(t);
  for (; i < dim; ++i) sum = fmaf(q[i], sq8_dec(code[i], vmin[i], vscale[i]), sum);
  return sum;
}

/* src/scalar_quantizer.cc:9-34: per-dimension [min, max]; scale = range / 255 (1 for a constant
 * dimension). Returns -1 when the data holds NaN or infinity (the reference throws). */
int qvo_sq8_train(const float* x, size_t n, size_t dim, float* vmin, float* vscale) {
  int finite = 1;
  for (size_t j = 0; j < dim; ++j) {
    vmin[j] = INFINITY;
    vscale[j] = -INFINITY; /* holds the maximum until the end */
  }
  for (size_t i = 0; i < n; ++i)
    for (size_t j = 0; j < dim; ++j) {
      const float v = x[i * dim + j];
      finite &= isfinite(v) != 0;
      if (v < vmin[j]) vmin[j] = v; /* std::min(lo, v) */
      if (vscale[j] < v) vscale[j] = v; /* std::max(hi, v) */
    }
  if (!finite) return -1;
  for (size_t j = 0; j < dim; ++j) {
    const float range = vscale[j] - vmin[j];
    if (!isfinite(range)) return -1;
    vscale[j] = range > 0.0f ? range / 255.0f : 1.0f;
  }
  return 0;
}

/* src/scalar_quantizer.cc:46-52: round-to-nearest-even of (v - vmin) / vscale, clamped to 0..255
 * (NaN lands on 0). */
void qvo_sq8_encode(const float* vmin, const float* vscale, size_t dim, const float* x, size_t n,
                    uint8_t* codes) {
  for (size_t i = 0; i < n; ++i)
    for (size_t j = 0; j < dim; ++j) {
      const float t = nearbyintf((x[i * dim + j] - vmin[j]) / vscale[j]);
      codes[i * dim + j] = (uint8_t)(t >= 255.0f ? 255.0f : (t > 0.0f ? t : 0.0f));
    }
}

/* src/hnsw_index.cc:723-741 (search_exact) with FloatSpace / Sq8Space distances (:179-233): for
 * each query (normalized first for cosine, :334-339), every listed node's distance (l2sqr, or
 * 1 - dot for inner product and cosine; NaN -> +inf), the k best kept and sorted ascending,
 * unfilled slots (UINT32_MAX, +inf). storage: 0 float32 rows (data = n x dim floats), 1 SQ8
 * codes (data = n x dim bytes, vmin / vscale per dimension). out_ids are node ids. */
int qvo_exact_scan(int storage, const void* data, const float* vmin, const float* vscale,
                   size_t dim, int metric, const uint32_t* ids, size_t n_ids,
                   const float* queries, size_t nq, size_t k, uint32_t* out_ids,
                   float* out_dists) {
  if (nq == 0 || k == 0) return 0;
  float* q = (float*)malloc(dim * sizeof(float));
  cand* heap = (cand*)malloc((k < n_ids ? k : n_ids) * sizeof(cand) + sizeof(cand));
  if (!q || !heap) { free(q); free(heap); return -1; }
  for (size_t qi = 0; qi < nq; ++qi) {
    memcpy(q, queries + qi * dim, dim * sizeof(float));
    if (metric == 2) normalize(q, dim, 2);
    topk t = {heap, 0, k < n_ids ? k : n_ids};
    for (size_t i = 0; i < n_ids; ++i) {
      const size_t id = ids[i];
      float d;
      if (storage == 0) {
        const float* x = (const float*)data + id * dim;
        d = metric == 0 ? qvo_l2sqr(q, x, dim, 2) : 1.0f - qvo_dot(q, x, dim, 2);
      } else {
        const uint8_t* c = (const uint8_t*)data + id * dim;
        d = metric == 0 ? qvo_l2sqr_sq8(q, c, vmin, vscale, dim)
                        : 1.0f - qvo_dot_sq8(q, c, vmin, vscale, dim);
      }
      if (d != d) d = INFINITY;
      cand c = {d, id};
      topk_push(&t, c);
    }
    qsort(t.h, t.n, sizeof(cand), cand_cmp);
    for (size_t j = 0; j < k; ++j) {
      out_ids[qi * k + j] = j < t.n ? (uint32_t)t.h[j].id : UINT32_MAX;
      out_dists[qi * k + j] = j < t.n ? t.h[j].d : INFINITY;
    }
  }
  free(q);
  free(heap);
  return 0;
}

/* ---- CentroidTable: src/internal/centroid_table.h:43-59 (reset), :65-75 (l2), :78-85 (dot),
 *      :94-144 (nearest_batch), :155-170 (argmin_n) -------------------------------------------- */

void qvo_centroid_norms(const float* cents, size_t k, size_t dim, float* norms) {
  for (size_t c = 0; c < k; ++c) {
    float norm = 0.0f;
    for (size_t j = 0; j < dim; ++j) norm += cents[c * dim + j] * cents[c * dim + j];
    norms[c] = norm;
  }
}

/* nearest_batch: d = ||c||^2 - 2<x,c> (or -<x,c> for max inner product), <x,c> summed over j in
 * ascending order from 0 with separately rounded products; the first strict minimum wins. */
void qvo_coarse_assign(const float* cents, size_t nlist, size_t dim, const float* x, size_t n,
                       int by_ip, uint32_t* out) {
  float* norms = (float*)malloc(nlist * sizeof(float));
  qvo_centroid_norms(cents, nlist, dim, norms);
  for (size_t p = 0; p < n; ++p) {
    const float* v = x + p * dim;
    float best_d = INFINITY;
    uint32_t best = 0;
    for (size_t c = 0; c < nlist; ++c) {
      float dot = 0.0f;
      for (size_t j = 0; j < dim; ++j) dot += v[j] * cents[c * dim + j];
      const float d = by_ip ? -dot : norms[c] - 2.0f * dot;
      if (d < best_d) {
        best_d = d;
        best = (uint32_t)c;
      }
    }
    out[p] = best;
  }
  free(norms);
}

/* src/product_quantizer.cc:165-171 with CentroidTable::l2 and argmin_n: per sub-space the code is
 * the first index attaining the minimum of sum_t (r_t - cb_t)^2 (t ascending, from 0). */
void qvo_pq_encode(const float* codebooks, size_t m, size_t dsub, const float* x, size_t n,
                   uint8_t* codes) {
  float dist[KS];
  for (size_t i = 0; i < n; ++i) {
    const float* v = x + i * m * dsub;
    for (size_t j = 0; j < m; ++j) {
      const float* cb = codebooks + j * KS * dsub;
      const float* r = v + j * dsub;
      for (size_t c = 0; c < KS; ++c) {
        float s = 0.0f;
        for (size_t t = 0; t < dsub; ++t) {
          const float d = r[t] - cb[c * dsub + t];
          s += d * d;
        }
        dist[c] = s;
      }
      float mn = INFINITY;
      for (size_t c = 0; c < KS; ++c) mn = dist[c] < mn ? dist[c] : mn;
      size_t code = 0;
      for (size_t c = 0; c < KS; ++c)
        if (dist[c] == mn) { code = c; break; }
      codes[i * m + j] = (uint8_t)code;
    }
  }
}

/* src/ivfpq_index.cc:208-246 (Impl::add): normalize for cosine, assign the cell (by inner product
 * only for kInnerProduct, :107), residual v - c (:243), PQ-encode the residual. */
void qvo_ivf_encode(const float* cents, size_t nlist, const float* codebooks, size_t m,
                    size_t dim, int metric, int order, const float* x, size_t n,
                    uint32_t* assign, uint8_t* codes) {
  float* v = (float*)malloc(dim * sizeof(float));
  float* r = (float*)malloc(dim * sizeof(float));
  for (size_t i = 0; i < n; ++i) {
    memcpy(v, x + i * dim, dim * sizeof(float));
    if (metric == 2) normalize(v, dim, order);
    qvo_coarse_assign(cents, nlist, dim, v, 1, metric == 1, &assign[i]);
    const float* c = cents + (size_t)assign[i] * dim;
    for (size_t j = 0; j < dim; ++j) r[j] = v[j] - c[j];
    qvo_pq_encode(codebooks, m, dim / m, r, 1, codes + i * m);
  }
  free(v);
  free(r);
}

/* src/ivfpq_index.cc:112-129 (Impl::precompute): v += r*r + 2*c*r over t ascending. */
void qvo_precompute(const float* cents, size_t nlist, const float* codebooks, size_t m,
                    size_t dsub, float* pre) {
  const size_t dim = m * dsub;
  for (size_t l = 0; l < nlist; ++l)
    for (size_t j = 0; j < m; ++j) {
      const float* cl = cents + l * dim + j * dsub;
      for (size_t c = 0; c < KS; ++c) {
        const float* r = codebooks + (j * KS + c) * dsub;
        float v = 0.0f;
        for (size_t t = 0; t < dsub; ++t) v += r[t] * r[t] + 2.0f * cl[t] * r[t];
        pre[(l * m + j) * KS + c] = v;
      }
    }
}

/* src/product_quantizer.cc:184-186 with CentroidTable::dot. */
void qvo_ip_table(const float* codebooks, size_t m, size_t dsub, const float* q, float* table) {
  for (size_t j = 0; j < m; ++j)
    for (size_t c = 0; c < KS; ++c) {
      float s = 0.0f;
      for (size_t t = 0; t < dsub; ++t) s += q[j * dsub + t] * codebooks[(j * KS + c) * dsub + t];
      table[j * KS + c] = s;
    }
}

/* src/product_quantizer.cc:180-182 with CentroidTable::l2. */
void qvo_l2_table(const float* codebooks, size_t m, size_t dsub, const float* q, float* table) {
  for (size_t j = 0; j < m; ++j)
    for (size_t c = 0; c < KS; ++c) {
      float s = 0.0f;
      for (size_t t = 0; t < dsub; ++t) {
        const float d = q[j * dsub + t] - codebooks[(j * KS + c) * dsub + t];
        s += d * d;
      }
      table[j * KS + c] = s;
    }
}

/* ---- IvfPqIndex::Impl::search_into: src/ivfpq_index.cc:275-381 -------------------------------- */

int qvo_ivf_search(const qvo_ivf_index* ix, const float* queries, size_t nq, size_t k,
                   size_t nprobe_req, size_t refine_factor, const uint64_t* bitmap,
                   uint64_t universe, int order, uint64_t* out_labels, float* out_dists) {
  const size_t d = ix->dim, nlist = ix->nlist, m = ix->m, dsub = d / m;
  const int ip = ix->metric != 0;
  const size_t count = (size_t)ix->offsets[nlist];
  for (size_t i = 0; i < nq * k; ++i) { /* :277-278 */
    out_labels[i] = UINT64_MAX;
    out_dists[i] = INFINITY;
  }
  if (k == 0) return 0;
  size_t nprobe = nprobe_req < 1 ? 1 : nprobe_req; /* :286 */
  if (nprobe > nlist) nprobe = nlist;
  const int refine = refine_factor > 0 && ix->vectors != NULL; /* :303-307 */
  const size_t factor = refine ? refine_factor : 1;
  size_t keep = factor > count / (k > 1 ? k : 1) ? count : k * factor;
  if (keep > count) keep = count;
  if (keep == 0) return 0; /* :308 */

  float* q = (float*)malloc(d * sizeof(float));
  cand* probes = (cand*)malloc(nlist * sizeof(cand));
  float* table = (float*)malloc(m * KS * sizeof(float));
  float* qtable = (float*)malloc(m * KS * sizeof(float));
  float* resid = (float*)malloc(d * sizeof(float));
  cand* heap = (cand*)malloc(keep * sizeof(cand));
  if (!q || !probes || !table || !qtable || !resid || !heap) return -1;

  for (size_t qi = 0; qi < nq; ++qi) {
    memcpy(q, queries + qi * d, d * sizeof(float));
    if (ix->metric == 2) normalize(q, d, order); /* :283, :131-136 */
    /* :285-300, coarse probe with CentroidTable::l2 / ::dot, j ascending from 0. */
    for (size_t l = 0; l < nlist; ++l) {
      const float* c = ix->centroids + l * d;
      float s = 0.0f;
      if (ip) {
        for (size_t j = 0; j < d; ++j) s += q[j] * c[j];
        s = -s;
      } else {
        for (size_t j = 0; j < d; ++j) {
          const float t = q[j] - c[j];
          s += t * t;
        }
      }
      probes[l].d = s;
      probes[l].id = l;
    }
    qsort(probes, nlist, sizeof(cand), cand_cmp); /* partial_sort, ties by list id */

    /* :309-318 */
    const int use_pre = ix->precomputed != NULL;
    if (ip) {
      qvo_ip_table(ix->codebooks, m, dsub, q, table);
    } else if (use_pre) {
      qvo_ip_table(ix->codebooks, m, dsub, q, qtable);
      for (size_t t = 0; t < m * KS; ++t) qtable[t] *= -2.0f;
    }
    topk t = {heap, 0, keep};
    for (size_t pi = 0; pi < nprobe; ++pi) { /* :326-360 */
      const size_t l = (size_t)probes[pi].id;
      const size_t b = (size_t)ix->offsets[l], e = (size_t)ix->offsets[l + 1];
      if (e == b) continue;
      float base = 0.0f;
      if (ip) {
        base = -probes[pi].d;
      } else if (use_pre) {
        base = probes[pi].d;
        const float* pre = ix->precomputed + l * m * KS;
        for (size_t u = 0; u < m * KS; ++u) table[u] = pre[u] + qtable[u];
      } else {
        const float* c = ix->centroids + l * d;
        for (size_t j = 0; j < d; ++j) resid[j] = q[j] - c[j];
        qvo_l2_table(ix->codebooks, m, dsub, resid, table);
      }
      for (size_t i = b; i < e; ++i) {
        const uint8_t* code = ix->codes + i * m;
        float s = 0.0f; /* src/product_quantizer.cc:188-217 */
        for (size_t j = 0; j < m; ++j) s += table[j * KS + code[j]];
        float dist = ip ? 1.0f - (base + s) : base + s;
        if (dist != dist) dist = INFINITY;
        if (!admitted(bitmap, universe, ix->labels[i])) continue;
        cand c = {dist, ((uint64_t)l << 32) | (uint64_t)(i - b)};
        topk_push(&t, c);
      }
    }
    size_t nres = t.n;
    if (refine) { /* :362-373 */
      for (size_t u = 0; u < t.n; ++u) {
        const size_t l = (size_t)(t.h[u].id >> 32), off = (size_t)(t.h[u].id & 0xffffffffu);
        const float* x = ix->vectors + ((size_t)ix->offsets[l] + off) * d;
        t.h[u].d = ip ? 1.0f - qvo_dot(q, x, d, order) : qvo_l2sqr(q, x, d, order);
      }
    }
    qsort(t.h, t.n, sizeof(cand), cand_cmp);
    if (nres > k) nres = k;
    for (size_t j = 0; j < nres; ++j) { /* :374-380 */
      const size_t l = (size_t)(t.h[j].id >> 32), off = (size_t)(t.h[j].id & 0xffffffffu);
      out_labels[qi * k + j] = ix->labels[(size_t)ix->offsets[l] + off];
      out_dists[qi * k + j] = t.h[j].d;
    }
  }
  free(q);
  free(probes);
  free(table);
  free(qtable);
  free(resid);
  free(heap);
  return 0;
}
