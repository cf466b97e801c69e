/* Test infrastructure, not product code: the CPU checker for the GPU search path.
 *
 * A plain-C restatement of vdb's search algorithms (KoduruChandrasekhar/HNSW-Vector-DB). Each
 * function names the reference file:line it follows. Built with -ffp-contract=off so that every
 * float operation happens exactly as written; fmaf() is used only where the reference's SIMD
 * kernels issue a fused multiply-add.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ distance kernels */

/* _mm512_reduce_add_ps as GCC implements it (avx512fintrin.h __MM512_REDUCE_OP): add the upper
 * 8 lanes onto the lower 8, then the upper 4 onto the lower 4, then lanes {2,3} onto {0,1},
 * then lane 1 onto lane 0. */
static float reduce16(const float s[16]) {
  float t3[8], t6[4];
  for (int i = 0; i < 8; ++i) t3[i] = s[8 + i] + s[i];
  for (int i = 0; i < 4; ++i) t6[i] = t3[4 + i] + t3[i];
  float t8_0 = t6[0] + t6[2], t8_1 = t6[1] + t6[3];
  return t8_0 + t8_1;
}

/* HorizontalSum of src/distance/avx2.cc:12-17: (v[j] + v[4+j]), then two hadds. */
static float hsum8(const float v[8]) {
  float s[4];
  for (int j = 0; j < 4; ++j) s[j] = v[j] + v[4 + j];
  return (s[0] + s[1]) + (s[2] + s[3]);
}

/* l2_sq_scalar / l2_sq_avx512 / l2_sq_avx2 (scalar.cc:8-15, avx512.cc:19-32, avx2.cc:26-35). */
float orc_l2(const float* a, const float* b, size_t d, int order) {
  if (order == ORC_ORDER_AVX512) {
    float acc0[16] = {0}, acc1[16] = {0}, s[16];
    size_t i = 0;
    for (; i + 32 <= d; i += 32)
      for (int j = 0; j < 16; ++j) {
        float t0 = a[i + j] - b[i + j], t1 = a[i + 16 + j] - b[i + 16 + j];
        acc0[j] = fmaf(t0, t0, acc0[j]);
        acc1[j] = fmaf(t1, t1, acc1[j]);
      }
    if (i < d)
      for (int j = 0; j < 16; ++j) {
        float t0 = a[i + j] - b[i + j];
        acc0[j] = fmaf(t0, t0, acc0[j]);
      }
    for (int j = 0; j < 16; ++j) s[j] = acc0[j] + acc1[j];
    return reduce16(s);
  }
  if (order == ORC_ORDER_AVX2) {
    float acc0[8] = {0}, acc1[8] = {0}, s[8];
    for (size_t i = 0; i < d; i += 16)
      for (int j = 0; j < 8; ++j) {
        float t0 = a[i + j] - b[i + j], t1 = a[i + 8 + j] - b[i + 8 + j];
        acc0[j] = fmaf(t0, t0, acc0[j]);
        acc1[j] = fmaf(t1, t1, acc1[j]);
      }
    for (int j = 0; j < 8; ++j) s[j] = acc0[j] + acc1[j];
    return hsum8(s);
  }
  float s = 0.f;
  for (size_t i = 0; i < d; ++i) {
    float t = a[i] - b[i];
    s += t * t;
  }
  return s;
}

/* dot_scalar / dot_avx512 / dot_avx2 (scalar.cc:17-21, avx512.cc:34-42, avx2.cc:37-44). */
float orc_dot(const float* a, const float* b, size_t d, int order) {
  if (order == ORC_ORDER_AVX512) {
    float acc0[16] = {0}, acc1[16] = {0}, s[16];
    size_t i = 0;
    for (; i + 32 <= d; i += 32)
      for (int j = 0; j < 16; ++j) {
        acc0[j] = fmaf(a[i + j], b[i + j], acc0[j]);
        acc1[j] = fmaf(a[i + 16 + j], b[i + 16 + j], acc1[j]);
      }
    if (i < d)
      for (int j = 0; j < 16; ++j) acc0[j] = fmaf(a[i + j], b[i + j], acc0[j]);
    for (int j = 0; j < 16; ++j) s[j] = acc0[j] + acc1[j];
    return reduce16(s);
  }
  if (order == ORC_ORDER_AVX2) {
    float acc0[8] = {0}, acc1[8] = {0}, s[8];
    for (size_t i = 0; i < d; i += 16)
      for (int j = 0; j < 8; ++j) {
        acc0[j] = fmaf(a[i + j], b[i + j], acc0[j]);
        acc1[j] = fmaf(a[i + 8 + j], b[i + 8 + j], acc1[j]);
      }
    for (int j = 0; j < 8; ++j) s[j] = acc0[j] + acc1[j];
    return hsum8(s);
  }
  float s = 0.f;
  for (size_t i = 0; i < d; ++i) s += a[i] * b[i];
  return s;
}

/* MetricDistance (cpu_features.cc:64-66): L2 -> squared L2, IP/Cosine -> minus the dot. */
float orc_metric_dist(int metric, const float* a, const float* b, size_t d, int order) {
  return metric == ORC_L2 ? orc_l2(a, b, d, order) : -orc_dot(a, b, d, order);
}

/* sq8_l2_* / sq8_ip_* (scalar.cc:25-41, avx512.cc:11-15 + 48-65, avx2.cc:20-24 + 47-74);
 * MetricSq8Distance picks l2 for L2, ip otherwise (cpu_features.cc:68-71). */
float orc_sq8_dist(int metric, const float* q, const uint8_t* c, const float* vmin,
                   const float* scale, size_t d, int order) {
  const int l2 = metric == ORC_L2;
  if (order == ORC_ORDER_AVX512) {
    float acc[16] = {0};
    for (size_t i = 0; i < d; i += 16)
      for (int j = 0; j < 16; ++j) {
        float x = fmaf((float)c[i + j], scale[i + j], vmin[i + j]);
        if (l2) {
          float t = q[i + j] - x;
          acc[j] = fmaf(t, t, acc[j]);
        } else {
          acc[j] = fmaf(q[i + j], x, acc[j]);
        }
      }
    float r = reduce16(acc);
    return l2 ? r : -r;
  }
  if (order == ORC_ORDER_AVX2) {
    float acc0[8] = {0}, acc1[8] = {0}, s[8];
    for (size_t i = 0; i < d; i += 16)
      for (int j = 0; j < 8; ++j) {
        float x0 = fmaf((float)c[i + j], scale[i + j], vmin[i + j]);
        float x1 = fmaf((float)c[i + 8 + j], scale[i + 8 + j], vmin[i + 8 + j]);
        if (l2) {
          float t0 = q[i + j] - x0, t1 = q[i + 8 + j] - x1;
          acc0[j] = fmaf(t0, t0, acc0[j]);
          acc1[j] = fmaf(t1, t1, acc1[j]);
        } else {
          acc0[j] = fmaf(q[i + j], x0, acc0[j]);
          acc1[j] = fmaf(q[i + 8 + j], x1, acc1[j]);
        }
      }
    for (int j = 0; j < 8; ++j) s[j] = acc0[j] + acc1[j];
    float r = hsum8(s);
    return l2 ? r : -r;
  }
  float s = 0.f;
  for (size_t i = 0; i < d; ++i) {
    float x = vmin[i] + (float)c[i] * scale[i];
    if (l2) {
      float t = q[i] - x;
      s += t * t;
    } else {
      s += q[i] * x;
    }
  }
  return l2 ? s : -s;
}

/* L2SqAny (scalar.cc:43-60): four accumulators, combined as (s0+s1)+(s2+s3). */
float orc_l2_any(const float* a, const float* b, size_t d) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  size_t i = 0;
  for (; i + 4 <= d; i += 4) {
    float t0 = a[i] - b[i], t1 = a[i + 1] - b[i + 1];
    float t2 = a[i + 2] - b[i + 2], t3 = a[i + 3] - b[i + 3];
    s0 += t0 * t0;
    s1 += t1 * t1;
    s2 += t2 * t2;
    s3 += t3 * t3;
  }
  for (; i < d; ++i) {
    float t = a[i] - b[i];
    s0 += t * t;
  }
  return (s0 + s1) + (s2 + s3);
}

/* DotAny (scalar.cc:62-73). */
float orc_dot_any(const float* a, const float* b, size_t d) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  size_t i = 0;
  for (; i + 4 <= d; i += 4) {
    s0 += a[i] * b[i];
    s1 += a[i + 1] * b[i + 1];
    s2 += a[i + 2] * b[i + 2];
    s3 += a[i + 3] * b[i + 3];
  }
  for (; i < d; ++i) s0 += a[i] * b[i];
  return (s0 + s1) + (s2 + s3);
}

/* NormalizeVector (src/util/dataset.cc:33-40): double sum of squares, float inverse norm. */
int orc_normalize(float* v, size_t dim) {
  double norm = 0;
  for (size_t i = 0; i < dim; ++i) norm += (double)v[i] * v[i];
  if (!(norm > 0) || !isfinite(norm)) return 0;
  float inv = (float)(1.0 / sqrt(norm));
  for (size_t i = 0; i < dim; ++i) v[i] *= inv;
  return 1;
}

/* ------------------------------------------------------------------ heaps (TopK) */

/* Neighbor ordering of include/vdb/types.h:19-25: by dist, ties by id. */
static int nb_less(orc_neighbor a, orc_neighbor b) {
  return a.dist < b.dist || (a.dist == b.dist && a.id < b.id);
}

/* A binary heap; max_heap != 0 keeps the largest on top (TopK, results), else the smallest
 * (the candidate queue of search_layer). */
typedef struct {
  orc_neighbor* v;
  size_t n, cap;
  int max_heap;
} heap_t;

static int heap_before(const heap_t* h, orc_neighbor a, orc_neighbor b) {
  return h->max_heap ? nb_less(b, a) : nb_less(a, b);
}

static void heap_init(heap_t* h, size_t cap, int max_heap) {
  h->v = (orc_neighbor*)malloc((cap + 1) * sizeof(orc_neighbor));
  h->n = 0;
  h->cap = cap + 1;
  h->max_heap = max_heap;
}

static void heap_free(heap_t* h) { free(h->v); }

static void heap_push(heap_t* h, orc_neighbor x) {
  if (h->n == h->cap) {
    h->cap *= 2;
    h->v = (orc_neighbor*)realloc(h->v, h->cap * sizeof(orc_neighbor));
  }
  size_t i = h->n++;
  while (i > 0) {
    size_t p = (i - 1) / 2;
    if (!heap_before(h, x, h->v[p])) break;
    h->v[i] = h->v[p];
    i = p;
  }
  h->v[i] = x;
}

static orc_neighbor heap_pop(heap_t* h) {
  orc_neighbor top = h->v[0], x = h->v[--h->n];
  size_t i = 0;
  for (;;) {
    size_t l = 2 * i + 1, r = l + 1, m = i;
    orc_neighbor best = x;
    if (l < h->n && heap_before(h, h->v[l], best)) {
      m = l;
      best = h->v[l];
    }
    if (r < h->n && heap_before(h, h->v[r], best)) m = r;
    if (m == i) break;
    h->v[i] = h->v[m];
    i = m;
  }
  if (h->n > 0) h->v[i] = x;
  return top;
}

static int cmp_nb(const void* a, const void* b) {
  orc_neighbor x = *(const orc_neighbor*)a, y = *(const orc_neighbor*)b;
  return nb_less(x, y) ? -1 : nb_less(y, x) ? 1 : 0;
}

/* TopK::push (topk.h:17-28): keep the k smallest by (dist, id). */
typedef struct {
  heap_t h;
  size_t k;
} topk_t;

static void topk_init(topk_t* t, size_t k) {
  heap_init(&t->h, k, 1);
  t->k = k;
}

static void topk_push(topk_t* t, float dist, uint32_t id) {
  if (t->k == 0) return;
  orc_neighbor n = {dist, id};
  if (t->h.n < t->k) {
    heap_push(&t->h, n);
  } else if (nb_less(n, t->h.v[0])) {
    heap_pop(&t->h);
    heap_push(&t->h, n);
  }
}

/* TopK::sorted_into (topk.h:44-47): closest first. Returns the count. */
static size_t topk_sorted(topk_t* t, orc_neighbor* out) {
  memcpy(out, t->h.v, t->h.n * sizeof(orc_neighbor));
  qsort(out, t->h.n, sizeof(orc_neighbor), cmp_nb);
  return t->h.n;
}

static uint32_t write_out(const orc_neighbor* s, size_t n, uint32_t k, float* out_dist,
                          uint32_t* out_id) {
  for (uint32_t j = 0; j < k; ++j) {
    out_dist[j] = j < n ? s[j].dist : INFINITY;
    out_id[j] = j < n ? s[j].id : UINT32_MAX;
  }
  return (uint32_t)(n < k ? n : k);
}

uint32_t orc_topk(const float* dist, const uint32_t* id, uint64_t n, uint32_t k, float* out_dist,
                  uint32_t* out_id) {
  topk_t t;
  topk_init(&t, k);
  for (uint64_t i = 0; i < n; ++i) topk_push(&t, dist[i], id[i]);
  orc_neighbor* s = (orc_neighbor*)malloc((t.h.n + 1) * sizeof(orc_neighbor));
  size_t m = topk_sorted(&t, s);
  for (size_t j = 0; j < m; ++j) {
    out_dist[j] = s[j].dist;
    out_id[j] = s[j].id;
  }
  free(s);
  heap_free(&t.h);
  return (uint32_t)m;
}

static int allowed(const uint64_t* bits, uint32_t id) {
  return bits == NULL || ((bits[id >> 6] >> (id & 63)) & 1u);
}

/* Rerank (src/index/index.cc:89-95): exact distances of the candidates, k best. */
static size_t rerank(int metric, const float* rows, uint32_t pd, const float* q,
                     const orc_neighbor* cands, size_t nc, size_t k, int order, orc_neighbor* out) {
  topk_t t;
  topk_init(&t, k);
  for (size_t i = 0; i < nc; ++i)
    topk_push(&t, orc_metric_dist(metric, q, rows + (size_t)cands[i].id * pd, pd, order),
              cands[i].id);
  size_t m = topk_sorted(&t, out);
  heap_free(&t.h);
  return m;
}

/* ------------------------------------------------------------------ flat + SQ8 */

uint32_t orc_flat_search(int metric, const float* rows, uint64_t n, uint32_t pd, const float* q,
                         uint32_t k, const uint64_t* allow_bits, int order, float* out_dist,
                         uint32_t* out_id) {
  topk_t t;
  topk_init(&t, k);
  for (uint64_t i = 0; i < n; ++i) {
    if (!allowed(allow_bits, (uint32_t)i)) continue;
    topk_push(&t, orc_metric_dist(metric, q, rows + i * pd, pd, order), (uint32_t)i);
  }
  orc_neighbor* s = (orc_neighbor*)malloc((t.h.n + 1) * sizeof(orc_neighbor));
  size_t m = topk_sorted(&t, s);
  uint32_t r = write_out(s, m, k, out_dist, out_id);
  free(s);
  heap_free(&t.h);
  return r;
}

/* Sq8Quantizer::train (sq8.cc:9-26). std::min/std::max keep the first argument on ties. */
void orc_sq8_train(const float* rows, uint64_t n, uint32_t dim, uint32_t pd, float* vmin,
                   float* scale) {
  float* vmax = (float*)malloc(dim * sizeof(float));
  for (uint32_t i = 0; i < pd; ++i) {
    vmin[i] = 0.f;
    scale[i] = 0.f;
  }
  if (n == 0) {
    free(vmax);
    return;
  }
  for (uint32_t i = 0; i < dim; ++i) {
    vmin[i] = INFINITY;
    vmax[i] = -INFINITY;
  }
  for (uint64_t r = 0; r < n; ++r) {
    const float* x = rows + r * pd;
    for (uint32_t i = 0; i < dim; ++i) {
      vmin[i] = x[i] < vmin[i] ? x[i] : vmin[i];
      vmax[i] = vmax[i] < x[i] ? x[i] : vmax[i];
    }
  }
  for (uint32_t i = 0; i < dim; ++i) scale[i] = (vmax[i] - vmin[i]) / 255.f;
  free(vmax);
}

/* Sq8Quantizer::encode (sq8.cc:28-37): nearbyint of an IEEE division, clamped to [0, 255]. */
void orc_sq8_encode(const float* x, uint32_t dim, uint32_t pd, const float* vmin,
                    const float* scale, uint8_t* code) {
  for (uint32_t i = 0; i < pd; ++i) {
    if (i >= dim || scale[i] <= 0.f) {
      code[i] = 0;
      continue;
    }
    float c = nearbyintf((x[i] - vmin[i]) / scale[i]);
    c = c < 0.f ? 0.f : (255.f < c ? 255.f : c);
    code[i] = (uint8_t)c;
  }
}

uint32_t orc_sq8_scan_search(int metric, const float* rows, uint64_t n, uint32_t pd,
                             const uint8_t* codes, const float* vmin, const float* scale,
                             const float* q, uint32_t k, uint32_t depth, int order,
                             float* out_dist, uint32_t* out_id) {
  topk_t t;
  topk_init(&t, depth);
  for (uint64_t i = 0; i < n; ++i)
    topk_push(&t, orc_sq8_dist(metric, q, codes + i * pd, vmin, scale, pd, order), (uint32_t)i);
  orc_neighbor* c = (orc_neighbor*)malloc((t.h.n + 1) * sizeof(orc_neighbor));
  orc_neighbor* o = (orc_neighbor*)malloc((k + 1) * sizeof(orc_neighbor));
  size_t nc = topk_sorted(&t, c);
  size_t m = rerank(metric, rows, pd, q, c, nc, k, order, o);
  uint32_t r = write_out(o, m, k, out_dist, out_id);
  free(c);
  free(o);
  heap_free(&t.h);
  return r;
}

/* ------------------------------------------------------------------ PQ / IVF-PQ */

void orc_pq_compute_table(const float* q, int metric, const float* centroids, uint32_t m,
                          uint32_t dsub, float* table) {
  for (uint32_t j = 0; j < m; ++j) {
    const float* qs = q + (size_t)j * dsub;
    float* t = table + (size_t)j * 256;
    for (uint32_t c = 0; c < 256; ++c) {
      const float* cen = centroids + ((size_t)j * 256 + c) * dsub;
      t[c] = metric == ORC_L2 ? orc_l2_any(qs, cen, dsub) : -orc_dot_any(qs, cen, dsub);
    }
  }
}

float orc_pq_adc(const float* table, const uint8_t* code, uint32_t m) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
  uint32_t j = 0;
  for (; j + 4 <= m; j += 4) {
    s0 += table[(j + 0) * 256 + code[j + 0]];
    s1 += table[(j + 1) * 256 + code[j + 1]];
    s2 += table[(j + 2) * 256 + code[j + 2]];
    s3 += table[(j + 3) * 256 + code[j + 3]];
  }
  for (; j < m; ++j) s0 += table[j * 256 + code[j]];
  return (s0 + s1) + (s2 + s3);
}

void orc_ivfpq_term2(const float* coarse, uint32_t nlist, uint32_t pd, const float* centroids,
                     uint32_t m, uint32_t dsub, float* term2) {
  float* norms = (float*)malloc((size_t)m * 256 * sizeof(float));
  for (uint32_t j = 0; j < m; ++j)
    for (uint32_t c = 0; c < 256; ++c) {
      const float* cen = centroids + ((size_t)j * 256 + c) * dsub;
      norms[j * 256 + c] = orc_dot_any(cen, cen, dsub);
    }
  for (uint32_t l = 0; l < nlist; ++l) {
    const float* cl = coarse + (size_t)l * pd;
    float* t = term2 + (size_t)l * m * 256;
    for (uint32_t j = 0; j < m; ++j)
      for (uint32_t c = 0; c < 256; ++c) {
        const float* cen = centroids + ((size_t)j * 256 + c) * dsub;
        t[j * 256 + c] = norms[j * 256 + c] + 2.f * orc_dot_any(cl + (size_t)j * dsub, cen, dsub);
      }
  }
  free(norms);
}

uint32_t orc_ivfpq_search(const orc_ivfpq* ix, int metric, const float* rows, const float* q,
                          uint32_t k, uint32_t nprobe_req, int rerank_req,
                          const uint64_t* allow_bits, int order, float* out_dist,
                          uint32_t* out_id, uint64_t* out_dc) {
  const uint32_t pd = ix->pd, d = ix->dim, m = ix->m, ts = m * 256;
  if (ix->nlist == 0 || k == 0) {
    if (out_dc) *out_dc = 0;
    return write_out(NULL, 0, k, out_dist, out_id);
  }
  uint64_t dc = ix->nlist;
  orc_neighbor* cd = (orc_neighbor*)malloc(ix->nlist * sizeof(orc_neighbor));
  for (uint32_t c = 0; c < ix->nlist; ++c) {
    cd[c].dist = orc_metric_dist(metric, q, ix->coarse + (size_t)c * pd, pd, order);
    cd[c].id = c;
  }
  uint32_t nprobe = nprobe_req < 1 ? 1 : (nprobe_req > ix->nlist ? ix->nlist : nprobe_req);
  /* partial_sort of the first nprobe by (dist, id) */
  qsort(cd, ix->nlist, sizeof(orc_neighbor), cmp_nb);
  size_t depth = rerank_req < 0 ? (10 * (size_t)k > 100 ? 10 * (size_t)k : 100) : (size_t)rerank_req;
  topk_t top;
  topk_init(&top, depth > k ? depth : k);
  float* table = (float*)malloc(ts * sizeof(float));
  float* qtab = (float*)malloc(ts * sizeof(float));
  float* resid = (float*)malloc(d * sizeof(float));
  const int l2 = metric == ORC_L2;
  const int pre = l2 && ix->term2 != NULL;
  if (!l2) orc_pq_compute_table(q, metric, ix->centroids, m, ix->dsub, table);
  if (pre) {
    orc_pq_compute_table(q, ORC_IP, ix->centroids, m, ix->dsub, qtab);
    for (uint32_t i = 0; i < ts; ++i) qtab[i] *= 2.f;
  }
  for (uint32_t pi = 0; pi < nprobe; ++pi) {
    const uint32_t l = cd[pi].id;
    const float* c = ix->coarse + (size_t)l * pd;
    float offset = 0;
    if (pre) {
      offset = cd[pi].dist;
      const float* t2 = ix->term2 + (size_t)l * ts;
      for (uint32_t i = 0; i < ts; ++i) table[i] = t2[i] + qtab[i];
    } else if (l2) {
      for (uint32_t j = 0; j < d; ++j) resid[j] = q[j] - c[j];
      orc_pq_compute_table(resid, ORC_L2, ix->centroids, m, ix->dsub, table);
    } else {
      offset = -orc_dot_any(q, c, d);
    }
    const uint64_t b = ix->list_off[l], e = ix->list_off[l + 1];
    for (uint64_t i = b; i < e; ++i) {
      if (!allowed(allow_bits, ix->ids[i])) continue;
      topk_push(&top, offset + orc_pq_adc(table, ix->codes + i * m, m), ix->ids[i]);
    }
    dc += e - b;
  }
  orc_neighbor* s = (orc_neighbor*)malloc((top.h.n + 1) * sizeof(orc_neighbor));
  size_t ns = topk_sorted(&top, s);
  uint32_t r;
  if (depth == 0) {
    r = write_out(s, ns, k, out_dist, out_id);
  } else {
    orc_neighbor* o = (orc_neighbor*)malloc((k + 1) * sizeof(orc_neighbor));
    size_t mo = rerank(metric, rows, pd, q, s, ns, k, order, o);
    dc += ns;
    r = write_out(o, mo, k, out_dist, out_id);
    free(o);
  }
  if (out_dc) *out_dc = dc;
  free(s);
  free(table);
  free(qtab);
  free(resid);
  free(cd);
  heap_free(&top.h);
  return r;
}

/* ------------------------------------------------------------------ HNSW */

typedef struct {
  const orc_hnsw* g;
  int metric, order;
  const float* rows;
  const uint8_t* codes;
  const float *vmin, *scale;
  uint32_t pd;
} space_t;

static float space_dist(const space_t* s, const float* q, uint32_t id) {
  if (s->codes != NULL)
    return orc_sq8_dist(s->metric, q, s->codes + (size_t)id * s->pd, s->vmin, s->scale, s->pd,
                        s->order);
  return orc_metric_dist(s->metric, q, s->rows + (size_t)id * s->pd, s->pd, s->order);
}

/* links_at (hnsw_graph.h:459-466): [count][links...] */
static const uint32_t* links_at(const orc_hnsw* g, uint32_t id, int layer) {
  if (layer == 0) return g->links0 + (size_t)id * (1 + g->M0);
  return g->upper + g->upper_off[id] + (size_t)(layer - 1) * (1 + g->M);
}

/* greedy<false> (hnsw_graph.h:482-508) */
static void greedy(const space_t* s, const float* q, uint32_t* cur, float* curd, int layer,
                   uint64_t* dc) {
  for (int changed = 1; changed;) {
    changed = 0;
    const uint32_t* ll = links_at(s->g, *cur, layer);
    const uint32_t cnt = ll[0];
    const uint32_t* nb = ll + 1;
    for (uint32_t j = 0; j < cnt; ++j) {
      float d = space_dist(s, q, nb[j]);
      ++*dc;
      if (d < *curd) {
        *curd = d;
        *cur = nb[j];
        changed = 1;
      }
    }
  }
}

/* search_layer<false, filtered> (hnsw_graph.h:513-567) on layer 0. Leaves the results in
 * `results` (a max-heap). */
static void search_layer0(const space_t* s, const float* q, uint32_t ep, float ep_dist, size_t ef,
                          const uint64_t* allow_bits, uint8_t* seen, heap_t* results,
                          uint64_t* dc) {
  heap_t cand;
  heap_init(&cand, 64, 0);
  const int filtered = allow_bits != NULL;
  seen[ep] = 1;
  float lower = INFINITY;
  orc_neighbor e0 = {ep_dist, ep};
  if (!filtered || allowed(allow_bits, ep)) {
    heap_push(results, e0);
    lower = ep_dist;
  }
  heap_push(&cand, e0);
  while (cand.n > 0) {
    orc_neighbor c = cand.v[0];
    if (c.dist > lower && (!filtered || results->n >= ef)) break;
    heap_pop(&cand);
    const uint32_t* ll = links_at(s->g, c.id, 0);
    const uint32_t cnt = ll[0];
    for (uint32_t j = 0; j < cnt; ++j) {
      const uint32_t e = ll[1 + j];
      if (seen[e]) continue;
      seen[e] = 1;
      const float de = space_dist(s, q, e);
      ++*dc;
      if (results->n < ef || de < lower) {
        orc_neighbor x = {de, e};
        heap_push(&cand, x);
        if (!filtered || allowed(allow_bits, e)) {
          heap_push(results, x);
          if (results->n > ef) heap_pop(results);
          lower = results->v[0].dist;
        }
      }
    }
  }
  heap_free(&cand);
}

/* HnswGraph::search (hnsw_graph.h:286-309): returns the sorted k best in out. */
static size_t graph_search(const space_t* s, const float* q, size_t k, size_t ef,
                           const uint64_t* allow_bits, orc_neighbor* out, uint64_t* dist_count) {
  const orc_hnsw* g = s->g;
  if (g->max_level < 0 || k == 0) return 0;
  uint64_t dc = 1;
  uint32_t cur = g->entry;
  float curd = space_dist(s, q, cur);
  for (int l = g->max_level; l > 0; --l) greedy(s, q, &cur, &curd, l, &dc);
  if (ef < k) ef = k;
  uint8_t* seen = (uint8_t*)calloc(g->cap > 0 ? g->cap : 1, 1);
  heap_t results;
  heap_init(&results, ef + 1, 1);
  search_layer0(s, q, cur, curd, ef, allow_bits, seen, &results, &dc);
  while (results.n > k) heap_pop(&results);
  size_t n = results.n;
  memcpy(out, results.v, n * sizeof(orc_neighbor));
  qsort(out, n, sizeof(orc_neighbor), cmp_nb);
  heap_free(&results);
  free(seen);
  *dist_count += dc;
  return n;
}

uint32_t orc_hnsw_search(const orc_hnsw* g, int metric, const float* rows, const uint8_t* codes,
                         const float* vmin, const float* scale, uint32_t pd, const float* q,
                         uint32_t k, uint32_t ef, const uint64_t* allow_bits, int order,
                         float* out_dist, uint32_t* out_id, uint64_t* out_dc) {
  space_t s = {g, metric, order, rows, codes, vmin, scale, pd};
  /* HnswIndex::search (hnsw_index.cc:22-34) passes max(p.ef, k). */
  size_t efk = ef > k ? ef : k;
  orc_neighbor* out = (orc_neighbor*)malloc((k + 1) * sizeof(orc_neighbor));
  uint64_t dc = 0;
  size_t n = graph_search(&s, q, k, efk, allow_bits, out, &dc);
  uint32_t r = write_out(out, n, k, out_dist, out_id);
  if (out_dc) *out_dc = dc;
  free(out);
  return r;
}

uint32_t orc_hnsw_sq8_search(const orc_hnsw* g, int metric, const float* rows,
                             const uint8_t* codes, const float* vmin, const float* scale,
                             uint32_t pd, const float* q, uint32_t k, uint32_t ef, int rerank_req,
                             const uint64_t* allow_bits, int order, float* out_dist,
                             uint32_t* out_id, uint64_t* out_dc) {
  space_t s = {g, metric, order, rows, codes, vmin, scale, pd};
  if (k == 0) {
    if (out_dc) *out_dc = 0;
    return write_out(NULL, 0, k, out_dist, out_id);
  }
  size_t depth = rerank_req < 0 ? (ef > k ? ef : k) : (size_t)rerank_req;
  size_t ef2 = ef > k ? ef : k;
  if (depth > ef2) ef2 = depth;
  uint64_t dc = 0;
  uint32_t r;
  if (depth == 0) {
    orc_neighbor* out = (orc_neighbor*)malloc((k + 1) * sizeof(orc_neighbor));
    size_t n = graph_search(&s, q, k, ef2, allow_bits, out, &dc);
    r = write_out(out, n, k, out_dist, out_id);
    free(out);
  } else {
    size_t kk = depth > k ? depth : k;
    orc_neighbor* cands = (orc_neighbor*)malloc((kk + 1) * sizeof(orc_neighbor));
    orc_neighbor* out = (orc_neighbor*)malloc((k + 1) * sizeof(orc_neighbor));
    size_t nc = graph_search(&s, q, kk, ef2, allow_bits, cands, &dc);
    size_t n = rerank(metric, rows, pd, q, cands, nc, k, order, out);
    dc += nc;
    r = write_out(out, n, k, out_dist, out_id);
    free(cands);
    free(out);
  }
  if (out_dc) *out_dc = dc;
  return r;
}
