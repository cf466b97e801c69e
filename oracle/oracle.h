/* Test infrastructure, not product code.
 *
 * A plain-C restatement of the reference's (vdb's) CPU search algorithms, used only by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker. Every function cites
 * the reference file:line it follows. The product never links this library.
 */
#ifndef VDB_ORACLE_H_
#define VDB_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Summation order of the fp32 distance kernels. The reference picks its kernel set at run time
 * (src/distance/cpu_features.cc:36-42); each set sums in a different, fixed order. */
enum { ORC_ORDER_SCALAR = 0, ORC_ORDER_AVX512 = 1, ORC_ORDER_AVX2 = 2 };
/* vdb::Metric, include/vdb/types.h:17 */
enum { ORC_L2 = 0, ORC_IP = 1, ORC_COSINE = 2 };

typedef struct {
  float dist;
  uint32_t id;
} orc_neighbor;

/* Distance kernels (src/distance/scalar.cc, avx2.cc, avx512.cc); d is the padded dim. */
float orc_l2(const float* a, const float* b, size_t d, int order);
float orc_dot(const float* a, const float* b, size_t d, int order);
float orc_metric_dist(int metric, const float* a, const float* b, size_t d, int order);
float orc_sq8_dist(int metric, const float* q, const uint8_t* code, const float* vmin,
                   const float* scale, size_t d, int order);
float orc_l2_any(const float* a, const float* b, size_t d);
float orc_dot_any(const float* a, const float* b, size_t d);

/* NormalizeVector, src/util/dataset.cc:33-40. Returns 0 for a zero/non-finite row. */
int orc_normalize(float* v, size_t dim);

/* TopK (src/util/topk.h:13-54): k smallest by (dist, id), written closest first.
 * Returns the number written. */
uint32_t orc_topk(const float* dist, const uint32_t* id, uint64_t n, uint32_t k, float* out_dist,
                  uint32_t* out_id);

/* FlatSearch over allowed rows (src/index/flat_index.cc:11-27). */
uint32_t orc_flat_search(int metric, const float* rows, uint64_t n, uint32_t pd, const float* q,
                         uint32_t k, const uint64_t* allow_bits, int order, float* out_dist,
                         uint32_t* out_id);

/* Sq8Quantizer::train / encode (src/index/quant/sq8.cc:9-37). */
void orc_sq8_train(const float* rows, uint64_t n, uint32_t dim, uint32_t pd, float* vmin,
                   float* scale);
void orc_sq8_encode(const float* x, uint32_t dim, uint32_t pd, const float* vmin,
                    const float* scale, uint8_t* code);

/* Exhaustive SQ8 scan + fp32 re-rank composed from reference primitives:
 * MetricSq8Distance -> TopK(depth) -> Rerank(MetricDistance) (src/index/index.cc:89-95). */
uint32_t orc_sq8_scan_search(int metric, const float* rows, uint64_t n, uint32_t pd,
                             const uint8_t* codes, const float* vmin, const float* scale,
                             const float* q, uint32_t k, uint32_t depth, int order,
                             float* out_dist, uint32_t* out_id);

/* ProductQuantizer::compute_table / adc (src/index/quant/pq.cc:63-73, pq.h:36-47). */
void orc_pq_compute_table(const float* q, int metric, const float* centroids, uint32_t m,
                          uint32_t dsub, float* table);
float orc_pq_adc(const float* table, const uint8_t* code, uint32_t m);

/* IvfPqIndex::precompute_tables (src/index/quant/ivf_pq.cc:152-167): term2 is nlist*m*256. */
void orc_ivfpq_term2(const float* coarse, uint32_t nlist, uint32_t pd, const float* centroids,
                     uint32_t m, uint32_t dsub, float* term2);

/* An IVF-PQ index as stored by IvfPqIndex::save (src/index/quant/ivf_pq.cc:236-249). */
typedef struct {
  uint32_t nlist, pd, dim, m, dsub;
  const float* coarse;    /* nlist * pd */
  const float* centroids; /* m * 256 * dsub */
  const uint64_t* list_off; /* nlist + 1, offsets into ids (and codes / m) */
  const uint32_t* ids;
  const uint8_t* codes;
  const float* term2; /* nlist*m*256 or NULL (no precomputed tables) */
} orc_ivfpq;

/* IvfPqIndex::search (src/index/quant/ivf_pq.cc:169-222) + FinishSearch (:28-36). */
uint32_t orc_ivfpq_search(const orc_ivfpq* ix, int metric, const float* rows, const float* q,
                          uint32_t k, uint32_t nprobe, int rerank, const uint64_t* allow_bits,
                          int order, float* out_dist, uint32_t* out_id, uint64_t* out_dc);

/* An HNSW graph as stored by HnswGraph::serialize (src/index/hnsw/hnsw_graph.h:387-401). */
typedef struct {
  uint64_t cap, size;
  uint32_t M, M0;
  int32_t max_level;
  uint32_t entry;
  const uint8_t* level;      /* cap */
  const uint32_t* links0;    /* cap * (1 + M0) */
  const uint32_t* upper;     /* concatenated level*(1+M) blocks */
  const uint64_t* upper_off; /* cap: offset (in u32) of node i's upper block */
} orc_hnsw;

/* HnswGraph::search (src/index/hnsw/hnsw_graph.h:286-309, greedy 482-508, search_layer
 * 513-567) over float rows (codes == NULL) or SQ8 codes (Sq8Space, hnsw_index.h:44-59). */
uint32_t orc_hnsw_search(const orc_hnsw* g, int metric, const float* rows, const uint8_t* codes,
                         const float* vmin, const float* scale, uint32_t pd, const float* q,
                         uint32_t k, uint32_t ef, const uint64_t* allow_bits, int order,
                         float* out_dist, uint32_t* out_id, uint64_t* out_dc);

/* HnswSq8Index::search (src/index/hnsw/hnsw_index.cc:82-102): beam over codes, then Rerank. */
uint32_t orc_hnsw_sq8_search(const orc_hnsw* g, int metric, const float* rows,
                             const uint8_t* codes, const float* vmin, const float* scale,
                             uint32_t pd, const float* q, uint32_t k, uint32_t ef, int rerank,
                             const uint64_t* allow_bits, int order, float* out_dist,
                             uint32_t* out_id, uint64_t* out_dc);

#ifdef __cplusplus
}
#endif
#endif /* VDB_ORACLE_H_ */
