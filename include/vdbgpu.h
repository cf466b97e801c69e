/* vdbgpu: B200-native batched nearest-neighbour search behind vdb's Index interface.
 *
 * A C ABI (plain pointers, sizes and integer status codes; no C++ types, no exceptions) over the
 * GPU implementation of vdb's search path (KoduruChandrasekhar/HNSW-Vector-DB). Every entry point
 * names the reference interface it replaces. Paths below are relative to the reference project.
 *
 * Pointer arguments that carry vectors or results may point to host memory or to device memory
 * of the context's GPU; the library detects which and copies host buffers itself.
 * Thread safety: a context serialises its calls; use one context per thread for concurrency.
 */
#ifndef VDBGPU_H_
#define VDBGPU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VDBGPU_ABI_VERSION 1

#if defined(__GNUC__)
#define VDBGPU_API __attribute__((visibility("default")))
#else
#define VDBGPU_API
#endif

/* Status codes: the values of vdb::Status::Code (include/vdb/status.h:14-26). */
typedef enum vdbgpu_status {
  VDBGPU_OK = 0,
  VDBGPU_INVALID_ARGUMENT = 1,
  VDBGPU_NOT_FOUND = 2,
  VDBGPU_ALREADY_EXISTS = 3,
  VDBGPU_IO_ERROR = 4,
  VDBGPU_CORRUPTION = 5,
  VDBGPU_FAILED_PRECONDITION = 6,
  VDBGPU_RESOURCE_EXHAUSTED = 7, /* device allocation failed */
  VDBGPU_UNAVAILABLE = 8,        /* no GPU, or a bounded device wait ran out */
  VDBGPU_NOT_SUPPORTED = 9,
  VDBGPU_INTERNAL = 10
} vdbgpu_status;

/* vdb::Metric (include/vdb/types.h:17): smaller distance is closer for every metric. */
typedef enum vdbgpu_metric {
  VDBGPU_METRIC_L2 = 0,     /* squared L2 */
  VDBGPU_METRIC_IP = 1,     /* minus the dot product */
  VDBGPU_METRIC_COSINE = 2  /* rows and queries normalised, minus the dot product */
} vdbgpu_metric;

/* vdb::IndexType (include/vdb/options.h:13), plus SQ8_FLAT: an exhaustive scan of SQ8 codes
 * with an fp32 re-rank, which has no reference index type. */
typedef enum vdbgpu_index_type {
  VDBGPU_INDEX_FLAT = 0,
  VDBGPU_INDEX_HNSW = 1,
  VDBGPU_INDEX_HNSW_SQ8 = 2,
  VDBGPU_INDEX_PQ_FLAT = 3,
  VDBGPU_INDEX_IVF_PQ = 4,
  VDBGPU_INDEX_SQ8_FLAT = 16
} vdbgpu_index_type;

/* vdb::SearchParams (include/vdb/options.h:59-67). */
typedef struct vdbgpu_search_params {
  uint64_t ef;       /* HNSW beam width; max(ef, k) is used (default 64) */
  uint64_t nprobe;   /* IVF lists to scan (default 16) */
  int32_t rerank;    /* candidates re-ranked on fp32 rows; -1 = auto, 0 = none */
  int32_t strategy;  /* vdb::FilterStrategy: 0 auto, 1 prefilter, 2 graph, 3 postfilter */
  uint64_t prefilter_threshold; /* default 10000 */
  uint64_t post_filter_alpha;   /* default 10 */
} vdbgpu_search_params;

typedef struct vdbgpu_index_info {
  int32_t type;
  int32_t metric;
  uint64_t rows;
  uint32_t dim;
  uint32_t padded_dim;
  uint64_t device_bytes; /* HBM held by the index */
} vdbgpu_index_info;

typedef struct vdbgpu_ctx vdbgpu_ctx;
typedef struct vdbgpu_index vdbgpu_index;

/* Library version (VDBGPU_ABI_VERSION). */
VDBGPU_API int vdbgpu_abi_version(void);

/* Kernel launches this library has made in this process, on every device (no counterpart in the
 * reference, which has no GPU): the difference across a timed region is its launch count. */
VDBGPU_API int vdbgpu_launch_count(uint64_t* out);

/* Number of visible CUDA devices (0 without a GPU). */
VDBGPU_API int vdbgpu_device_count(int* out);

/* Opens a context on `device` (one stream, one workspace). No reference counterpart: the
 * reference runs on host threads (src/util/thread_pool.h:15-44). */
VDBGPU_API int vdbgpu_open(int device, vdbgpu_ctx** out);
VDBGPU_API void vdbgpu_close(vdbgpu_ctx* ctx);

/* Copies the context's last error message (NUL-terminated, truncated to cap) and returns its
 * full length. Replaces vdb::Status::ToString (include/vdb/status.h). */
VDBGPU_API size_t vdbgpu_last_error(const vdbgpu_ctx* ctx, char* buf, size_t cap);

/* Launches the context's work on `stream` (a cudaStream_t of the context's device; NULL restores
 * the context's own stream), like cublasSetStream. */
VDBGPU_API int vdbgpu_set_stream(vdbgpu_ctx* ctx, void* stream);

/* Enables (1) or disables (0) per-stage device timing of searches, read back with
 * vdbgpu_stage_times. The counterpart of SearchExplain's micros (include/vdb/collection.h). */
VDBGPU_API int vdbgpu_set_timing(vdbgpu_ctx* ctx, int enable);

/* Device milliseconds of the last search's stages (CUDA events on the launching stream):
 * out[0] = query preparation (plus, for a seeded flat / SQ8 scan, the scan of the row sample
 * and the seed), out[1] = the dominant scan or walk kernel, out[2] = selection and re-rank.
 * Returns the number of stages written (0 when timing is off). */
VDBGPU_API int vdbgpu_stage_times(vdbgpu_ctx* ctx, float* out, int cap);

/* Work counters of the last search's dominant kernel, collected while timing is on. For the
 * tensor-core scan: out[0] chunks of 32 columns filtered, out[1] chunks with a candidate,
 * out[2] candidates appended, out[3] candidate-list compactions. Returns the count written. */
VDBGPU_API int vdbgpu_stage_counters(vdbgpu_ctx* ctx, uint64_t* out, int cap);

/* Blocks until the context's stream is idle. */
VDBGPU_API int vdbgpu_synchronize(vdbgpu_ctx* ctx);

/* Sets vdb::SearchParams defaults (include/vdb/options.h:59-67). */
VDBGPU_API void vdbgpu_search_params_default(vdbgpu_search_params* p);

/* LoadIndex (src/index/index.h:61-62, src/index/index.cc:58-87): parses an index file written
 * by the reference's Index::save (magic VDBFLAT1 / VDBHNSW1 / VDBHSQ81 / VDBPQFL1 / VDBIVFP1,
 * CRC32C footer) over the segment's float rows (VectorView, src/util/aligned_buffer.h:56-63:
 * nrows x padded_dim floats, zero padded) and copies everything the search needs to the GPU.
 * The rows are read, not retained. */
VDBGPU_API int vdbgpu_index_load(vdbgpu_ctx* ctx, const void* file_bytes, size_t nbytes, int metric,
                      const float* rows, uint64_t nrows, uint32_t dim, uint32_t padded_dim,
                      vdbgpu_index** out);

/* CreateIndex + Index::build (src/index/index.h:58-59, index.cc:16-36) for index types built on
 * the GPU: FLAT (nothing to train) and SQ8_FLAT (Sq8Quantizer::train/encode,
 * src/index/quant/sq8.cc:9-37, bit-exact). */
VDBGPU_API int vdbgpu_index_create(vdbgpu_ctx* ctx, int type, int metric, const float* rows, uint64_t nrows,
                        uint32_t dim, uint32_t padded_dim, vdbgpu_index** out);

VDBGPU_API void vdbgpu_index_free(vdbgpu_index* index);

VDBGPU_API int vdbgpu_index_get_info(const vdbgpu_index* index, vdbgpu_index_info* out);

/* Index::search for a batch (src/index/index.h:44-45): the k nearest allowed rows of each of
 * nq queries (nq x padded_dim floats, already padded and, for cosine, normalised as
 * CollectionImpl::PrepareQuery does, src/engine/collection_impl.cc:1023-1034), closest first,
 * ties by row id. Missing slots are (+inf, UINT32_MAX). allow_bits (nullable) is a dense bitset
 * of allowed rows (bit r of word r/64), the RowFilter of src/index/index.h:23-27.
 * out_dist_comps (nullable, nq values) receives IndexSearchStats::distance_computations
 * (src/index/index.h:29-32). params may be NULL (defaults). The call returns once the results
 * are written: it synchronises the launching stream (also part-way through, for a large flat /
 * SQ8 batch, to learn which queries its seeded scan must rescan). */
VDBGPU_API int vdbgpu_index_search(vdbgpu_index* index, const float* queries, uint64_t nq, uint32_t k,
                        const vdbgpu_search_params* params, const uint64_t* allow_bits,
                        float* out_dist, uint32_t* out_row, uint64_t* out_dist_comps);

/* Index::search for FLAT and SQ8_FLAT indexes without allocating any device memory. No
 * counterpart in the reference: it exists for callers that must not allocate device memory while
 * they search (a host whose device memory is owned by its own allocator, or a serving loop that
 * cannot afford cudaMalloc's synchronisation or its failure under memory pressure).
 * Scratch comes from a fixed array of about 8.4 MB compiled into the library, which every GPU that
 * loads the library holds until the process exits; its device address is looked up on the first
 * call on each device.
 * Limits: nq <= 128 queries per call, padded_dim <= 256; larger requests fail with
 * VDBGPU_INVALID_ARGUMENT. queries, out_dist and out_row must be device memory of the index's
 * device (nq x padded_dim, nq x k, nq x k). Work is launched on `stream` (NULL: the context's
 * stream) and the call returns once it has finished. All calls share the one scratch array: calls
 * whose work overlaps on the GPU race and must be serialised by the caller. Results are those of
 * vdbgpu_index_search with the same parameters (no filter, no statistics); an empty index gives
 * misses (+inf, UINT32_MAX) in every slot. The scan runs on at most 16 SMs: the entry point is
 * meant for small batches, where latency rather than throughput matters. */
VDBGPU_API int vdbgpu_index_search_noalloc(vdbgpu_index* index, const float* queries, uint64_t nq,
                                           uint32_t k, const vdbgpu_search_params* params,
                                           float* out_dist, uint32_t* out_row, void* stream);

/* CheckIndexFile (src/index/index.cc:46-56) + the magic dispatch of LoadIndex (index.cc:58-87)
 * without a GPU: verifies the CRC32C footer and reports the index type of the magic. */
VDBGPU_API int vdbgpu_index_file_inspect(const void* file_bytes, size_t nbytes, int* type);

/* The SQ8 quantiser and codes of an SQ8 index (Sq8Quantizer::vmin/scale, src/index/quant/
 * sq8.h:24-25): vmin, scale receive padded_dim floats; codes (nullable) nrows x padded_dim. */
VDBGPU_API int vdbgpu_index_sq8_export(const vdbgpu_index* index, float* vmin, float* scale,
                            uint8_t* codes);

/* ------------------------------------------------------------------ collections (read path)
 *
 * A collection's on-disk segments on one GPU (or this rank's share of them), searched as
 * vdb::Collection::SearchBatch does (src/engine/collection_impl.cc:1121-1136): per segment the
 * planner of SearchDiskSegment (src/engine/planner.cc:42-129) over the segment's filter bitmap,
 * then the merge of CollectionImpl::Search (collection_impl.cc:1079-1108). The mutable and frozen
 * in-memory segments stay with the host (SearchMutable); their hits merge with
 * vdbgpu_merge_hits. */

typedef struct vdbgpu_collection vdbgpu_collection;

/* One merged hit (24 bytes): ordered by (dist, part, row); part = the segment's position among
 * the collection's disk segments; id = the external id (vdb::VectorId). A miss has
 * id UINT64_MAX, dist +inf, part and row UINT32_MAX. */
typedef struct vdbgpu_hit {
  float dist;
  uint32_t part;
  uint32_t row;
  uint32_t pad;
  uint64_t id;
} vdbgpu_hit;

/* Collection::Open's recovery of the on-disk state (CollectionImpl::Recover, collection_impl.cc:
 * 95-150, Segment::Open, src/storage/segment_reader.cc:20-122): reads CURRENT, the manifest and
 * every segment directory (vectors.f32, ids.u64, meta.bin, index.<type>). With nshards > 1 only
 * the segments whose manifest position % nshards == shard are loaded (one shard per GPU).
 * A segment's persisted delete set (the manifest entry's deletes_file, a "VDBDEL01" blob holding a
 * portable roaring bitmap) is loaded as its delete bits; a value at or past the segment's rows is
 * VDBGPU_CORRUPTION, as Segment::Open. The logs (wal/<n>.log from the manifest's wal_log_number)
 * are replayed as recovery does (collection_impl.cc:160-235): records after flushed_lsn delete
 * the old rows of their ids and append upserts to the mutable segment, which shard 0 holds and
 * searches exhaustively (merge part 0; disk segments are parts 1..n in manifest order). Damaged
 * logs give recovery's errors (VDBGPU_CORRUPTION); a torn tail of the newest log is ignored. The
 * directory is not modified. Later deletes go through vdbgpu_collection_set_deleted. */
VDBGPU_API int vdbgpu_collection_open(vdbgpu_ctx* ctx, const char* path, uint32_t shard,
                                      uint32_t nshards, vdbgpu_collection** out);

/* An empty collection with the reference's options JSON (src/engine/options_json.cc:72-104:
 * dim, metric, index type, schema), to be filled with vdbgpu_collection_add_segment. */
VDBGPU_API int vdbgpu_collection_create(vdbgpu_ctx* ctx, const char* options_json,
                                        vdbgpu_collection** out);

/* One segment from the contents of its files: rows = n x padded_dim floats (host or device; the
 * body of vectors.f32), ids = n external ids (host), meta = the payload of meta.bin (u64 rows,
 * u64 offsets[rows + 1], EncodeMetaRow rows; NULL/0 = no metadata), index_file = the whole
 * index file. ordinal = the segment's position among the collection's disk segments. */
VDBGPU_API int vdbgpu_collection_add_segment(vdbgpu_collection* c, uint32_t segment_id,
                                             uint32_t ordinal, const float* rows, uint64_t n,
                                             const uint64_t* ids, const void* meta,
                                             size_t meta_bytes, const void* index_file,
                                             size_t index_bytes);

/* The deleted rows of a segment (Segment::deletes, src/storage/segment.h): bit r of 32-bit word
 * r / 32 (host); NULL clears them. */
VDBGPU_API int vdbgpu_collection_set_deleted(vdbgpu_collection* c, uint32_t segment_id,
                                             const uint32_t* bits);

VDBGPU_API void vdbgpu_collection_free(vdbgpu_collection* c);

typedef struct vdbgpu_collection_info {
  uint32_t dim;
  uint32_t padded_dim;
  int32_t metric;
  int32_t index_type;
  uint32_t segments_total;
  uint32_t segments_local;
  uint64_t rows_local;
  uint64_t device_bytes;
} vdbgpu_collection_info;

VDBGPU_API int vdbgpu_collection_get_info(const vdbgpu_collection* c, vdbgpu_collection_info* out);

/* Collection::SearchBatch: nq raw queries (nq x dim, host or device; prepared on the GPU as
 * PrepareQuery does), one filter (JSON, the language of src/meta/filter.h; NULL = none) for
 * all. out_ids (nq x k) / out_dist (nq x k), host or device: misses UINT64_MAX / +inf. Errors:
 * VDBGPU_INVALID_ARGUMENT for a bad filter, k outside 1..10000, a non-finite or (cosine) zero
 * query, with the reference's messages; VDBGPU_NOT_SUPPORTED for k > 240. */
VDBGPU_API int vdbgpu_collection_search(vdbgpu_collection* c, const float* queries, uint64_t nq,
                                        uint32_t k, const vdbgpu_search_params* params,
                                        const char* filter_json, uint64_t* out_ids,
                                        float* out_dist);

/* Several filters in one batch: query i uses filters[query_filter[i]] (-1 = no filter);
 * query_filter NULL = filters[0] for all. Results as nfilters separate SearchBatch calls over
 * each filter's queries. out_hits (nq x k, host or device, nullable) receives the merged hit
 * records (the input of vdbgpu_merge_hits on another rank). */
VDBGPU_API int vdbgpu_collection_search_grouped(vdbgpu_collection* c, const float* queries,
                                                uint64_t nq, uint32_t k,
                                                const vdbgpu_search_params* params,
                                                const char* const* filters, uint32_t nfilters,
                                                const int32_t* query_filter, uint64_t* out_ids,
                                                float* out_dist, vdbgpu_hit* out_hits);

/* Work counters of the collection's last search (the batch form of SearchExplain's
 * distance_computations): out[0] queries, [1] rows scored exactly (prefilter and exact
 * fallback, summed over queries), [2] distance computations of index searches (counted only
 * while enabled), [3] prefilter (filter, segment) pairs, [4] filtered-index pairs, [5] post-filter
 * pairs, [6] empty pairs, [7] filter bitmap words evaluated, [8] (query, segment) index searches,
 * [9..12] host wall microseconds of the filter bitmaps and planning, the exact searches over
 * bitmaps, the index searches, and the rest of the call. enable: 1 / 0 turns the index-search count on / off, -1 leaves it. Returns the count written. */
VDBGPU_API int vdbgpu_collection_stats(vdbgpu_collection* c, int enable, uint64_t* out, int cap);

/* Collection::Search with explain for one query: JSON array with one object per local segment,
 * the mutable segment first {"id", "kind" ("mutable" / "disk"), "strategy", "matches",
 * "live_rows", "distance_computations", "results"}
 * (SegmentExplain, include/vdb/collection.h:45-58). Returns VDBGPU_RESOURCE_EXHAUSTED when cap
 * is too small. */
VDBGPU_API int vdbgpu_collection_explain(vdbgpu_collection* c, const float* query, uint32_t k,
                                         const vdbgpu_search_params* params,
                                         const char* filter_json, char* out_json, size_t cap);

/* SegmentColumns::Evaluate (src/meta/columns.cc:185-250) of a filter on one segment, minus its
 * deleted rows (planner.cc:64-65): out_words receives (rows + 31) / 32 words (bit r of word
 * r / 32, host or device), matches (nullable) the number of rows. */
VDBGPU_API int vdbgpu_collection_filter_bitmap(vdbgpu_collection* c, const char* filter_json,
                                               uint32_t segment_id, uint32_t* out_words,
                                               uint64_t* matches);

/* The merge of CollectionImpl::Search over lists of hits that are each already merged
 * (ascending (dist, part, row), one hit per id): lists = nlists x nq x k records (host or
 * device), e.g. the per-GPU results of a sharded collection gathered over NCCL. Writes the
 * first k distinct ids per query. out_hits nullable. */
VDBGPU_API int vdbgpu_merge_hits(vdbgpu_ctx* ctx, const vdbgpu_hit* lists, uint32_t nlists,
                                 uint64_t nq, uint32_t k, uint64_t* out_ids, float* out_dist,
                                 vdbgpu_hit* out_hits);

/* ------------------------------------------------------- collections sharded over GPUs
 *
 * The exchange step of a collection whose disk segments are spread over the GPUs of one node
 * (vdbgpu_collection_open with shard / nshards, one process or thread per GPU). The reference has
 * no sharding: it searches every segment and merges the per-segment lists in one process
 * (CollectionImpl::Search, src/engine/collection_impl.cc:1056-1108). Each rank merges its own
 * segments with vdbgpu_collection_search_grouped (out_hits); vdbgpu_shard_merge moves those k
 * records per query between ranks with NCCL over NVLink and runs the same merge on the receiving
 * GPU, which gives the unsharded result. NCCL (libnccl.so.2) is loaded on first use; without it
 * these calls return VDBGPU_UNAVAILABLE. */

#define VDBGPU_SHARD_ID_BYTES 128

typedef struct vdbgpu_shard_group vdbgpu_shard_group;

/* A rendezvous token (ncclGetUniqueId) for one group: made on one rank, handed to every rank by the
 * host's own channel, VDBGPU_SHARD_ID_BYTES bytes. */
VDBGPU_API int vdbgpu_shard_id(void* out_id);

/* Joins the group as `rank` of `nranks` on the context's device (every rank calls it with the same
 * token). Every wait of the group (this rendezvous, each exchange) is bounded by timeout_ms (<= 0:
 * 60 s); a wait that runs out aborts the group and returns VDBGPU_UNAVAILABLE, as does an NCCL
 * failure. */
VDBGPU_API int vdbgpu_shard_group_open(vdbgpu_ctx* ctx, const void* id, int rank, int nranks,
                                       int timeout_ms, vdbgpu_shard_group** out);
VDBGPU_API void vdbgpu_shard_group_close(vdbgpu_shard_group* g);

/* The exchange: every rank's local nq x k merged records (host or device memory of the context's
 * device) go to every rank (root < 0, an all-gather) or to `root` alone (a gather), and the
 * receiving ranks merge the nranks lists as vdbgpu_merge_hits does (out_ids / out_dist / out_hits
 * host or device, nullable; ignored on ranks that do not receive). Every rank must call it with
 * the same nq, k and root, in the same order. After a failure the group is aborted and further
 * calls return VDBGPU_FAILED_PRECONDITION. */
VDBGPU_API int vdbgpu_shard_merge(vdbgpu_shard_group* g, const vdbgpu_hit* local, uint64_t nq,
                                  uint32_t k, int root, uint64_t* out_ids, float* out_dist,
                                  vdbgpu_hit* out_hits);

/* Index::build for HNSW (HnswIndex, src/index/hnsw/hnsw_index.h:12-41) on the GPU: a graph over
 * nrows rows (nrows x padded_dim floats, host or device; cosine rows already normalised) with
 * M links per upper layer and 2M on layer 0, returned as a complete index file in the
 * reference's format (HnswIndex::save, hnsw_index.cc:36-41), readable by vdbgpu_index_load,
 * vdbgpu_collection_add_segment and the reference's LoadIndex. Nodes are linked by
 * HnswGraph's neighbour heuristic (hnsw_graph.h:569-616) applied to every node's `candidates`
 * exact nearest neighbours (0 = 4M, at most 127) instead of the reference's one-at-a-time
 * insertion, so the graph is not the reference's. Levels follow level_for (hnsw_graph.h:
 * 470-474) with `seed`. *out_file is malloc'd; release it with vdbgpu_buffer_free. */
VDBGPU_API int vdbgpu_hnsw_build(vdbgpu_ctx* ctx, int metric, const float* rows, uint64_t nrows,
                                 uint32_t dim, uint32_t padded_dim, uint32_t M, uint32_t candidates,
                                 uint64_t seed, void** out_file, size_t* out_bytes);

/* HnswIndex::extend (src/index/hnsw/hnsw_index.cc:50-58) on the GPU: the index.hnsw file
 * (file_bytes, the graph over the first rows) with the remaining rows of `rows` (nrows x
 * padded_dim floats, host or device, nrows >= the graph's rows) inserted, as a complete index
 * file in the same format (the graph's M, seed and ef_construction field kept). New nodes take
 * level_for's levels with the graph's seed; each links to select_neighbors of its exact nearest
 * neighbours among the old nodes and the new nodes inserted up to its round, and back links
 * re-prune full lists with the heuristic, as vdbgpu_hnsw_build does. The reference's extend
 * inserts one node at a time on host threads (order-dependent); this graph is valid in the same
 * format, not the same graph. Only HNSW files (not HNSW-SQ8, PQ or IVF-PQ, which the reference
 * cannot extend either: VDBGPU_NOT_SUPPORTED). *out_file is malloc'd; release it with
 * vdbgpu_buffer_free. */
VDBGPU_API int vdbgpu_hnsw_extend(vdbgpu_ctx* ctx, int metric, const void* file_bytes, size_t nbytes,
                                  const float* rows, uint64_t nrows, uint32_t dim, uint32_t padded_dim,
                                  void** out_file, size_t* out_bytes);

/* Index::build + save for IVF-PQ (type VDBGPU_INDEX_IVF_PQ) and PQ-flat (VDBGPU_INDEX_PQ_FLAT) on
 * the GPU (IvfPqIndex::build, src/index/quant/ivf_pq.cc:106-150; PqFlatIndex::build, :45-58):
 * the reference's seeded k-means (kmeans.cc:55-174) replayed exactly (host RNG and sums, GPU
 * nearest-centroid searches in the reference kernel set's summation order), so the returned
 * file is the reference's own index file, byte for byte, for the same rows (nrows x padded_dim
 * floats, host or device), nlist, pq_m, max_train_points_per_centroid and seed. Padded
 * dimensions up to 256 and sub-vectors (dim / pq_m) up to 64 floats; larger requests return
 * VDBGPU_NOT_SUPPORTED. *out_file is malloc'd; release it with vdbgpu_buffer_free. */
VDBGPU_API int vdbgpu_ivfpq_build(vdbgpu_ctx* ctx, int type, const float* rows, uint64_t nrows,
                                  uint32_t dim, uint32_t padded_dim, uint32_t nlist, uint32_t pq_m,
                                  uint32_t max_train_ppc, uint64_t seed, void** out_file,
                                  size_t* out_bytes);

/* Releases a buffer returned by the library (vdbgpu_hnsw_build, vdbgpu_ivfpq_build). */
VDBGPU_API void vdbgpu_buffer_free(void* p);

/* Applies write-ahead log records to a collection opened with vdbgpu_collection_open, as recovery
 * replays them (ApplyOp, src/engine/collection_impl.cc:574-599): `records` are the bytes the
 * reference appends to its log for a write batch (WalWriter::append, src/storage/wal.cc: records
 * framed as in a log file, without the 16-byte file header). Upserts are appended to the mutable
 * segment (rebuilt on shard 0), and the old rows of upserted or deleted ids are deleted on this
 * shard's segments. Records at or below the last applied LSN are skipped, so a batch may overlap
 * what the directory's log already held; an LSN gap is VDBGPU_CORRUPTION and a damaged record
 * VDBGPU_INVALID_ARGUMENT (or VDBGPU_CORRUPTION for a well-framed record with a bad payload), each
 * after the records before it were applied; the refused record is not consumed and may be sent
 * again. *applied (nullable) = records applied. A flush of the reference (a new disk segment) is followed by reopening. */
VDBGPU_API int vdbgpu_collection_apply_log(vdbgpu_collection* c, const void* records, size_t bytes,
                                           uint64_t* applied);

/* The recovery of vdbgpu_collection_open (manifest, delete sets, log replay) on the host, without
 * a GPU, reported as Collection::Stats (src/engine/collection_impl.cc:1168-1225): JSON
 * {"live_rows", "total_rows", "deleted_rows", "last_lsn", "flushed_lsn", "recovery_records",
 * "segments": [{"id", "kind", "index", "rows", "deleted", "lsn"}]}, the mutable segment first.
 * On error out_json holds the message and the status code is returned; VDBGPU_RESOURCE_EXHAUSTED
 * when cap is too small (out_json then holds a truncated prefix). Reads only. */
VDBGPU_API int vdbgpu_collection_inspect(const char* path, char* out_json, size_t cap);

/* FilterExpr::Parse (src/meta/filter_parser.cc) against a schema (JSON, schema.cc:246-270),
 * without a GPU: VDBGPU_OK with the parsed filter's description (FilterExpr::ToString) in out,
 * or the reference's status code with its message in out. */
VDBGPU_API int vdbgpu_filter_describe(const char* schema_json, const char* filter_json, char* out,
                                      size_t cap);

#ifdef __cplusplus
}
#endif
#endif /* VDBGPU_H_ */
