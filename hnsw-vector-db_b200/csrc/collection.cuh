// Kernels of the multi-segment read path (CollectionImpl::Search, src/engine/collection_impl.cc:
// 1036-1119, and SearchDiskSegment, src/engine/planner.cc:42-129) on the GPU:
//
//   prepare_queries   PrepareQuery (collection_impl.cc:1023-1034): pad, finite check, cosine
//                     NormalizeVector (src/util/dataset.cc:33-40) in the same double arithmetic
//   leaf_range        numeric leaves of SegmentColumns::Leaf (src/meta/columns.cc:210-224) as
//                     per-row predicates over the value column (same sets as the sorted-array Range)
//   posting_scatter   keyword / keyword_list postings into a dense bitmap
//   filter_program    And / Or / Not / AndNot over leaf bitmaps (SegmentColumns::Evaluate,
//                     columns.cc:185-205) minus deleted rows, with the match count per segment
//   compact_rows      a bitmap into its rows in ascending order (the iteration order of
//                     ExactOverBitmap, planner.cc:31-38)
//   exact_rows        exact top-k over listed rows, fp32 distances in the reference kernel set's
//                     summation order (bit-exact)
//   pack_hits         index results into per-segment top-k lists (graph, post-filter, plain)
//   merge_parts       the merge of collection_impl.cc:1079-1108: order by (dist, part, row), one
//                     hit per external id, first k
//
// Bitmaps are dense: bit r of 32-bit word r / 32; every bitmap has `words` words, a multiple of 8
// (rows padded to 256, padding bits zero).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vdbgpu {

// ---- queries
cudaError_t LaunchPrepareQueries(const float* in, const uint32_t* perm, uint64_t nq, uint32_t dim,
                                 uint32_t pd, bool cosine, float* out, int* qstatus, cudaStream_t st);

// ---- leaf bitmaps
struct RangeTask {
  uint32_t* out;
  const uint32_t* present;
  const double* values;
  const double* set;  // In: the literal set (nset values); null: the range [lo, hi]
  double lo, hi;
  int lo_incl, hi_incl, nset;
  uint32_t words;
};
cudaError_t LaunchLeafRange(const RangeTask* tasks, int ntasks, uint32_t max_words, cudaStream_t st);

struct ScatterTask {
  uint32_t* out;
  const uint32_t* rows;
  uint32_t count;
};
cudaError_t LaunchPostingScatter(const ScatterTask* tasks, int ntasks, cudaStream_t st);

// ---- filter programs
enum ProgOp : int { kProgPush = 0, kProgAnd = 1, kProgOr = 2, kProgAndNot = 3, kProgNot = 4, kProgZero = 5 };
struct ProgInstr {
  int op;
  const uint32_t* bits;  // kProgPush
};
constexpr int kProgStack = 40;
constexpr int kProgChunkWords = 2048;  // words per CTA (256 threads x 8)

struct ProgramTask {
  const ProgInstr* prog;
  int nprog;
  uint32_t words;
  const uint32_t* all;       // rows mask (for Not)
  const uint32_t* deletes;   // deleted rows or null
  uint32_t* out;             // result bitmap or null (count only)
  uint32_t* chunk_counts;    // ceil(words / kProgChunkWords) counts
  unsigned long long* matches;
};
cudaError_t LaunchFilterProgram(const ProgramTask* tasks, int ntasks, uint32_t max_words, int* status,
                                cudaStream_t st);

struct CompactTask {
  const uint32_t* bits;
  uint32_t words;
  const uint32_t* chunk_counts;
  uint32_t* rows_out;
};
cudaError_t LaunchCompactRows(const CompactTask* tasks, int ntasks, uint32_t max_words, cudaStream_t st);

// ---- exact top-k over listed rows
struct ExactItem {
  const float* rows;        // segment rows, n x pd
  const uint32_t* list;     // ascending rows to score
  uint32_t count;
  uint32_t q0, nq;          // sorted queries [q0, q0 + nq), nq <= 4
  uint64_t* out;            // packed (dist, row) keys: query j at out + j * out_stride
  uint64_t* dc;             // distance computations of query j at dc[j * dc_stride] (+= count) or null
  const int* only_if;       // when set, query j is scored only if only_if[j * dc_stride] != 0
};
struct ExactArgs {
  const ExactItem* items;
  int nitems;
  const float* queries;     // prepared, sorted, nq x pd
  int pd, k, metric, order;
  uint64_t out_stride, dc_stride;
  int* status;
};
cudaError_t LaunchExactRows(const ExactArgs& a, cudaStream_t st);

// ---- index results -> per-segment lists
struct PackItem {
  const float* dist;        // nq x kin
  const uint32_t* row;
  uint32_t kin, nq;
  const uint32_t* keep;     // post-filter bitmap or null
  uint32_t need;            // graph: queries with fewer valid results get short[q] = 1
  uint64_t* out;            // query j at out + j * out_stride
  int* short_flag;          // query j at short_flag[j * flag_stride] or null
};
cudaError_t LaunchPackHits(const PackItem* items, int nitems, uint32_t max_nq, int k, uint64_t out_stride,
                           uint64_t flag_stride, cudaStream_t st);

// ---- merge
struct HitRecord {  // one merged hit: ordered by (dist, part, row); 24 bytes
  float dist;
  uint32_t part;
  uint32_t row;
  uint32_t pad;
  uint64_t id;
};
struct MergeArgs {
  // Per-segment lists (kind 0): parts x nq x k packed keys, part p's global number part_no[p],
  // its external ids ids[p]. Per-rank lists (kind 1): lists x nq x k HitRecords.
  int kind;
  int nlists, k;
  uint64_t nq;
  const uint64_t* keys;
  const uint32_t* part_no;
  const uint64_t* const* ids;
  const HitRecord* records;
  HitRecord* out_records;   // nq x k (row perm[q]) or null
  uint64_t* out_ids;        // nq x k (row perm[q]) or null
  float* out_dist;
  const uint32_t* perm;     // sorted query -> caller's query, or null
};
cudaError_t LaunchMerge(const MergeArgs& a, cudaStream_t st);

}  // namespace vdbgpu
