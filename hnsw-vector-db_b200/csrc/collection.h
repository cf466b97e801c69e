// The engine read path on the GPU: a collection's on-disk segments (Segment, src/storage/
// segment.h; opened as Segment::Open does, src/storage/segment_reader.cc:20-122) with their
// metadata columns (SegmentColumns, src/meta/columns.h), the per-segment planner
// (SearchDiskSegment, src/engine/planner.cc:42-129) and the merge of CollectionImpl::Search
// (src/engine/collection_impl.cc:1036-1119), batched over queries (SearchBatch, :1121-1136).
//
// A batch carries one or more filters; each query names the filter it uses (or none). Queries
// are grouped by filter, every (filter, segment) pair is planned as the reference plans it for
// a single query (the plan depends only on the match count, the live rows, ef, k and the index
// type), and the searches of all pairs run batched on the GPU.
#pragma once

#include <memory>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "collection.cuh"
#include "filter.h"
#include "runtime.h"

namespace vdbgpu {

struct CollectionOptions {  // the part of vdb::CollectionOptions the read path uses
  uint32_t dim = 0, pd = 0;
  int metric = 0;       // 0 l2, 1 ip, 2 cosine (vdb::Metric)
  int index_type = 1;   // IndexKind of every segment
  Schema schema;
};
Status CollectionOptionsFromJson(const JsonValue& j, CollectionOptions* o);

// One metadata column of a segment (SegmentColumns::Column, src/meta/columns.h:44-59).
struct GpuColumn {
  FieldType type = FieldType::Int64;
  DeviceBuffer present;                          // bitmap
  DeviceBuffer values;                           // int64 / float64: the value as a double per row
  std::unordered_map<std::string, int32_t> dict; // keyword / keyword_list: value -> code
  std::vector<uint64_t> post_off;                // host: postings of code c at [off[c], off[c+1])
  DeviceBuffer post_rows;                        // ascending rows per code
  DeviceBuffer true_rows, false_rows;            // bool
};

struct GpuSegment {
  uint32_t id = 0;
  uint32_t ordinal = 0;  // the merge's part order: 0 the mutable segment, then disk segments
  bool is_mutable = false;  // rebuilt from the log; always searched exhaustively
  uint64_t rows = 0, words = 0;
  uint64_t deleted = 0;
  std::unique_ptr<GpuIndex> index;
  DeviceBuffer ids;       // external ids (VectorId) per row
  DeviceBuffer all;       // rows mask
  DeviceBuffer deletes;   // deleted rows, or empty
  DeviceBuffer live;      // all & ~deletes, or empty
  std::vector<GpuColumn> cols;
};

// SegmentExplain (include/vdb/collection.h:45-58) of one segment for one query.
struct PartExplain {
  uint32_t segment_id = 0;
  bool is_mutable = false;
  std::string strategy;
  uint64_t live_rows = 0, matches = 0, dc = 0, results = 0;
};

struct RecoveryState;  // collection_store.h

class GpuCollection {
 public:
  // Opens a collection directory written by the reference (CURRENT -> MANIFEST-<n> -> segments,
  // their delete sets, then the logs replayed into the mutable segment). With nshards > 1 only
  // the segments whose manifest position % nshards == shard are loaded; shard 0 holds the
  // mutable segment.
  static Status Open(Context& ctx, const std::string& path, uint32_t shard, uint32_t nshards,
                     std::unique_ptr<GpuCollection>* out);
  // The same recovery on the host only, reported as Collection::Stats (collection_impl.cc:
  // 1168-1225): JSON {live_rows, total_rows, deleted_rows, last_lsn, flushed_lsn,
  // recovery_records, segments: [{id, kind, index, rows, deleted, lsn}]}, the mutable segment first.
  static Status Inspect(const std::string& path, std::string* json);
  // Applies log records (the bytes the reference appends to its log for a write batch: records
  // framed as in a log file, without the file header) as recovery replays them: deletes of old
  // rows on this shard's disk segments, upserts appended to the mutable segment (rebuilt on shard
  // 0). Records at or below the last applied LSN are skipped; a gap or a damaged record fails the
  // call after the records before it were applied. *applied = records applied. Only for
  // collections opened from a directory.
  Status ApplyLog(Context& ctx, std::string_view records, uint64_t* applied);
  // An empty collection with the reference's options JSON (engine/options_json.cc), to which
  // segments are added from their files' contents.
  static Status Create(std::string_view options_json, std::unique_ptr<GpuCollection>* out);
  // rows: n x pd floats (host or device), as in vectors.f32 after its header; ids: n external
  // ids (host); meta: the payload of meta.bin (empty = no metadata); index_file: the index file.
  Status AddSegment(Context& ctx, uint32_t id, uint32_t ordinal, const float* rows, uint64_t n,
                    const uint64_t* ids, std::string_view meta, std::string_view index_file);
  // Marks rows of a segment deleted (bit r of word r / 32; null = none).
  Status SetDeleted(Context& ctx, uint32_t segment_id, const uint32_t* bits_host);

  struct Request {
    const float* queries = nullptr;  // nq x dim (host or device)
    uint64_t nq = 0;
    uint32_t k = 10;
    SearchParams params;
    std::vector<std::string> filters;   // filter JSON texts
    const int32_t* query_filter = nullptr;  // host, per query: index into filters or -1 (none);
                                            // null: every query uses filters[0] (none if empty)
    uint64_t* out_ids = nullptr;        // nq x k (host or device) or null
    float* out_dist = nullptr;
    HitRecord* out_records = nullptr;   // nq x k merged records (host or device) or null
    std::vector<std::vector<PartExplain>>* explain = nullptr;  // per query, per local segment
  };
  Status Search(Context& ctx, const Request& r);
  // The rows of one segment that a filter selects, minus deleted rows (SegmentColumns::Evaluate,
  // src/meta/columns.cc:185-250; planner.cc:64-65): (rows + 31) / 32 words into out (host or
  // device), the count into *matches.
  Status FilterBitmap(Context& ctx, std::string_view filter, uint32_t segment_id, uint32_t* out,
                      uint64_t* matches);

  // A filter leaf as the GPU evaluates it (collection_host.cc).
  struct LeafSpec;

  // Work of the last Search: [0] queries, [1] rows scored exactly (prefilter and fallback, per
  // query), [2] distance computations of index searches (only while stats are enabled), [3]
  // prefilter pairs, [4] filtered-index pairs, [5] post-filter pairs, [6] empty pairs, [7] filter
  // bitmap words evaluated, [8] (query, segment) index searches; [9..12] host wall microseconds of
  // filter bitmaps + planning, exact search over bitmaps, index searches, and the rest.
  static constexpr int kStats = 13;
  void set_stats(bool on) { stats_on_ = on; }
  const uint64_t* stats() const { return stats_; }

  const CollectionOptions& options() const { return opt_; }
  uint32_t segments_total() const { return total_segments_; }
  size_t segments_local() const { return segs_.size(); }
  uint64_t rows_local() const;
  uint64_t device_bytes() const;

 private:
  struct Batch;
  Status SearchGroups(Context& ctx, Batch& b);
  Status Bitmaps(Context& ctx, Batch& b, const std::vector<uint32_t>& fq, size_t s0, size_t cs,
                 std::vector<uint64_t>* matches);
  uint64_t MaxWords() const;
  Status UploadMutable(Context& ctx);
  size_t SegmentsPerChunk(const Batch& b, size_t nfilters) const;
  uint32_t* PairBits(size_t fi, size_t si, size_t cs) const;
  Status RunIndex(Context& ctx, Batch& b, size_t s, uint32_t g, uint32_t kk, const SearchParams& p,
                  const uint32_t* allow, const uint32_t* keep, uint32_t need, int* short_flags);

  CollectionOptions opt_;
  uint32_t total_segments_ = 0;
  bool stats_on_ = false;
  uint64_t stats_[kStats] = {};
  std::vector<std::unique_ptr<GpuSegment>> segs_;
  std::shared_ptr<RecoveryState> log_;  // host recovery state (collections opened from a directory)
  // Per-batch device scratch (grow-only).
  MultiScratch multi_;
  DeviceBuffer q_raw_, perm_, prepared_, qstatus_, keys_, dc_, short_, leafbits_, pairbits_,
      counts_, matches_, rowlists_, tmp_dist_, tmp_row_, tasks_, merged_, out_ids_, out_dist_;
};

}  // namespace vdbgpu
