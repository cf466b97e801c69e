// The on-disk side of a collection directory written by the reference, on the host: file reads,
// blob framing, persisted delete sets, options and manifest, metadata rows, write-ahead log
// records, and the recovery that Collection::Open runs (CollectionImpl::Recover,
// src/engine/collection_impl.cc:76-235) before anything is uploaded to a GPU.
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include "collection.h"
#include "formats.h"

namespace vdbgpu {

constexpr size_t kSegmentHeaderSize = 4096;  // src/storage/segment.h:33

template <class T>
T GetAt(const char* p, size_t off) {
  T v;
  std::memcpy(&v, p + off, sizeof(T));
  return v;
}

inline uint32_t PaddedDim(uint32_t d) { return (d + 15) / 16 * 16; }  // include/vdb/types.h:30-32

// Whole-file reads as PosixEnv::read_file (src/storage/posix_env.cc:99-124); ReadPrefix reads
// the first n bytes and reports the file's size.
Status ReadFile(const std::string& path, std::string* out);
Status ReadPrefix(const std::string& path, size_t n, std::string* out, uint64_t* size);
// DecodeBlob (src/storage/file_format.cc:20-33): [magic 8][u32 version][u32 crc32c][u64 len].
Status DecodeBlob(std::string_view file, std::string_view magic, std::string_view* payload);
// A persisted delete set (CRoaring's portable serialization) as (rows + 31) / 32 words.
Status DecodeDeleteSet(std::string_view p, uint64_t rows, std::vector<uint32_t>* words);

bool ParseMetricName(const std::string& s, int* m);
bool ParseIndexTypeName(const std::string& s, int* t);
const char* IndexFileName(int t);
// OptionsFromJson as recovery applies it to a manifest's options (no range checks).
Status ManifestOptionsFromJson(const JsonValue& j, CollectionOptions* o);

struct RowValue {  // one decoded field of one row (the last occurrence wins, as DecodeMetaRow)
  bool has = false;
  double num = 0;
  bool b = false;
  std::vector<std::string> strs;
};

// One row of EncodeMetaRow (src/meta/schema.cc:97-124) into row; false when malformed.
bool DecodeMetaRowValues(const Schema& schema, std::string_view data, std::vector<RowValue>* rowp);

// One write-ahead log record (src/storage/wal.cc framing).
struct WalRecordView {
  uint8_t type = 0;
  uint64_t lsn = 0;
  std::string_view payload;
};
bool TryParseWalRecord(std::string_view data, size_t pos, WalRecordView* rec, size_t* len);

// vectors.f32 header checks of Segment::Open (segment_reader.cc:36-51).
Status CheckSegmentHeader(const std::string& dir, const char* h, uint64_t file_size, uint64_t rows,
                          const CollectionOptions& opt);

// One disk segment of the manifest, with its ids and delete bits once read.
struct SegEntry {
  uint32_t id = 0;
  uint64_t rows = 0, lsn = 0;
  std::string deletes_file, dir;
  std::vector<uint64_t> ids;  // read for the id map, then released
  std::vector<uint32_t> del;  // (rows + 31) / 32 words; empty until read
};

Status LoadIds(SegEntry* e);
Status LoadDeletes(SegEntry* e);

// The mutable segment rebuilt from the logs (MutableSegment, src/engine/mutable_segment.h):
// rows appended in log order, padded to pd floats, with their external ids, metadata rows and
// delete bits.
struct MutableRows {
  uint64_t n = 0;
  uint64_t max_lsn = 0;   // of the rows appended (MutableSegment::max_lsn)
  uint64_t last_lsn = 0;  // the collection's
  uint64_t records = 0;   // records replayed at open
  std::vector<float> rows;
  std::vector<uint64_t> ids;
  std::vector<std::string> meta;
  std::vector<uint32_t> del;
  // meta.bin's payload for these rows: u64 rows, u64 offsets[rows + 1], the rows.
  std::string MetaPayload() const {
    std::string out(8 * (n + 2), '\0');
    std::memcpy(&out[0], &n, 8);
    uint64_t off = 0;
    for (uint64_t i = 0; i <= n; ++i) {
      std::memcpy(&out[8 * (i + 1)], &off, 8);
      if (i < n) off += meta[i].size();
    }
    for (const auto& m : meta) out += m;
    return out;
  }
};

constexpr uint64_t kMutableMaxRows = uint64_t{1} << 26;  // MutableSegment::kDefaultMaxRows

// The external-id map and ApplyOp's rule for one record (collection_impl.cc:574-599, replay
// form): the id's old row is deleted unless the segment holding it is at least as new as the
// record, in which case an upserted row is appended already deleted.
struct LogApplier {
  struct Loc {
    int64_t seg;  // index into segs, -1 = the mutable segment
    uint32_t row;
  };
  std::unordered_map<uint64_t, Loc> ids;
  std::vector<bool> touched;  // disk segments whose delete bits changed
  uint64_t expected = 1;      // the LSN the next record must carry

  // Recover step 4: live rows of every segment, oldest segment first.
  void Build(const std::vector<SegEntry>& segs);

  // Applies one record: records at or below skip_below are skipped, any other must carry the
  // expected LSN.
  Status Apply(const WalRecordView& rec, uint64_t skip_below, const CollectionOptions& opt,
               std::vector<SegEntry>& segs, MutableRows* mut);
};

// What a collection keeps on the host after Open: the manifest's segments (delete bits, lsn; ids
// only while the id map is built), the mutable segment's rows, and the id map once a log record
// has been applied.
struct RecoveryState {
  std::string path;
  uint32_t shard = 0, nshards = 1;
  uint32_t mutable_id = 0;
  uint64_t flushed_lsn = 0;
  std::vector<SegEntry> segs;
  MutableRows mut;
  LogApplier ap;
  bool have_map = false;
};

// The directory as Collection::Open recovers it: options, segments with their delete bits (those
// of shard `shard` of nshards, or of every segment when the logs hold records or `all`), and the
// mutable segment replayed from the logs. Reads only.
Status RecoverDir(const std::string& path, uint32_t shard, uint32_t nshards, bool all, CollectionOptions* opt,
                  RecoveryState* d);

}  // namespace vdbgpu
