#include "collection.h"

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <unordered_map>

#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include "formats.h"
#include "hnsw.cuh"

namespace vdbgpu {

namespace {

uint64_t NowUs() {
  return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::microseconds>(
                                   std::chrono::steady_clock::now().time_since_epoch())
                                   .count());
}

constexpr size_t kSegmentHeaderSize = 4096;  // src/storage/segment.h:33
constexpr size_t kBlobHeaderSize = 24;       // src/storage/file_format.h:13
constexpr uint64_t kMaxK = 10000;            // include/vdb/collection.h kMaxK
constexpr uint32_t kMaxGpuK = 240;
constexpr uint32_t kScatterChunk = 16384;

uint64_t RoundUp(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

// Whole-file reads as the reference's PosixEnv::read_file (src/storage/posix_env.cc:99-124):
// errors are IOError "<call> <path>: <strerror>". With a limit, only the first `limit` bytes.
Status ErrnoStatus(const char* what, const std::string& path, int err) {
  return Status(Status::kIOError, std::string(what) + " " + path + ": " + std::strerror(err));
}

Status ReadFileLimit(const std::string& path, uint64_t limit, std::string* out, uint64_t* size) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return ErrnoStatus("open", path, errno);
  struct stat st {};
  if (::fstat(fd, &st) != 0) {
    const int e = errno;
    ::close(fd);
    return ErrnoStatus("stat", path, e);
  }
  if (size != nullptr) *size = static_cast<uint64_t>(st.st_size);
  out->resize(static_cast<size_t>(std::min<uint64_t>(limit, static_cast<uint64_t>(st.st_size))));
  size_t got = 0;
  while (got < out->size()) {
    const ssize_t n = ::read(fd, &(*out)[got], out->size() - got);
    if (n < 0) {
      if (errno == EINTR) continue;
      const int e = errno;
      ::close(fd);
      return ErrnoStatus("read", path, e);
    }
    if (n == 0) break;
    got += static_cast<size_t>(n);
  }
  out->resize(got);
  ::close(fd);
  return Status::OK();
}

Status ReadFile(const std::string& path, std::string* out) { return ReadFileLimit(path, UINT64_MAX, out, nullptr); }

// The first n bytes of a file (fewer if it is shorter) and its size.
Status ReadPrefix(const std::string& path, size_t n, std::string* out, uint64_t* size) {
  return ReadFileLimit(path, n, out, size);
}

template <class T>
T GetAt(const char* p, size_t off) {
  T v;
  std::memcpy(&v, p + off, sizeof(T));
  return v;
}

// DecodeBlob (src/storage/file_format.cc:20-33): [magic 8][u32 version][u32 crc32c][u64 len].
Status DecodeBlob(std::string_view file, std::string_view magic, std::string_view* payload) {
  if (file.size() < kBlobHeaderSize) return Status(Status::kCorruption, "file shorter than its header");
  if (file.substr(0, magic.size()) != magic) return Status(Status::kCorruption, "bad file magic");
  const uint32_t version = GetAt<uint32_t>(file.data(), 8);
  const uint32_t crc = GetAt<uint32_t>(file.data(), 12);
  const uint64_t len = GetAt<uint64_t>(file.data(), 16);
  if (version != 1) return Status(Status::kCorruption, "unsupported file version");
  if (len != file.size() - kBlobHeaderSize) return Status(Status::kCorruption, "file length mismatch");
  const std::string_view p = file.substr(kBlobHeaderSize);
  if (Crc32c(p.data(), p.size()) != crc) return Status(Status::kCorruption, "file checksum mismatch");
  *payload = p;
  return Status::OK();
}

// A delete file's payload (src/storage/segment_writer.cc:28-37 writes it with
// roaring::Roaring::write(buf, true)): CRoaring's portable serialization. Layout:
//   cookie u32: 12346 (no run containers), followed by the container count u32; or
//               12347 | (count - 1) << 16, followed by a bitset of (count + 7) / 8 bytes that
//               marks run containers;
//   count × (key u16, cardinality - 1 u16), the high 16 bits of the values and their number;
//   count × u32 byte offsets of the containers (absent with runs and count < 4);
//   the containers: a run container is u16 n, then n × (start u16, length - 1 u16); otherwise
//   cardinality > 4096 is a bitmap of 1024 u64 words, else an array of u16 values.
// The set becomes the segment's delete bits, (rows + 31) / 32 words; like Segment::Open
// (src/storage/segment_reader.cc:107-115) a value at or past rows is corruption.
Status DecodeDeleteSet(std::string_view p, uint64_t rows, std::vector<uint32_t>* words) {
  const Status bad(Status::kCorruption, "bad delete set");
  size_t at = 0;
  auto need = [&](size_t n) { return at <= p.size() && p.size() - at >= n; };
  auto u16 = [&]() { const uint16_t x = GetAt<uint16_t>(p.data(), at); at += 2; return x; };
  auto u32 = [&]() { const uint32_t x = GetAt<uint32_t>(p.data(), at); at += 4; return x; };
  words->assign((rows + 31) / 32, 0u);
  if (!need(4)) return bad;
  const uint32_t cookie = u32();
  uint32_t count = 0;
  bool runs = false;
  std::string_view runbits;
  if ((cookie & 0xFFFFu) == 12347u) {
    runs = true;
    count = (cookie >> 16) + 1;
    if (!need((count + 7) / 8)) return bad;
    runbits = p.substr(at, (count + 7) / 8);
    at += (count + 7) / 8;
  } else if (cookie == 12346u) {
    if (!need(4)) return bad;
    count = u32();
    if (count > 65536) return bad;
  } else {
    return bad;
  }
  if (!need(4 * static_cast<size_t>(count))) return bad;
  std::vector<uint16_t> keys(count);
  std::vector<uint32_t> cards(count);
  for (uint32_t i = 0; i < count; ++i) {
    keys[i] = u16();
    cards[i] = static_cast<uint32_t>(u16()) + 1;
    if (i > 0 && keys[i] <= keys[i - 1]) return bad;
  }
  if (!runs || count >= 4) {
    if (!need(4 * static_cast<size_t>(count))) return bad;
    at += 4 * static_cast<size_t>(count);
  }
  const Status range(Status::kCorruption, "delete set out of range");
  auto set = [&](uint64_t v) {
    if (v >= rows) return false;
    (*words)[v / 32] |= 1u << (v % 32);
    return true;
  };
  for (uint32_t i = 0; i < count; ++i) {
    const uint64_t hi = static_cast<uint64_t>(keys[i]) << 16;
    if (runs && (static_cast<uint8_t>(runbits[i / 8]) >> (i % 8) & 1u)) {
      if (!need(2)) return bad;
      const uint32_t n = u16();
      if (!need(4 * static_cast<size_t>(n))) return bad;
      for (uint32_t r = 0; r < n; ++r) {
        const uint32_t start = u16(), len = u16();
        if (start + len > 0xFFFFu) return bad;
        if (hi + start + len >= rows) return range;
        for (uint32_t x = start; x <= start + len; ++x) set(hi + x);
      }
    } else if (cards[i] > 4096) {
      if (!need(8192)) return bad;
      for (uint32_t w = 0; w < 1024; ++w) {
        const uint64_t bits = GetAt<uint64_t>(p.data(), at + 8 * w);
        for (uint64_t b = bits; b != 0; b &= b - 1)
          if (!set(hi + 64 * w + static_cast<uint32_t>(__builtin_ctzll(b)))) return range;
      }
      at += 8192;
    } else {
      if (!need(2 * static_cast<size_t>(cards[i]))) return bad;
      for (uint32_t k = 0; k < cards[i]; ++k)
        if (!set(hi + u16())) return range;
    }
  }
  return Status::OK();
}

bool OnDevice(const void* p) {
  if (p == nullptr) return false;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

bool ParseMetricName(const std::string& s, int* m) {
  if (s == "l2" || s == "L2" || s == "euclidean") *m = 0;
  else if (s == "ip" || s == "inner_product" || s == "dot") *m = 1;
  else if (s == "cosine" || s == "angular") *m = 2;
  else return false;
  return true;
}

bool ParseIndexTypeName(const std::string& s, int* t) {
  if (s == "flat") *t = kIndexFlat;
  else if (s == "hnsw") *t = kIndexHnsw;
  else if (s == "hnsw_sq8" || s == "sq8") *t = kIndexHnswSq8;
  else if (s == "pq" || s == "pq_flat") *t = kIndexPqFlat;
  else if (s == "ivf_pq" || s == "ivfpq") *t = kIndexIvfPq;
  else return false;
  return true;
}

// IndexFileName (src/storage/segment_writer.cc:21) with IndexTypeName (src/util/status.cc:55-64).
const char* IndexFileName(int t) {
  switch (t) {
    case kIndexFlat: return "index.flat";
    case kIndexHnsw: return "index.hnsw";
    case kIndexHnswSq8: return "index.hnsw_sq8";
    case kIndexPqFlat: return "index.pq";
    case kIndexIvfPq: return "index.ivf_pq";
  }
  return "index.unknown";
}

uint32_t PaddedDim(uint32_t d) { return (d + 15) / 16 * 16; }  // include/vdb/types.h:30-32

template <class T>
Status UploadVec(Context& ctx, const std::vector<T>& v, DeviceBuffer* out) {
  VDBGPU_RETURN_IF_ERROR(out->alloc(std::max<size_t>(1, v.size()) * sizeof(T)));
  if (!v.empty())
    VDBGPU_CUDA(cudaMemcpyAsync(out->get(), v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, ctx.stream()));
  return Status::OK();
}

// Copies n bytes of host structs into a grow-only device buffer at byte offset off (stream order).
Status Stage(Context& ctx, DeviceBuffer* buf, size_t off, const void* src, size_t n, void** dev) {
  *dev = static_cast<uint8_t*>(buf->get()) + off;
  if (n > 0) VDBGPU_CUDA(cudaMemcpyAsync(*dev, src, n, cudaMemcpyHostToDevice, ctx.stream()));
  return Status::OK();
}

}  // namespace

// OptionsFromJson (src/engine/options_json.cc:72-104): the fields the read path needs.
Status CollectionOptionsFromJson(const JsonValue& j, CollectionOptions* o) {
  if (!j.is_object()) return Status(Status::kInvalidArgument, "options must be a JSON object");
  const JsonValue* d = j.get("dim");
  if (d == nullptr || !d->is_integer() || (d->kind == JsonValue::kInt && d->i < 0))
    return Status(Status::kInvalidArgument, "dim must be a non-negative integer");
  const uint64_t dim = d->kind == JsonValue::kInt ? static_cast<uint64_t>(d->i) : d->u;
  if (dim == 0 || dim > 16384) return Status(Status::kInvalidArgument, "dim must be in 1..16384");
  o->dim = static_cast<uint32_t>(dim);
  o->pd = PaddedDim(o->dim);
  o->metric = 0;
  if (const JsonValue* m = j.get("metric")) {
    if (!m->is_string() || !ParseMetricName(m->s, &o->metric))
      return Status(Status::kInvalidArgument, "unknown metric (use l2, ip or cosine)");
  }
  o->index_type = kIndexHnsw;
  if (const JsonValue* idx = j.get("index")) {
    const JsonValue* t = idx->is_string() ? idx : idx->get("type");
    if (t != nullptr && (!t->is_string() || !ParseIndexTypeName(t->s, &o->index_type)))
      return Status(Status::kInvalidArgument, "unknown index type");
  }
  if (const JsonValue* s = j.get("schema")) VDBGPU_RETURN_IF_ERROR(SchemaFromJson(*s, &o->schema));
  return Status::OK();
}

// OptionsFromJson exactly as recovery applies it to the manifest's options
// (src/engine/options_json.cc:10-30, 55-106): every field's type is checked, no range is (Open
// does not run ValidateOptions); the read path keeps dim, metric, index type and schema.
Status ManifestOptionsFromJson(const JsonValue& j, CollectionOptions* o) {
  if (!j.is_object()) return Status(Status::kInvalidArgument, "options must be a JSON object");
  auto unsigned_of = [](const JsonValue& obj, const char* key, uint64_t* out) -> Status {
    const JsonValue* v = obj.get(key);
    if (v == nullptr) return Status::OK();
    if (v->kind != JsonValue::kUint && !(v->kind == JsonValue::kInt && v->i >= 0))
      return Status(Status::kInvalidArgument, std::string(key) + " must be a non-negative integer");
    if (out != nullptr) *out = v->kind == JsonValue::kUint ? v->u : static_cast<uint64_t>(v->i);
    return Status::OK();
  };
  auto number_of = [](const JsonValue& obj, const char* key) -> Status {
    const JsonValue* v = obj.get(key);
    if (v != nullptr && !v->is_number()) return Status(Status::kInvalidArgument, std::string(key) + " must be a number");
    return Status::OK();
  };
  uint64_t dim = 0;
  VDBGPU_RETURN_IF_ERROR(unsigned_of(j, "dim", &dim));
  o->dim = static_cast<uint32_t>(dim);
  o->pd = PaddedDim(o->dim);
  o->metric = 0;
  if (const JsonValue* m = j.get("metric")) {
    if (!m->is_string() || !ParseMetricName(m->s, &o->metric))
      return Status(Status::kInvalidArgument, "unknown metric (use l2, ip or cosine)");
  }
  o->index_type = kIndexHnsw;
  if (const JsonValue* idx = j.get("index")) {
    if (idx->is_string()) {
      if (!ParseIndexTypeName(idx->s, &o->index_type)) return Status(Status::kInvalidArgument, "unknown index type");
    } else if (!idx->is_null()) {
      if (!idx->is_object()) return Status(Status::kInvalidArgument, "index must be an object");
      if (const JsonValue* t = idx->get("type")) {
        if (!t->is_string() || !ParseIndexTypeName(t->s, &o->index_type))
          return Status(Status::kInvalidArgument, "unknown index type");
      }
      for (const char* k : {"M", "ef_construction", "pq_m", "m", "nlist", "max_train_points_per_centroid", "seed"})
        VDBGPU_RETURN_IF_ERROR(unsigned_of(*idx, k, nullptr));
    }
  }
  o->schema.clear();
  if (const JsonValue* s = j.get("schema")) VDBGPU_RETURN_IF_ERROR(SchemaFromJson(*s, &o->schema));
  if (const JsonValue* s = j.get("sync")) {
    if (!s->is_string() || (s->s != "always" && s->s != "interval" && s->s != "none"))
      return Status(Status::kInvalidArgument, "unknown sync mode (use always, interval or none)");
  }
  for (const char* k : {"sync_interval_ms", "flush_bytes", "flush_age_ms", "tier_base_rows", "tier_fanout"})
    VDBGPU_RETURN_IF_ERROR(unsigned_of(j, k, nullptr));
  VDBGPU_RETURN_IF_ERROR(number_of(j, "merge_into_largest_ratio"));
  VDBGPU_RETURN_IF_ERROR(number_of(j, "delete_compaction_ratio"));
  return Status::OK();
}

// ------------------------------------------------------------------------------- loading

Status GpuCollection::Create(std::string_view options_json, std::unique_ptr<GpuCollection>* out) {
  JsonValue j;
  if (!ParseJson(options_json, &j)) return Status(Status::kInvalidArgument, "options must be JSON");
  auto c = std::make_unique<GpuCollection>();
  VDBGPU_RETURN_IF_ERROR(CollectionOptionsFromJson(j, &c->opt_));
  *out = std::move(c);
  return Status::OK();
}

namespace {

// SegmentColumns::Build (src/meta/columns.cc:23-125) from meta.bin's payload: u64 rows,
// u64 offsets[rows + 1], then each row as EncodeMetaRow (src/meta/schema.cc:97-124).
struct HostColumn {
  std::vector<uint32_t> present, trues, falses;
  std::vector<double> values;
  std::unordered_map<std::string, int32_t> dict;
  std::vector<std::vector<uint32_t>> postings;
};

struct RowValue {  // one decoded field of one row (the last occurrence wins, as DecodeMetaRow)
  bool has = false;
  double num = 0;
  bool b = false;
  std::vector<std::string> strs;
};

// One row of EncodeMetaRow (src/meta/schema.cc:97-124) into row (fields it does not hold keep
// has = false; the last occurrence of a field wins, as DecodeMetaRow). False when malformed.
bool DecodeMetaRowValues(const Schema& schema, std::string_view data, std::vector<RowValue>* rowp) {
  std::vector<RowValue>& row = *rowp;
  for (auto& v : row) v.has = false;
  if (!data.empty()) {
    Reader rr(data);
    uint16_t count = 0;
    if (!rr.u16(&count)) return false;
    for (uint16_t k = 0; k < count; ++k) {
      uint16_t fid = 0;
      uint8_t type = 0;
      if (!rr.u16(&fid) || !rr.u8(&type) || fid >= schema.size()) return false;
      if (type != static_cast<uint8_t>(schema[fid].type)) return false;
      RowValue& v = row[fid];
      v.has = true;
      v.strs.clear();
      switch (static_cast<FieldType>(type)) {
        case FieldType::Int64: {
          int64_t x = 0;
          if (!rr.i64(&x)) return false;
          v.num = static_cast<double>(x);
          break;
        }
        case FieldType::Float64: {
          double x = 0;
          if (!rr.f64(&x)) return false;
          v.num = x;
          break;
        }
        case FieldType::Keyword: {
          uint32_t len = 0;
          std::string_view sv;
          if (!rr.u32(&len) || !rr.bytes(len, &sv)) return false;
          v.strs.emplace_back(sv);
          break;
        }
        case FieldType::KeywordList: {
          uint32_t cnt = 0;
          if (!rr.u32(&cnt) || cnt > rr.remaining() / 4) return false;
          for (uint32_t e = 0; e < cnt; ++e) {
            uint32_t len = 0;
            std::string_view sv;
            if (!rr.u32(&len) || !rr.bytes(len, &sv)) return false;
            v.strs.emplace_back(sv);
          }
          break;
        }
        case FieldType::Bool: {
          uint8_t b = 0;
          if (!rr.u8(&b)) return false;
          v.b = b != 0;
          break;
        }
        default: return false;
      }
    }
    if (rr.remaining() != 0) return false;
  }
  return true;
}

Status BuildColumns(const Schema& schema, uint64_t n, uint64_t words, std::string_view meta,
                    std::vector<HostColumn>* cols) {
  cols->assign(schema.size(), HostColumn{});
  for (size_t f = 0; f < schema.size(); ++f) {
    HostColumn& c = (*cols)[f];
    c.present.assign(words, 0);
    if (schema[f].type == FieldType::Int64 || schema[f].type == FieldType::Float64) c.values.assign(n, 0.0);
    if (schema[f].type == FieldType::Bool) {
      c.trues.assign(words, 0);
      c.falses.assign(words, 0);
    }
  }
  if (meta.empty()) return Status::OK();
  Reader r(meta);
  uint64_t rows = 0;
  std::string_view offs_bytes;
  if (!r.u64(&rows) || rows != n || !r.bytes((n + 1) * 8, &offs_bytes))
    return Status(Status::kCorruption, "bad meta.bin");
  std::vector<uint64_t> offs(n + 1);
  std::memcpy(offs.data(), offs_bytes.data(), offs_bytes.size());
  std::string_view bytes;
  r.bytes(r.remaining(), &bytes);
  for (uint64_t i = 0; i < n; ++i)
    if (offs[i] > offs[i + 1] || offs[i + 1] > bytes.size()) return Status(Status::kCorruption, "bad meta.bin offsets");
  std::vector<RowValue> row(schema.size());
  for (uint64_t ri = 0; ri < n; ++ri) {
    const std::string_view data = bytes.substr(offs[ri], offs[ri + 1] - offs[ri]);
    const Status bad(Status::kCorruption, "bad metadata at row " + std::to_string(ri));
    if (!DecodeMetaRowValues(schema, data, &row)) return bad;
    const uint32_t r32 = static_cast<uint32_t>(ri);
    for (size_t f = 0; f < schema.size(); ++f) {
      const RowValue& v = row[f];
      if (!v.has) continue;
      HostColumn& c = (*cols)[f];
      c.present[r32 >> 5] |= 1u << (r32 & 31);
      switch (schema[f].type) {
        case FieldType::Int64:
        case FieldType::Float64: c.values[ri] = v.num; break;
        case FieldType::Keyword:
        case FieldType::KeywordList:
          for (const auto& s : v.strs) {
            auto [it, inserted] = c.dict.emplace(s, static_cast<int32_t>(c.postings.size()));
            if (inserted) c.postings.emplace_back();
            auto& pr = c.postings[static_cast<size_t>(it->second)];
            if (pr.empty() || pr.back() != r32) pr.push_back(r32);
          }
          break;
        case FieldType::Bool:
          (v.b ? c.trues : c.falses)[r32 >> 5] |= 1u << (r32 & 31);
          break;
      }
    }
  }
  return Status::OK();
}

}  // namespace

namespace {

// ---- The log replay of Collection::Open (CollectionImpl::Recover step 5,
// src/engine/collection_impl.cc:160-235; ApplyOp, :574-599).

// Log files (src/storage/wal.h:27-37, src/storage/wal.cc): a 16-byte header ("VDBWAL01", u32
// version 1, u32 0), then records [u32 crc32c][u32 payload length][u8 type: 1 upsert, 2 delete]
// [u64 lsn][payload]; the crc covers everything after itself. Upsert payload: u64 id, u32 dim,
// dim floats, u32 metadata length, the metadata row as EncodeMetaRow. Delete payload: u64 id.
constexpr size_t kWalFileHeaderSize = 16, kWalRecordHeaderSize = 17;

struct WalRecordView {
  uint8_t type = 0;
  uint64_t lsn = 0;
  std::string_view payload;
};

bool TryParseWalRecord(std::string_view data, size_t pos, WalRecordView* rec, size_t* len) {
  if (data.size() - pos < kWalRecordHeaderSize) return false;
  const char* p = data.data() + pos;
  const uint32_t plen = GetAt<uint32_t>(p, 4);
  if (plen > data.size() - pos - kWalRecordHeaderSize) return false;
  const uint8_t type = static_cast<uint8_t>(p[8]);
  if (type != 1 && type != 2) return false;
  if (Crc32c(p + 4, kWalRecordHeaderSize - 4 + plen) != GetAt<uint32_t>(p, 0)) return false;
  rec->type = type;
  rec->lsn = GetAt<uint64_t>(p, 9);
  rec->payload = std::string_view(p + kWalRecordHeaderSize, plen);
  *len = kWalRecordHeaderSize + plen;
  return true;
}

// ParseWal (wal.cc): hands every valid record to cb in order. A bad record with no valid record at
// any later offset is a torn tail (*torn); one followed by a valid record is corruption.
Status ParseWalRecords(std::string_view data, const std::function<Status(const WalRecordView&)>& cb, bool* torn) {
  *torn = false;
  if (data.size() < kWalFileHeaderSize) {
    *torn = !data.empty();
    return Status::OK();
  }
  if (data.substr(0, 8) != "VDBWAL01" || GetAt<uint32_t>(data.data(), 8) != 1)
    return Status(Status::kCorruption, "bad log file header");
  size_t pos = kWalFileHeaderSize;
  while (pos < data.size()) {
    WalRecordView rec;
    size_t len = 0;
    if (TryParseWalRecord(data, pos, &rec, &len)) {
      VDBGPU_RETURN_IF_ERROR(cb(rec));
      pos += len;
      continue;
    }
    for (size_t off = pos + 1; off + kWalRecordHeaderSize <= data.size(); ++off) {
      WalRecordView later;
      size_t later_len = 0;
      if (TryParseWalRecord(data, off, &later, &later_len))
        return Status(Status::kCorruption,
                      "corrupt log record at offset " + std::to_string(pos) + " followed by valid records");
    }
    *torn = true;
    break;
  }
  return Status::OK();
}

// "<prefix><digits><suffix>" -> the number (ParseWalFileName, ParseManifestFileName,
// ParseSegmentDirName).
bool ParseNumberedName(std::string_view name, std::string_view prefix, std::string_view suffix, uint64_t* num) {
  if (name.size() <= prefix.size() + suffix.size() || name.substr(0, prefix.size()) != prefix ||
      name.substr(name.size() - suffix.size()) != suffix)
    return false;
  uint64_t n = 0;
  for (char ch : name.substr(prefix.size(), name.size() - prefix.size() - suffix.size())) {
    if (ch < '0' || ch > '9') return false;
    n = n * 10 + static_cast<uint64_t>(ch - '0');
  }
  *num = n;
  return true;
}

std::vector<std::string> ListDir(const std::string& path) {
  std::vector<std::string> names;
  if (DIR* d = opendir(path.c_str())) {
    while (const dirent* e = readdir(d)) {
      const std::string n = e->d_name;
      if (n != "." && n != "..") names.push_back(n);
    }
    closedir(d);
  }
  return names;
}

// vectors.f32 header checks of Segment::Open (segment_reader.cc:36-51) against the manifest and
// the collection's options: the 4 KiB header and the file's size.
Status CheckSegmentHeader(const std::string& dir, const char* h, uint64_t file_size, uint64_t rows,
                          const CollectionOptions& opt) {
  if (file_size < kSegmentHeaderSize) return Status(Status::kCorruption, dir + ": vectors.f32 shorter than its header");
  if (std::memcmp(h, "VDBSEG01", 8) != 0) return Status(Status::kCorruption, dir + ": bad magic");
  if (GetAt<uint32_t>(h, kSegmentHeaderSize - 4) != Crc32c(h, kSegmentHeaderSize - 4))
    return Status(Status::kCorruption, dir + ": header checksum mismatch");
  const uint64_t data_len = GetAt<uint64_t>(h, 40);
  if (GetAt<uint32_t>(h, 8) != 1 || GetAt<uint32_t>(h, 12) != static_cast<uint32_t>(opt.metric) ||
      GetAt<uint64_t>(h, 16) != rows || GetAt<uint32_t>(h, 24) != opt.dim || GetAt<uint32_t>(h, 28) != opt.pd ||
      GetAt<uint64_t>(h, 32) != kSegmentHeaderSize || rows > (file_size / 4) ||
      data_len != rows * opt.pd * sizeof(float) || file_size - kSegmentHeaderSize < data_len)
    return Status(Status::kCorruption, dir + ": header does not match the manifest");
  return Status::OK();
}

// One disk segment of the manifest, with its ids and delete bits once read.
struct SegEntry {
  uint32_t id = 0;
  uint64_t rows = 0, lsn = 0;
  std::string deletes_file, dir;
  std::vector<uint64_t> ids;  // read for the id map, then released
  std::vector<uint32_t> del;  // (rows + 31) / 32 words; empty until read
};

Status LoadIds(SegEntry* e) {
  std::string idsf;
  VDBGPU_RETURN_IF_ERROR(ReadFile(e->dir + "/ids.u64", &idsf));
  std::string_view ids_p;
  Status st = DecodeBlob(idsf, "VDBIDS01", &ids_p);
  if (!st.ok()) return Status(Status::kCorruption, e->dir + "/ids.u64: " + st.message());
  if (ids_p.size() != e->rows * 8) return Status(Status::kCorruption, e->dir + ": ids.u64 size mismatch");
  e->ids.resize(e->rows);
  if (e->rows > 0) std::memcpy(e->ids.data(), ids_p.data(), e->rows * 8);
  return Status::OK();
}

// The persisted delete set (segment_reader.cc:101-116): a "VDBDEL01" blob named by the manifest
// entry's deletes_file.
Status LoadDeletes(SegEntry* e) {
  e->del.assign((e->rows + 31) / 32, 0u);
  if (e->deletes_file.empty()) return Status::OK();
  std::string delf;
  VDBGPU_RETURN_IF_ERROR(ReadFile(e->dir + "/" + e->deletes_file, &delf));
  std::string_view del_p;
  Status st = DecodeBlob(delf, "VDBDEL01", &del_p);
  if (!st.ok()) return Status(Status::kCorruption, e->dir + "/" + e->deletes_file + ": " + st.message());
  st = DecodeDeleteSet(del_p, e->rows, &e->del);
  if (!st.ok()) return Status(st.code(), e->dir + ": " + st.message());
  return Status::OK();
}

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
  void Build(const std::vector<SegEntry>& segs) {
    std::vector<size_t> order(segs.size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = i;
    std::sort(order.begin(), order.end(), [&](size_t a, size_t b) {
      return segs[a].lsn < segs[b].lsn || (segs[a].lsn == segs[b].lsn && segs[a].id < segs[b].id);
    });
    for (size_t i : order)
      for (uint64_t r = 0; r < segs[i].rows; ++r)
        if (!(segs[i].del[r / 32] >> (r % 32) & 1u)) ids[segs[i].ids[r]] = Loc{static_cast<int64_t>(i), static_cast<uint32_t>(r)};
    touched.assign(segs.size(), false);
  }

  // Applies one record: records at or below skip_below are skipped, any other must carry the
  // expected LSN.
  Status Apply(const WalRecordView& rec, uint64_t skip_below, const CollectionOptions& opt,
               std::vector<SegEntry>& segs, MutableRows* mut) {
    if (rec.lsn <= skip_below) return Status::OK();
    if (rec.lsn != expected)
      return Status(Status::kCorruption, "log sequence gap: expected LSN " + std::to_string(expected) +
                                             ", found " + std::to_string(rec.lsn));
    ++expected;
    mut->last_lsn = std::max(mut->last_lsn, rec.lsn);
    Reader r(rec.payload);
    uint64_t id = 0;
    std::string_view vec, meta;
    if (rec.type == 2) {
      if (!r.u64(&id) || r.remaining() != 0)
        return Status(Status::kCorruption, "bad delete record at LSN " + std::to_string(rec.lsn));
    } else {
      uint32_t dim = 0, mlen = 0;
      if (!r.u64(&id) || !r.u32(&dim) || dim == 0 || !r.bytes(static_cast<size_t>(dim) * 4, &vec) ||
          !r.u32(&mlen) || !r.bytes(mlen, &meta) || r.remaining() != 0 || dim != opt.dim)
        return Status(Status::kCorruption, "bad upsert record at LSN " + std::to_string(rec.lsn));
      std::vector<RowValue> row(opt.schema.size());
      if (!DecodeMetaRowValues(opt.schema, meta, &row))
        return Status(Status::kCorruption, "bad metadata at LSN " + std::to_string(rec.lsn));
      if (mut->n >= kMutableMaxRows) return Status(Status::kResourceExhausted, "mutable segment is full");
    }
    auto mark = [&](const Loc& l) {
      if (l.seg >= 0) touched[static_cast<size_t>(l.seg)] = true;
      std::vector<uint32_t>& d = l.seg < 0 ? mut->del : segs[static_cast<size_t>(l.seg)].del;
      d[l.row / 32] |= 1u << (l.row % 32);
    };
    auto it = ids.find(id);
    const bool old_is_newer =
        it != ids.end() && it->second.seg >= 0 && segs[static_cast<size_t>(it->second.seg)].lsn >= rec.lsn;
    if (it != ids.end() && !old_is_newer) mark(it->second);
    if (rec.type == 2) {
      if (it != ids.end() && !old_is_newer) ids.erase(it);
      return Status::OK();
    }
    const uint32_t pd = opt.pd;
    mut->rows.resize((mut->n + 1) * pd, 0.0f);
    std::memcpy(mut->rows.data() + mut->n * pd, vec.data(), vec.size());
    mut->ids.push_back(id);
    mut->meta.emplace_back(meta);
    mut->max_lsn = std::max(mut->max_lsn, rec.lsn);
    if (mut->n % 32 == 0) mut->del.push_back(0u);
    const Loc here{-1, static_cast<uint32_t>(mut->n)};
    ++mut->n;
    if (old_is_newer) {
      mark(here);
    } else {
      ids[id] = here;
    }
    return Status::OK();
  }
};

// Recover step 5 (collection_impl.cc:160-235): the records after flushed_lsn of every log, in
// order; a torn tail is accepted only at the end of the newest log (recovery truncates it there;
// this loader reads the directory without changing it).
Status ReplayLogs(const std::vector<std::pair<std::string, std::string>>& logs, uint64_t flushed_lsn,
                  const CollectionOptions& opt, std::vector<SegEntry>& segs, MutableRows* mut, LogApplier* ap) {
  for (size_t li = 0; li < logs.size(); ++li) {
    const std::string& path = logs[li].first;
    bool torn = false;
    Status ps = ParseWalRecords(logs[li].second, [&](const WalRecordView& rec) -> Status {
      const uint64_t before = ap->expected;
      VDBGPU_RETURN_IF_ERROR(ap->Apply(rec, flushed_lsn, opt, segs, mut));
      if (ap->expected != before) ++mut->records;
      return Status::OK();
    }, &torn);
    if (!ps.ok()) return Status(ps.code(), path + ": " + ps.message());
    if (torn && li + 1 != logs.size())
      return Status(Status::kCorruption, path + ": damaged record in a log that is not the newest");
  }
  return Status::OK();
}

}  // namespace

// What a collection keeps on the host after Open: the manifest's segments (delete bits, lsn; ids
// only while the id map is built), the mutable segment's rows, and the id map once a log record
// has been applied.
struct GpuCollection::LogState {
  std::string path;
  uint32_t shard = 0, nshards = 1;
  uint32_t mutable_id = 0;
  uint64_t flushed_lsn = 0;
  std::vector<SegEntry> segs;
  MutableRows mut;
  LogApplier ap;
  bool have_map = false;
};

namespace {

// The directory as Collection::Open recovers it (CollectionImpl::Recover, collection_impl.cc:
// 76-235), on the host: options, segments with their delete bits (those of shard `shard` of
// nshards, or of every segment when the logs hold records or `all`), and the mutable segment
// replayed from the logs. Reads only.
Status RecoverDir(const std::string& path, uint32_t shard, uint32_t nshards, bool all, CollectionOptions* opt,
                  GpuCollection::LogState* d) {
  // ReadCurrentManifest (src/storage/manifest.cc:116-127).
  std::string current;
  VDBGPU_RETURN_IF_ERROR(ReadFile(path + "/CURRENT", &current));
  while (!current.empty() && (current.back() == '\n' || current.back() == '\r')) current.pop_back();
  uint64_t number = 0;
  if (!ParseNumberedName(current, "MANIFEST-", "", &number)) return Status(Status::kCorruption, "bad CURRENT file");
  std::string mf;
  VDBGPU_RETURN_IF_ERROR(ReadFile(path + "/" + current, &mf));
  std::string_view payload;
  VDBGPU_RETURN_IF_ERROR(DecodeBlob(mf, "VDBMAN01", &payload));
  // DecodeManifest (manifest.cc:75-106): nlohmann::json's at() and get<T>() on every key, their
  // exceptions reported as "bad manifest: <what()>".
  JsonValue j;
  if (!ParseJson(payload, &j) || !j.is_object()) return Status(Status::kCorruption, "manifest is not valid JSON");
  auto type_name = [](const JsonValue& v) -> std::string {
    switch (v.kind) {
      case JsonValue::kNull: return "null";
      case JsonValue::kBool: return "boolean";
      case JsonValue::kString: return "string";
      case JsonValue::kArray: return "array";
      case JsonValue::kObject: return "object";
      default: return "number";
    }
  };
  auto bad = [](const std::string& what) { return Status(Status::kCorruption, "bad manifest: " + what); };
  auto at = [&](const JsonValue& o, const char* key, const JsonValue** out) -> Status {
    if (!o.is_object()) return bad("[json.exception.type_error.304] cannot use at() with " + type_name(o));
    *out = o.get(key);
    if (*out == nullptr) return bad(std::string("[json.exception.out_of_range.403] key '") + key + "' not found");
    return Status::OK();
  };
  // get<unsigned T>(): numbers and booleans convert (static_cast), anything else is a type error.
  auto get_u64 = [&](const JsonValue& v, uint64_t* out) -> Status {
    switch (v.kind) {
      case JsonValue::kUint: *out = v.u; return Status::OK();
      case JsonValue::kInt: *out = static_cast<uint64_t>(v.i); return Status::OK();
      case JsonValue::kDouble:
        *out = v.d >= 0 && v.d < 18446744073709551616.0 ? static_cast<uint64_t>(v.d)
                                                          : static_cast<uint64_t>(static_cast<int64_t>(v.d));
        return Status::OK();
      case JsonValue::kBool: *out = v.b ? 1 : 0; return Status::OK();
      default: return bad("[json.exception.type_error.302] type must be number, but is " + type_name(v));
    }
  };
  auto key_u64 = [&](const JsonValue& o, const char* key, uint64_t* out) -> Status {
    const JsonValue* v = nullptr;
    VDBGPU_RETURN_IF_ERROR(at(o, key, &v));
    return get_u64(*v, out);
  };
  // j.value("format_version", 0) != 1: a present value converts like get<int>().
  int64_t version = 0;
  if (const JsonValue* fv = j.get("format_version")) {
    uint64_t x = 0;
    VDBGPU_RETURN_IF_ERROR(get_u64(*fv, &x));
    version = fv->kind == JsonValue::kDouble ? static_cast<int64_t>(fv->d) : static_cast<int64_t>(x);
  }
  if (version != 1) return Status(Status::kCorruption, "unknown manifest version");
  uint64_t mnumber = 0, next = 0, flushed_lsn = 0, wal_log_number = 0;
  VDBGPU_RETURN_IF_ERROR(key_u64(j, "number", &mnumber));
  const JsonValue* opts = nullptr;
  VDBGPU_RETURN_IF_ERROR(at(j, "options", &opts));
  VDBGPU_RETURN_IF_ERROR(ManifestOptionsFromJson(*opts, opt));
  VDBGPU_RETURN_IF_ERROR(key_u64(j, "next_file_number", &next));
  VDBGPU_RETURN_IF_ERROR(key_u64(j, "flushed_lsn", &flushed_lsn));
  VDBGPU_RETURN_IF_ERROR(key_u64(j, "wal_log_number", &wal_log_number));
  const JsonValue* segs = nullptr;
  VDBGPU_RETURN_IF_ERROR(at(j, "segments", &segs));
  // Range-for over a JSON value: an array's elements, an object's values, nothing for null, the
  // value itself otherwise.
  std::vector<const JsonValue*> seg_list;
  if (segs->is_array()) {
    for (const auto& v : segs->arr) seg_list.push_back(&v);
  } else if (segs->is_object()) {
    for (const auto& kv : segs->obj) seg_list.push_back(&kv.second);
  } else if (!segs->is_null()) {
    seg_list.push_back(segs);
  }
  d->path = path;
  d->shard = shard;
  d->nshards = nshards;
  d->flushed_lsn = flushed_lsn;
  std::vector<SegEntry>& entries = d->segs;
  entries.resize(seg_list.size());
  for (size_t i = 0; i < seg_list.size(); ++i) {
    const JsonValue& s = *seg_list[i];
    SegEntry& e = entries[i];
    uint64_t id = 0, deleted = 0;
    VDBGPU_RETURN_IF_ERROR(key_u64(s, "id", &id));
    e.id = static_cast<uint32_t>(id);
    VDBGPU_RETURN_IF_ERROR(key_u64(s, "rows", &e.rows));
    VDBGPU_RETURN_IF_ERROR(key_u64(s, "deleted", &deleted));
    VDBGPU_RETURN_IF_ERROR(key_u64(s, "lsn", &e.lsn));
    const JsonValue* dfv = nullptr;
    VDBGPU_RETURN_IF_ERROR(at(s, "deletes_file", &dfv));
    if (!dfv->is_string()) return bad("[json.exception.type_error.302] type must be string, but is " + type_name(*dfv));
    e.deletes_file = dfv->s;
    const JsonValue* files = nullptr;
    VDBGPU_RETURN_IF_ERROR(at(s, "files", &files));
    // it.key() needs an object iterator; null and empty arrays iterate nothing.
    if (files->is_object()) {
      for (const auto& kv : files->obj) {
        uint64_t x = 0;
        VDBGPU_RETURN_IF_ERROR(key_u64(kv.second, "size", &x));
        VDBGPU_RETURN_IF_ERROR(key_u64(kv.second, "crc", &x));
      }
    } else if (!files->is_null() && !(files->is_array() && files->arr.empty())) {
      return bad("[json.exception.invalid_iterator.207] cannot use key() for non-object iterators");
    }
    char name[32];
    std::snprintf(name, sizeof(name), "seg-%06u", e.id);
    e.dir = path + "/segments/" + name;
  }
  if (mnumber != number) return Status(Status::kCorruption, "manifest number does not match CURRENT");
  // The next file number (Recover steps 1, 2 and 5): past every manifest, segment directory and
  // log; the mutable segment takes it.
  uint64_t num = 0;
  for (const auto& n : ListDir(path))
    if (ParseNumberedName(n, "MANIFEST-", "", &num)) next = std::max(next, num + 1);
  for (const auto& n : ListDir(path + "/segments"))
    if (ParseNumberedName(n, "seg-", "", &num)) next = std::max(next, num + 1);
  std::vector<std::pair<uint64_t, std::string>> lognames;
  for (const auto& n : ListDir(path + "/wal")) {
    if (!ParseNumberedName(n, "", ".log", &num)) continue;
    next = std::max(next, num + 1);
    if (num >= wal_log_number) lognames.emplace_back(num, path + "/wal/" + n);
  }
  std::sort(lognames.begin(), lognames.end());
  std::vector<std::pair<std::string, std::string>> logs;
  bool any_records = false;
  for (const auto& [n, p] : lognames) {
    std::string data;
    VDBGPU_RETURN_IF_ERROR(ReadFile(p, &data));
    any_records |= data.size() > kWalFileHeaderSize;
    logs.emplace_back(p, std::move(data));
  }
  d->mutable_id = static_cast<uint32_t>(next);
  for (const SegEntry& e : entries) {
    std::string h;
    uint64_t size = 0;
    VDBGPU_RETURN_IF_ERROR(ReadPrefix(e.dir + "/vectors.f32", kSegmentHeaderSize, &h, &size));
    VDBGPU_RETURN_IF_ERROR(CheckSegmentHeader(e.dir, h.data(), size, e.rows, *opt));
  }
  // Delete sets: of this shard's segments, and of every segment when the logs hold records (an
  // upsert or delete may name a row of any segment, so the id map needs every segment's ids).
  for (size_t i = 0; i < entries.size(); ++i)
    if (all || any_records || i % nshards == shard) VDBGPU_RETURN_IF_ERROR(LoadDeletes(&entries[i]));
  d->mut.last_lsn = flushed_lsn;
  for (const SegEntry& e : entries) d->mut.last_lsn = std::max(d->mut.last_lsn, e.lsn);
  // Records continue from flushed_lsn + 1 (collection_impl.cc:183); after the replay, from the
  // last record replayed. In a directory the reference wrote this is also its next LSN: a bulk
  // load or compaction takes the LSN of the last record, it does not advance it.
  d->ap.expected = flushed_lsn + 1;
  if (any_records) {
    for (SegEntry& e : entries) VDBGPU_RETURN_IF_ERROR(LoadIds(&e));
    d->ap.Build(entries);
    d->have_map = true;
    for (SegEntry& e : entries) std::vector<uint64_t>().swap(e.ids);
    VDBGPU_RETURN_IF_ERROR(ReplayLogs(logs, flushed_lsn, *opt, entries, &d->mut, &d->ap));
  }
  return Status::OK();
}

}  // namespace

Status GpuCollection::Open(Context& ctx, const std::string& path, uint32_t shard, uint32_t nshards,
                           std::unique_ptr<GpuCollection>* out) {
  if (nshards == 0 || shard >= nshards) return Status(Status::kInvalidArgument, "bad shard");
  auto c = std::make_unique<GpuCollection>();
  c->log_ = std::make_shared<LogState>();
  LogState& d = *c->log_;
  VDBGPU_RETURN_IF_ERROR(RecoverDir(path, shard, nshards, false, &c->opt_, &d));
  const uint32_t pd = c->opt_.pd;
  for (size_t i = 0; i < d.segs.size(); ++i) {
    if (i % nshards != shard) continue;
    const SegEntry& e = d.segs[i];
    const std::string& dir = e.dir;
    // vectors.f32 header checks of Segment::Open (segment_reader.cc:36-51).
    std::string vec;
    VDBGPU_RETURN_IF_ERROR(ReadFile(dir + "/vectors.f32", &vec));
    VDBGPU_RETURN_IF_ERROR(CheckSegmentHeader(dir, vec.data(), vec.size(), e.rows, c->opt_));
    const char* h = vec.data();
    SegEntry ide = e;  // this segment's ids, for the upload only
    VDBGPU_RETURN_IF_ERROR(LoadIds(&ide));
    std::string metaf, indexf;
    VDBGPU_RETURN_IF_ERROR(ReadFile(dir + "/meta.bin", &metaf));
    VDBGPU_RETURN_IF_ERROR(ReadFile(dir + "/" + IndexFileName(c->opt_.index_type), &indexf));
    std::string_view meta_p;
    Status st = DecodeBlob(metaf, "VDBMETA1", &meta_p);
    if (!st.ok()) return Status(Status::kCorruption, dir + "/meta.bin: " + st.message());
    // Part 0 of the merge is the mutable segment (collection_impl.cc:1056-1059); disk segments
    // follow in manifest order.
    st = c->AddSegment(ctx, e.id, static_cast<uint32_t>(i + 1), reinterpret_cast<const float*>(h + kSegmentHeaderSize),
                       e.rows, ide.ids.data(), meta_p, indexf);
    if (!st.ok()) return Status(st.code(), dir + ": " + st.message());
    bool any = false;
    for (uint32_t w : e.del) any |= w != 0;
    if (any) {
      st = c->SetDeleted(ctx, e.id, e.del.data());
      if (!st.ok()) return Status(st.code(), dir + ": " + st.message());
    }
  }
  VDBGPU_RETURN_IF_ERROR(c->UploadMutable(ctx));
  *out = std::move(c);
  return Status::OK();
}

// The mutable segment lives on shard 0 and is searched exhaustively (SearchMutable,
// planner.cc:131-149) through a flat index over its rows; it is rebuilt whole after a change.
Status GpuCollection::UploadMutable(Context& ctx) {
  const LogState& d = *log_;
  segs_.erase(std::remove_if(segs_.begin(), segs_.end(), [](const auto& s) { return s->is_mutable; }), segs_.end());
  if (d.shard == 0 && d.mut.n > 0) {
    std::string flat = "VDBFLAT1";
    const uint32_t crc = Crc32c(flat.data(), flat.size());
    flat.append(reinterpret_cast<const char*>(&crc), 4);
    const std::string meta = d.mut.MetaPayload();
    VDBGPU_RETURN_IF_ERROR(AddSegment(ctx, d.mutable_id, 0, d.mut.rows.data(), d.mut.n, d.mut.ids.data(), meta, flat));
    for (auto& s : segs_)
      if (s->ordinal == 0) s->is_mutable = true;
    bool any = false;
    for (uint32_t w : d.mut.del) any |= w != 0;
    if (any) VDBGPU_RETURN_IF_ERROR(SetDeleted(ctx, d.mutable_id, d.mut.del.data()));
  }
  total_segments_ = static_cast<uint32_t>(d.segs.size() + (d.mut.n > 0 ? 1 : 0));
  return Status::OK();
}

Status GpuCollection::ApplyLog(Context& ctx, std::string_view records, uint64_t* applied) {
  if (applied != nullptr) *applied = 0;
  if (!log_) return Status(Status::kFailedPrecondition, "the collection was not opened from a directory");
  LogState& d = *log_;
  if (!d.have_map) {
    // The id map, built on first use from every segment's ids and current delete bits.
    for (SegEntry& e : d.segs) {
      if (e.del.empty()) VDBGPU_RETURN_IF_ERROR(LoadDeletes(&e));
      VDBGPU_RETURN_IF_ERROR(LoadIds(&e));
    }
    const uint64_t expected = d.ap.expected;
    // Rows already in the mutable segment keep their ids (later rows of an id win).
    d.ap.Build(d.segs);
    for (uint64_t r = 0; r < d.mut.n; ++r)
      if (!(d.mut.del[r / 32] >> (r % 32) & 1u)) d.ap.ids[d.mut.ids[r]] = LogApplier::Loc{-1, static_cast<uint32_t>(r)};
    d.ap.expected = expected;
    for (SegEntry& e : d.segs) std::vector<uint64_t>().swap(e.ids);
    d.have_map = true;
  }
  d.ap.touched.assign(d.segs.size(), false);
  const uint64_t n_before = d.mut.n;
  const uint64_t del_before = [&] {
    uint64_t c = 0;
    for (uint32_t w : d.mut.del) c += static_cast<uint64_t>(__builtin_popcount(w));
    return c;
  }();
  // The records as the log holds them (no file header); a damaged record fails the call, after
  // the records before it have been applied.
  Status st = Status::OK();
  size_t pos = 0;
  uint64_t count = 0;
  while (pos < records.size()) {
    WalRecordView rec;
    size_t len = 0;
    if (!TryParseWalRecord(records, pos, &rec, &len)) {
      st = Status(Status::kInvalidArgument, "bad log record at offset " + std::to_string(pos));
      break;
    }
    const uint64_t before = d.ap.expected;
    st = d.ap.Apply(rec, d.ap.expected - 1, opt_, d.segs, &d.mut);
    if (!st.ok()) break;
    count += d.ap.expected != before ? 1 : 0;
    pos += len;
  }
  for (size_t i = 0; i < d.segs.size(); ++i) {
    if (!d.ap.touched[i] || i % d.nshards != d.shard) continue;
    VDBGPU_RETURN_IF_ERROR(SetDeleted(ctx, d.segs[i].id, d.segs[i].del.data()));
  }
  uint64_t del_after = 0;
  for (uint32_t w : d.mut.del) del_after += static_cast<uint64_t>(__builtin_popcount(w));
  if (d.mut.n != n_before || del_after != del_before) VDBGPU_RETURN_IF_ERROR(UploadMutable(ctx));
  if (applied != nullptr) *applied = count;
  return st;
}

Status GpuCollection::Inspect(const std::string& path, std::string* json) {
  LogState d;
  CollectionOptions opt;
  VDBGPU_RETURN_IF_ERROR(RecoverDir(path, 0, 1, true, &opt, &d));
  auto count = [](const std::vector<uint32_t>& bits, uint64_t rows) {
    uint64_t c = 0;
    for (uint64_t w = 0; w < bits.size(); ++w) {
      const uint32_t valid = w < rows / 32 ? 0xFFFFFFFFu : (w == rows / 32 ? (1u << (rows % 32)) - 1u : 0u);
      c += static_cast<uint64_t>(__builtin_popcount(bits[w] & valid));
    }
    return c;
  };
  std::string segs;
  uint64_t total = 0, deleted = 0;
  auto add = [&](uint32_t id, const char* kind, const std::string& index, uint64_t rows, uint64_t del, uint64_t lsn) {
    if (!segs.empty()) segs += ",";
    segs += "{\"id\":" + std::to_string(id) + ",\"kind\":\"" + kind + "\",\"index\":\"" + index +
            "\",\"rows\":" + std::to_string(rows) + ",\"deleted\":" + std::to_string(del) +
            ",\"lsn\":" + std::to_string(lsn) + "}";
    total += rows;
    deleted += del;
  };
  add(d.mutable_id, "mutable", "flat", d.mut.n, count(d.mut.del, d.mut.n), d.mut.max_lsn);
  const std::string index = std::string(IndexFileName(opt.index_type)).substr(6);
  for (const SegEntry& e : d.segs) add(e.id, "disk", index, e.rows, count(e.del, e.rows), e.lsn);
  *json = "{\"live_rows\":" + std::to_string(total - deleted) + ",\"total_rows\":" + std::to_string(total) +
          ",\"deleted_rows\":" + std::to_string(deleted) + ",\"last_lsn\":" + std::to_string(d.mut.last_lsn) +
          ",\"flushed_lsn\":" + std::to_string(d.flushed_lsn) +
          ",\"recovery_records\":" + std::to_string(d.mut.records) + ",\"segments\":[" + segs + "]}";
  return Status::OK();
}

Status GpuCollection::AddSegment(Context& ctx, uint32_t id, uint32_t ordinal, const float* rows, uint64_t n,
                                 const uint64_t* ids, std::string_view meta, std::string_view index_file) {
  if (n >= (uint64_t{1} << 32) - 256) return Status(Status::kNotSupported, "segment too large");
  auto seg = std::make_unique<GpuSegment>();
  seg->id = id;
  seg->ordinal = ordinal;
  seg->rows = n;
  seg->words = RoundUp(std::max<uint64_t>(n, 1), 256) / 32;
  VDBGPU_RETURN_IF_ERROR(LoadIndexFile(ctx, index_file.data(), index_file.size(), opt_.metric, rows, n,
                                       opt_.dim, opt_.pd, &seg->index));
  std::vector<uint64_t> idv(ids, ids + n);
  VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, idv, &seg->ids));
  std::vector<uint32_t> all(seg->words, 0);
  for (uint64_t w = 0; w < n / 32; ++w) all[w] = 0xFFFFFFFFu;
  if (n % 32 != 0) all[n / 32] = (1u << (n % 32)) - 1u;
  VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, all, &seg->all));
  std::vector<HostColumn> hc;
  VDBGPU_RETURN_IF_ERROR(BuildColumns(opt_.schema, n, seg->words, meta, &hc));
  seg->cols.resize(opt_.schema.size());
  for (size_t f = 0; f < hc.size(); ++f) {
    GpuColumn& g = seg->cols[f];
    HostColumn& h = hc[f];
    g.type = opt_.schema[f].type;
    VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, h.present, &g.present));
    if (!h.values.empty()) VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, h.values, &g.values));
    if (g.type == FieldType::Bool) {
      VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, h.trues, &g.true_rows));
      VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, h.falses, &g.false_rows));
    }
    if (g.type == FieldType::Keyword || g.type == FieldType::KeywordList) {
      g.dict = std::move(h.dict);
      g.post_off.assign(h.postings.size() + 1, 0);
      std::vector<uint32_t> flat;
      for (size_t c = 0; c < h.postings.size(); ++c) {
        g.post_off[c + 1] = g.post_off[c] + h.postings[c].size();
        flat.insert(flat.end(), h.postings[c].begin(), h.postings[c].end());
      }
      VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, flat, &g.post_rows));
    }
  }
  VDBGPU_RETURN_IF_ERROR(ctx.Sync("segment upload"));
  segs_.push_back(std::move(seg));
  std::sort(segs_.begin(), segs_.end(), [](const auto& a, const auto& b) { return a->ordinal < b->ordinal; });
  total_segments_ = std::max(total_segments_, ordinal + 1);
  return Status::OK();
}

Status GpuCollection::SetDeleted(Context& ctx, uint32_t segment_id, const uint32_t* bits) {
  for (auto& s : segs_) {
    if (s->id != segment_id) continue;
    if (bits == nullptr) {
      s->deletes.reset();
      s->live.reset();
      s->deleted = 0;
      return Status::OK();
    }
    std::vector<uint32_t> del(s->words, 0), live(s->words, 0);
    uint64_t cnt = 0;
    for (uint64_t w = 0; w < s->words; ++w) {
      uint32_t all = w < s->rows / 32 ? 0xFFFFFFFFu : (w == s->rows / 32 ? (1u << (s->rows % 32)) - 1u : 0u);
      del[w] = (w * 32 < s->rows ? bits[w] : 0u) & all;
      live[w] = all & ~del[w];
      cnt += static_cast<uint64_t>(__builtin_popcount(del[w]));
    }
    VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, del, &s->deletes));
    VDBGPU_RETURN_IF_ERROR(UploadVec(ctx, live, &s->live));
    s->deleted = cnt;
    return ctx.Sync("set deleted");
  }
  return Status(Status::kNotFound, "no segment " + std::to_string(segment_id));
}

uint64_t GpuCollection::rows_local() const {
  uint64_t n = 0;
  for (const auto& s : segs_) n += s->rows;
  return n;
}

uint64_t GpuCollection::device_bytes() const {
  uint64_t b = 0;
  for (const auto& s : segs_) {
    b += s->index->device_bytes() + s->ids.size() + s->all.size() + s->deletes.size() + s->live.size();
    for (const auto& c : s->cols)
      b += c.present.size() + c.values.size() + c.post_rows.size() + c.true_rows.size() + c.false_rows.size();
  }
  return b;
}

// ------------------------------------------------------------------------------- search

// A leaf of a filter as SegmentColumns::Leaf (src/meta/columns.cc:207-250) evaluates it.
struct GpuCollection::LeafSpec {
  enum Kind { kRange, kIn, kPosting, kPresent, kTrue, kFalse } kind = kRange;
  int field = 0;
  double lo = 0, hi = 0;
  bool lo_incl = true, hi_incl = true;
  std::vector<double> set;
  std::vector<std::string> strings;
};

namespace {

struct Step {
  int op;
  int leaf;  // kProgPush: leaf index
};

struct Compiler {
  std::vector<GpuCollection::LeafSpec>* leaves;
  std::map<std::string, int>* keys;
  int depth = 0, max_depth = 0;

  int Leaf(GpuCollection::LeafSpec spec) {
    std::string key = std::to_string(static_cast<int>(spec.kind)) + ":" + std::to_string(spec.field) + ":";
    char buf[64];
    std::snprintf(buf, sizeof(buf), "%a:%a:%d%d", spec.lo, spec.hi, spec.lo_incl ? 1 : 0, spec.hi_incl ? 1 : 0);
    key += buf;
    for (double d : spec.set) {
      std::snprintf(buf, sizeof(buf), ",%a", d);
      key += buf;
    }
    for (const auto& s : spec.strings) key += "," + std::to_string(s.size()) + ":" + s;
    auto it = keys->find(key);
    if (it != keys->end()) return it->second;
    const int id = static_cast<int>(leaves->size());
    leaves->push_back(std::move(spec));
    (*keys)[key] = id;
    return id;
  }

  void Push(std::vector<Step>* out, int op, int leaf = -1) {
    out->push_back({op, leaf});
    if (op == kProgPush || op == kProgZero) {
      max_depth = std::max(max_depth, ++depth);
    } else if (op != kProgNot) {
      --depth;
    }
  }

  GpuCollection::LeafSpec Range(int field, double lo, bool li, double hi, bool hi_incl) {
    GpuCollection::LeafSpec s;
    s.kind = GpuCollection::LeafSpec::kRange;
    s.field = field;
    s.lo = lo;
    s.lo_incl = li;
    s.hi = hi;
    s.hi_incl = hi_incl;
    return s;
  }

  GpuCollection::LeafSpec Simple(GpuCollection::LeafSpec::Kind k, int field) {
    GpuCollection::LeafSpec s;
    s.kind = k;
    s.field = field;
    return s;
  }

  void Node(const FilterNode& n, std::vector<Step>* out) {
    using Op = FilterNode::Op;
    using LK = GpuCollection::LeafSpec;
    constexpr double kInf = INFINITY;
    switch (n.op) {
      case Op::And:
      case Op::Or:
        Node(*n.children[0], out);
        for (size_t i = 1; i < n.children.size(); ++i) {
          Node(*n.children[i], out);
          Push(out, n.op == Op::And ? kProgAnd : kProgOr);
        }
        return;
      case Op::Not:
        Node(*n.children[0], out);
        Push(out, kProgNot);
        return;
      default: break;
    }
    if (n.op == Op::Exists) {
      Push(out, kProgPush, Leaf(Simple(LK::kPresent, n.field)));
      if (!n.boolean) Push(out, kProgNot);
      return;
    }
    switch (n.type) {
      case FieldType::Int64:
      case FieldType::Float64:
        switch (n.op) {
          case Op::Eq: Push(out, kProgPush, Leaf(Range(n.field, n.numbers[0], true, n.numbers[0], true))); return;
          case Op::Ne:
            Push(out, kProgPush, Leaf(Simple(LK::kPresent, n.field)));
            Push(out, kProgPush, Leaf(Range(n.field, n.numbers[0], true, n.numbers[0], true)));
            Push(out, kProgAndNot);
            return;
          case Op::In: {
            LK s = Simple(LK::kIn, n.field);
            s.set = n.numbers;
            Push(out, kProgPush, Leaf(std::move(s)));
            return;
          }
          case Op::Lt: Push(out, kProgPush, Leaf(Range(n.field, -kInf, true, n.numbers[0], false))); return;
          case Op::Lte: Push(out, kProgPush, Leaf(Range(n.field, -kInf, true, n.numbers[0], true))); return;
          case Op::Gt: Push(out, kProgPush, Leaf(Range(n.field, n.numbers[0], false, kInf, true))); return;
          case Op::Gte: Push(out, kProgPush, Leaf(Range(n.field, n.numbers[0], true, kInf, true))); return;
          default: Push(out, kProgZero); return;
        }
      case FieldType::Keyword:
      case FieldType::KeywordList: {
        LK s = Simple(LK::kPosting, n.field);
        switch (n.op) {
          case Op::Eq:
            s.strings = {n.strings[0]};
            Push(out, kProgPush, Leaf(std::move(s)));
            return;
          case Op::Ne:
            s.strings = {n.strings[0]};
            Push(out, kProgPush, Leaf(Simple(LK::kPresent, n.field)));
            Push(out, kProgPush, Leaf(std::move(s)));
            Push(out, kProgAndNot);
            return;
          case Op::In:
            s.strings = n.strings;
            Push(out, kProgPush, Leaf(std::move(s)));
            return;
          default: Push(out, kProgZero); return;
        }
      }
      case FieldType::Bool:
        if (n.op == Op::Eq) {
          Push(out, kProgPush, Leaf(Simple(n.boolean ? LK::kTrue : LK::kFalse, n.field)));
        } else if (n.op == Op::Ne) {
          Push(out, kProgPush, Leaf(Simple(n.boolean ? LK::kFalse : LK::kTrue, n.field)));
        } else {
          Push(out, kProgZero);
        }
        return;
    }
    Push(out, kProgZero);
  }
};

}  // namespace

struct GpuCollection::Batch {
  const Request* r = nullptr;
  uint64_t nq = 0;
  uint32_t k = 0;
  uint32_t F = 0;                       // filters; group F = unfiltered queries
  std::vector<uint32_t> perm;           // sorted position -> caller's query
  std::vector<uint64_t> goff;           // group g = sorted [goff[g], goff[g + 1])
  std::vector<std::vector<Step>> progs; // per filter
  std::vector<LeafSpec> leaves;
  float* prepared = nullptr;            // sorted, nq x pd
  uint64_t* keys = nullptr;             // segments x nq x k
  uint64_t* dc = nullptr;               // segments x nq
  int* shortf = nullptr;                // segments x nq
  // explain: strategy per (segment, group) and fallback per (segment, query)
  std::vector<std::string> strat;       // segments x (F + 1)
  std::vector<uint64_t> matches;        // segments x (F + 1)
};

Status GpuCollection::Search(Context& ctx, const Request& r) {
  if (r.k == 0 || r.k > kMaxK) return Status(Status::kInvalidArgument, "k must be in 1..10000");
  if (r.k > kMaxGpuK) return Status(Status::kNotSupported, "k above 240 is not supported on the GPU");
  if (r.nq == 0) return Status::OK();
  for (auto& v : stats_) v = 0;
  stats_[0] = r.nq;
  const uint64_t t_search = NowUs();
  const uint32_t pd = opt_.pd, dim = opt_.dim;
  Batch b;
  b.r = &r;
  b.nq = r.nq;
  b.k = r.k;
  b.F = static_cast<uint32_t>(r.filters.size());
  // Filters: parse and compile (FilterExpr::Parse, then Leaf / Evaluate structure).
  std::map<std::string, int> leaf_keys;
  for (const auto& text : r.filters) {
    std::unique_ptr<FilterExpr> f;
    VDBGPU_RETURN_IF_ERROR(FilterExpr::Parse(text, opt_.schema, &f));
    Compiler c{&b.leaves, &leaf_keys};
    std::vector<Step> prog;
    c.Node(f->root(), &prog);
    if (c.max_depth > kProgStack) return Status(Status::kNotSupported, "filter too deep for the GPU evaluator");
    b.progs.push_back(std::move(prog));
  }
  // Group the queries by filter (stable).
  std::vector<uint32_t> grp(b.nq);
  for (uint64_t q = 0; q < b.nq; ++q) {
    int32_t v = r.query_filter != nullptr ? r.query_filter[q] : (b.F > 0 ? 0 : -1);
    if (v >= static_cast<int32_t>(b.F)) return Status(Status::kInvalidArgument, "query filter index out of range");
    grp[q] = v < 0 ? b.F : static_cast<uint32_t>(v);
  }
  b.goff.assign(b.F + 2, 0);
  for (uint64_t q = 0; q < b.nq; ++q) ++b.goff[grp[q] + 1];
  for (uint32_t g = 0; g <= b.F; ++g) b.goff[g + 1] += b.goff[g];
  b.perm.resize(b.nq);
  {
    std::vector<uint64_t> pos(b.goff.begin(), b.goff.end() - 1);
    for (uint64_t q = 0; q < b.nq; ++q) b.perm[pos[grp[q]]++] = static_cast<uint32_t>(q);
  }
  cudaStream_t st = ctx.stream();
  // PrepareQuery on the device.
  const float* qin = r.queries;
  if (!OnDevice(r.queries)) {
    VDBGPU_RETURN_IF_ERROR(q_raw_.ensure(b.nq * dim * sizeof(float)));
    VDBGPU_CUDA(cudaMemcpyAsync(q_raw_.get(), r.queries, b.nq * dim * sizeof(float), cudaMemcpyHostToDevice, st));
    qin = q_raw_.as<float>();
  }
  VDBGPU_RETURN_IF_ERROR(perm_.ensure(b.nq * 4));
  VDBGPU_CUDA(cudaMemcpyAsync(perm_.get(), b.perm.data(), b.nq * 4, cudaMemcpyHostToDevice, st));
  VDBGPU_RETURN_IF_ERROR(prepared_.ensure(b.nq * pd * sizeof(float)));
  VDBGPU_RETURN_IF_ERROR(qstatus_.ensure(b.nq * sizeof(int)));
  VDBGPU_CUDA(LaunchPrepareQueries(qin, perm_.as<uint32_t>(), b.nq, dim, pd, opt_.metric == 2,
                                   prepared_.as<float>(), qstatus_.as<int>(), st));
  {
    std::vector<int> qs(b.nq);
    VDBGPU_CUDA(cudaMemcpyAsync(qs.data(), qstatus_.get(), b.nq * sizeof(int), cudaMemcpyDeviceToHost, st));
    VDBGPU_RETURN_IF_ERROR(ctx.Sync("prepare queries"));
    uint64_t first = UINT64_MAX;
    int code = 0;
    for (uint64_t i = 0; i < b.nq; ++i)
      if (qs[i] != 0 && b.perm[i] < first) {
        first = b.perm[i];
        code = qs[i];
      }
    if (code == 1) return Status(Status::kInvalidArgument, "query has a NaN or infinite value");
    if (code == 2) return Status(Status::kInvalidArgument, "a zero query cannot be normalized for cosine");
  }
  b.prepared = prepared_.as<float>();
  const size_t S = segs_.size();
  VDBGPU_RETURN_IF_ERROR(keys_.ensure(std::max<size_t>(1, S * b.nq * b.k) * 8));
  VDBGPU_RETURN_IF_ERROR(dc_.ensure(std::max<size_t>(1, S * b.nq) * 8));
  VDBGPU_RETURN_IF_ERROR(short_.ensure(std::max<size_t>(1, S * b.nq) * 4));
  VDBGPU_CUDA(cudaMemsetAsync(keys_.get(), 0xFF, S * b.nq * b.k * 8, st));
  VDBGPU_CUDA(cudaMemsetAsync(dc_.get(), 0, S * b.nq * 8, st));
  VDBGPU_CUDA(cudaMemsetAsync(short_.get(), 0, S * b.nq * 4, st));
  b.keys = keys_.as<uint64_t>();
  b.dc = dc_.as<uint64_t>();
  b.shortf = short_.as<int>();
  b.strat.assign(S * (b.F + 1), "");
  b.matches.assign(S * (b.F + 1), 0);
  VDBGPU_RETURN_IF_ERROR(SearchGroups(ctx, b));
  if (stats_on_ && S > 0) {
    std::vector<uint64_t> dc(S * b.nq);
    VDBGPU_CUDA(cudaMemcpyAsync(dc.data(), b.dc, dc.size() * 8, cudaMemcpyDeviceToHost, st));
    VDBGPU_RETURN_IF_ERROR(ctx.Sync("stats"));
    uint64_t tot = 0;
    for (uint64_t v : dc) tot += v;
    stats_[2] = tot >= stats_[1] ? tot - stats_[1] : 0;
  }

  // Merge the per-segment lists (collection_impl.cc:1079-1108).
  std::vector<uint32_t> part_no(S);
  std::vector<const uint64_t*> idp(S);
  for (size_t s = 0; s < S; ++s) {
    part_no[s] = segs_[s]->ordinal;
    idp[s] = segs_[s]->ids.as<uint64_t>();
  }
  const size_t meta_bytes = RoundUp(S * 4, 16) + S * 8;
  VDBGPU_RETURN_IF_ERROR(tasks_.ensure(std::max<size_t>(meta_bytes, 64)));
  void *part_dev, *ids_dev;
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, 0, part_no.data(), S * 4, &part_dev));
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, RoundUp(S * 4, 16), idp.data(), S * 8, &ids_dev));
  MergeArgs ma{};
  ma.kind = 0;
  ma.nlists = static_cast<int>(S);
  ma.k = static_cast<int>(b.k);
  ma.nq = b.nq;
  ma.keys = b.keys;
  ma.part_no = static_cast<const uint32_t*>(part_dev);
  ma.ids = static_cast<const uint64_t* const*>(ids_dev);
  ma.perm = perm_.as<uint32_t>();
  const bool rec_dev = OnDevice(r.out_records), ids_dev_ok = OnDevice(r.out_ids) && OnDevice(r.out_dist);
  if (r.out_records != nullptr) {
    if (rec_dev) {
      ma.out_records = r.out_records;
    } else {
      VDBGPU_RETURN_IF_ERROR(merged_.ensure(b.nq * b.k * sizeof(HitRecord)));
      ma.out_records = merged_.as<HitRecord>();
    }
  }
  if (r.out_ids != nullptr) {
    if (ids_dev_ok) {
      ma.out_ids = r.out_ids;
      ma.out_dist = r.out_dist;
    } else {
      VDBGPU_RETURN_IF_ERROR(out_ids_.ensure(b.nq * b.k * 8));
      VDBGPU_RETURN_IF_ERROR(out_dist_.ensure(b.nq * b.k * 4));
      ma.out_ids = out_ids_.as<uint64_t>();
      ma.out_dist = out_dist_.as<float>();
    }
  }
  if (S == 0) {
    // No local segment: every slot is a miss.
    ma.nlists = 0;
  }
  VDBGPU_CUDA(LaunchMerge(ma, st));
  if (r.out_records != nullptr && !rec_dev)
    VDBGPU_CUDA(cudaMemcpyAsync(r.out_records, merged_.get(), b.nq * b.k * sizeof(HitRecord), cudaMemcpyDeviceToHost, st));
  if (r.out_ids != nullptr && !ids_dev_ok) {
    VDBGPU_CUDA(cudaMemcpyAsync(r.out_ids, out_ids_.get(), b.nq * b.k * 8, cudaMemcpyDefault, st));
    VDBGPU_CUDA(cudaMemcpyAsync(r.out_dist, out_dist_.get(), b.nq * b.k * 4, cudaMemcpyDefault, st));
  }
  if (r.explain != nullptr) {
    std::vector<uint64_t> keys(S * b.nq * b.k), dc(S * b.nq);
    std::vector<int> sh(S * b.nq);
    if (!keys.empty()) {
      VDBGPU_CUDA(cudaMemcpyAsync(keys.data(), b.keys, keys.size() * 8, cudaMemcpyDeviceToHost, st));
      VDBGPU_CUDA(cudaMemcpyAsync(dc.data(), b.dc, dc.size() * 8, cudaMemcpyDeviceToHost, st));
      VDBGPU_CUDA(cudaMemcpyAsync(sh.data(), b.shortf, sh.size() * 4, cudaMemcpyDeviceToHost, st));
    }
    VDBGPU_RETURN_IF_ERROR(ctx.Sync("explain"));
    r.explain->assign(b.nq, std::vector<PartExplain>(S));
    std::vector<uint32_t> gof(b.nq);
    for (uint32_t g = 0; g <= b.F; ++g)
      for (uint64_t i = b.goff[g]; i < b.goff[g + 1]; ++i) gof[i] = g;
    for (uint64_t i = 0; i < b.nq; ++i) {
      const uint64_t q = b.perm[i];
      for (size_t s = 0; s < S; ++s) {
        PartExplain& e = (*r.explain)[q][s];
        e.segment_id = segs_[s]->id;
        e.is_mutable = segs_[s]->is_mutable;
        e.live_rows = segs_[s]->rows - segs_[s]->deleted;
        e.strategy = b.strat[s * (b.F + 1) + gof[i]];
        e.matches = b.matches[s * (b.F + 1) + gof[i]];
        if (sh[s * b.nq + i] != 0 && e.strategy == "filtered_index") e.strategy = "filtered_index+exact_fallback";
        e.dc = e.is_mutable ? e.matches : dc[s * b.nq + i];  // SearchMutable scores every match
        uint64_t res = 0;
        for (uint32_t j = 0; j < b.k; ++j) res += keys[(s * b.nq + i) * b.k + j] != ~0ull ? 1 : 0;
        e.results = res;
      }
    }
  }
  Status done = ctx.Sync("collection search");
  const uint64_t total = NowUs() - t_search;
  const uint64_t parts = stats_[9] + stats_[10] + stats_[11];
  stats_[12] = total > parts ? total - parts : 0;
  return done;
}

// Searches the index of segment s for the queries of group g with kk results per query, then
// packs them into the segment's lists (graph: need = min(k, matches) for the exact fallback;
// post-filter: keep = the filter bitmap).
Status GpuCollection::RunIndex(Context& ctx, Batch& b, size_t s, uint32_t g, uint32_t kk, const SearchParams& p,
                               const uint32_t* allow, const uint32_t* keep, uint32_t need, int* short_flags) {
  const uint64_t q0 = b.goff[g], nqg = b.goff[g + 1] - q0;
  if (nqg == 0) return Status::OK();
  stats_[8] += nqg;
  if (kk > 256) return Status(Status::kNotSupported, "post-filter depth above 256 is not supported on the GPU");
  GpuSegment& seg = *segs_[s];
  VDBGPU_RETURN_IF_ERROR(tmp_dist_.ensure(nqg * kk * 4));
  VDBGPU_RETURN_IF_ERROR(tmp_row_.ensure(nqg * kk * 4));
  SearchBatch sb{};
  sb.queries = b.prepared + q0 * opt_.pd;
  sb.nq = nqg;
  sb.k = kk;
  sb.params = p;
  sb.allow = allow;
  sb.out_dist = tmp_dist_.as<float>();
  sb.out_row = tmp_row_.as<uint32_t>();
  sb.dist_comps = b.dc + s * b.nq + q0;
  VDBGPU_RETURN_IF_ERROR(seg.index->Search(ctx, sb));
  PackItem it{};
  it.dist = tmp_dist_.as<float>();
  it.row = tmp_row_.as<uint32_t>();
  it.kin = kk;
  it.nq = static_cast<uint32_t>(nqg);
  it.keep = keep;
  it.need = need;
  it.out = b.keys + (s * b.nq + q0) * b.k;
  it.short_flag = short_flags;
  VDBGPU_RETURN_IF_ERROR(tasks_.ensure(sizeof(PackItem)));
  void* dev;
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, 0, &it, sizeof(it), &dev));
  VDBGPU_CUDA(LaunchPackHits(static_cast<const PackItem*>(dev), 1, static_cast<uint32_t>(nqg), static_cast<int>(b.k),
                             b.k, 1, ctx.stream()));
  return Status::OK();
}

uint64_t GpuCollection::MaxWords() const {
  uint64_t w = 0;
  for (const auto& sg : segs_) w = std::max(w, sg->words);
  return w;
}

// Leaves materialised per segment: numeric ranges / sets and postings (presence and bool
// bitmaps are used in place).
static int CountSlots(const std::vector<GpuCollection::LeafSpec>& leaves, std::vector<int>* slot) {
  slot->assign(leaves.size(), -1);
  int n = 0;
  for (size_t l = 0; l < leaves.size(); ++l)
    if (leaves[l].kind == GpuCollection::LeafSpec::kRange || leaves[l].kind == GpuCollection::LeafSpec::kIn ||
        leaves[l].kind == GpuCollection::LeafSpec::kPosting)
      (*slot)[l] = n++;
  return n;
}

// Segments per chunk: the leaf and pair bitmaps of one chunk within ~12 GiB of scratch.
size_t GpuCollection::SegmentsPerChunk(const Batch& b, size_t nfilters) const {
  std::vector<int> slot;
  const int nslots = CountSlots(b.leaves, &slot);
  const uint64_t per_seg = (static_cast<uint64_t>(nslots) + nfilters) * MaxWords() * 4;
  return static_cast<size_t>(std::max<uint64_t>(
      1, std::min<uint64_t>(segs_.size(), (12ull << 30) / std::max<uint64_t>(per_seg, 1))));
}

uint32_t* GpuCollection::PairBits(size_t fi, size_t si, size_t cs) const {
  return pairbits_.as<uint32_t>() + (static_cast<uint64_t>(fi) * cs + si) * MaxWords();
}

// The filter bitmaps (minus deleted rows) of filters fq over segments [s0, s0 + cs) into
// pairbits_ (PairBits), with their match counts (SegmentColumns::Evaluate, columns.cc:185-250,
// then planner.cc:64-66).
Status GpuCollection::Bitmaps(Context& ctx, Batch& b, const std::vector<uint32_t>& fq, size_t s0, size_t cs,
                              std::vector<uint64_t>* matches) {
  cudaStream_t st = ctx.stream();
  const uint64_t max_words = MaxWords();
  const uint64_t nchunks_w = (max_words + kProgChunkWords - 1) / kProgChunkWords;
  std::vector<int> slot;
  const int nslots = CountSlots(b.leaves, &slot);
  for (size_t si = 0; si < cs; ++si) stats_[7] += fq.size() * segs_[s0 + si]->words;
  VDBGPU_RETURN_IF_ERROR(leafbits_.ensure(std::max<uint64_t>(1, nslots * cs * max_words) * 4));
  VDBGPU_RETURN_IF_ERROR(pairbits_.ensure(std::max<uint64_t>(1, fq.size() * cs * max_words) * 4));
  VDBGPU_RETURN_IF_ERROR(counts_.ensure(std::max<uint64_t>(1, fq.size() * cs * nchunks_w) * 4));
  VDBGPU_RETURN_IF_ERROR(matches_.ensure(std::max<uint64_t>(1, fq.size() * cs) * 8));
  if (nslots > 0) VDBGPU_CUDA(cudaMemsetAsync(leafbits_.get(), 0, nslots * cs * max_words * 4, st));
  VDBGPU_CUDA(cudaMemsetAsync(matches_.get(), 0, fq.size() * cs * 8, st));
  auto leaf_ptr = [&](size_t l, size_t si) -> uint32_t* {
    return leafbits_.as<uint32_t>() + (static_cast<uint64_t>(slot[l]) * cs + si) * max_words;
  };
  auto pair_ptr = [&](size_t fi, size_t si) -> uint32_t* { return PairBits(fi, si, cs); };
  // ---- leaves (columns.cc:207-250).
  std::vector<RangeTask> ranges;
  std::vector<ScatterTask> scatters;
  std::vector<std::vector<bool>> leaf_empty(b.leaves.size(), std::vector<bool>(cs, false));
  size_t set_values = 0;
  for (const auto& l : b.leaves) set_values += l.set.size();
  for (size_t l = 0; l < b.leaves.size(); ++l) {
    const LeafSpec& ls = b.leaves[l];
    for (size_t si = 0; si < cs; ++si) {
      GpuSegment& seg = *segs_[s0 + si];
      const GpuColumn& col = seg.cols[static_cast<size_t>(ls.field)];
      if (ls.kind == LeafSpec::kRange || ls.kind == LeafSpec::kIn) {
        RangeTask t{};
        t.out = leaf_ptr(l, si);
        t.present = col.present.as<uint32_t>();
        t.values = col.values.as<double>();
        t.lo = ls.lo;
        t.hi = ls.hi;
        t.lo_incl = ls.lo_incl;
        t.hi_incl = ls.hi_incl;
        t.nset = static_cast<int>(ls.set.size());
        t.words = static_cast<uint32_t>(seg.words);
        ranges.push_back(t);
      } else if (ls.kind == LeafSpec::kPosting) {
        bool any = false;
        for (const auto& sv : ls.strings) {
          auto it = col.dict.find(sv);
          if (it == col.dict.end()) continue;
          const uint64_t a = col.post_off[static_cast<size_t>(it->second)];
          const uint64_t e = col.post_off[static_cast<size_t>(it->second) + 1];
          for (uint64_t c = a; c < e; c += kScatterChunk) {
            ScatterTask t{};
            t.out = leaf_ptr(l, si);
            t.rows = col.post_rows.as<uint32_t>() + c;
            t.count = static_cast<uint32_t>(std::min<uint64_t>(kScatterChunk, e - c));
            scatters.push_back(t);
            any = true;
          }
        }
        leaf_empty[l][si] = !any;
      }
    }
  }
  // Stage the task tables: ranges | set values | scatters | programs | program tasks.
  std::vector<ProgInstr> instrs;
  std::vector<ProgramTask> ptasks;
  std::vector<size_t> prog_at;
  for (size_t fi = 0; fi < fq.size(); ++fi) {
    for (size_t si = 0; si < cs; ++si) {
      GpuSegment& seg = *segs_[s0 + si];
      prog_at.push_back(instrs.size());
      for (const Step& stp : b.progs[fq[fi]]) {
        ProgInstr in{};
        in.op = stp.op;
        if (stp.op == kProgPush) {
          const LeafSpec& ls = b.leaves[static_cast<size_t>(stp.leaf)];
          const GpuColumn& col = seg.cols[static_cast<size_t>(ls.field)];
          switch (ls.kind) {
            case LeafSpec::kPresent: in.bits = col.present.as<uint32_t>(); break;
            case LeafSpec::kTrue: in.bits = col.true_rows.as<uint32_t>(); break;
            case LeafSpec::kFalse: in.bits = col.false_rows.as<uint32_t>(); break;
            case LeafSpec::kPosting:
              if (leaf_empty[static_cast<size_t>(stp.leaf)][si]) in.op = kProgZero;
              else in.bits = leaf_ptr(static_cast<size_t>(stp.leaf), si);
              break;
            default: in.bits = leaf_ptr(static_cast<size_t>(stp.leaf), si); break;
          }
        }
        instrs.push_back(in);
      }
    }
  }
  const size_t o_ranges = 0;
  const size_t o_sets = RoundUp(o_ranges + ranges.size() * sizeof(RangeTask), 16);
  const size_t o_scat = RoundUp(o_sets + set_values * sizeof(double), 16);
  const size_t o_instr = RoundUp(o_scat + scatters.size() * sizeof(ScatterTask), 16);
  const size_t o_ptask = RoundUp(o_instr + instrs.size() * sizeof(ProgInstr), 16);
  const size_t total = RoundUp(o_ptask + fq.size() * cs * sizeof(ProgramTask), 16);
  VDBGPU_RETURN_IF_ERROR(tasks_.ensure(total));
  uint8_t* tb = static_cast<uint8_t*>(tasks_.get());
  {
    // Set values for In leaves, then point the range tasks at them.
    std::vector<double> allsets;
    std::vector<size_t> set_off(b.leaves.size(), 0);
    for (size_t l = 0; l < b.leaves.size(); ++l) {
      set_off[l] = allsets.size();
      allsets.insert(allsets.end(), b.leaves[l].set.begin(), b.leaves[l].set.end());
    }
    size_t ri = 0;
    for (size_t l = 0; l < b.leaves.size(); ++l) {
      if (b.leaves[l].kind != LeafSpec::kRange && b.leaves[l].kind != LeafSpec::kIn) continue;
      for (size_t si = 0; si < cs; ++si, ++ri)
        ranges[ri].set = b.leaves[l].kind == LeafSpec::kIn
                             ? reinterpret_cast<const double*>(tb + o_sets) + set_off[l]
                             : nullptr;
    }
    void* d;
    VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_sets, allsets.data(), allsets.size() * sizeof(double), &d));
  }
  for (size_t fi = 0; fi < fq.size(); ++fi) {
    for (size_t si = 0; si < cs; ++si) {
      GpuSegment& seg = *segs_[s0 + si];
      const size_t pi = fi * cs + si;
      ProgramTask t{};
      t.prog = reinterpret_cast<const ProgInstr*>(tb + o_instr) + prog_at[pi];
      t.nprog = static_cast<int>(b.progs[fq[fi]].size());
      t.words = static_cast<uint32_t>(seg.words);
      t.all = seg.all.as<uint32_t>();
      t.deletes = seg.deleted > 0 ? seg.deletes.as<uint32_t>() : nullptr;
      t.out = pair_ptr(fi, si);
      t.chunk_counts = counts_.as<uint32_t>() + pi * nchunks_w;
      t.matches = reinterpret_cast<unsigned long long*>(matches_.as<uint64_t>() + pi);
      ptasks.push_back(t);
    }
  }
  void* d;
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_ranges, ranges.data(), ranges.size() * sizeof(RangeTask), &d));
  VDBGPU_CUDA(LaunchLeafRange(static_cast<const RangeTask*>(d), static_cast<int>(ranges.size()),
                              static_cast<uint32_t>(max_words), st));
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_scat, scatters.data(), scatters.size() * sizeof(ScatterTask), &d));
  VDBGPU_CUDA(LaunchPostingScatter(static_cast<const ScatterTask*>(d), static_cast<int>(scatters.size()), st));
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_instr, instrs.data(), instrs.size() * sizeof(ProgInstr), &d));
  VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_ptask, ptasks.data(), ptasks.size() * sizeof(ProgramTask), &d));
  VDBGPU_CUDA(LaunchFilterProgram(static_cast<const ProgramTask*>(d), static_cast<int>(ptasks.size()),
                                  static_cast<uint32_t>(max_words), ctx.status_word(), st));
  matches->assign(fq.size() * cs, 0);
  VDBGPU_CUDA(cudaMemcpyAsync(matches->data(), matches_.get(), matches->size() * 8, cudaMemcpyDeviceToHost, st));
  VDBGPU_RETURN_IF_ERROR(ctx.Sync("filter bitmaps"));
  return Status::OK();
}

Status GpuCollection::FilterBitmap(Context& ctx, std::string_view filter, uint32_t segment_id, uint32_t* out,
                                   uint64_t* matches) {
  size_t si = segs_.size();
  for (size_t i = 0; i < segs_.size(); ++i)
    if (segs_[i]->id == segment_id) si = i;
  if (si == segs_.size()) return Status(Status::kNotFound, "no segment " + std::to_string(segment_id));
  Batch b;
  std::map<std::string, int> leaf_keys;
  std::unique_ptr<FilterExpr> f;
  VDBGPU_RETURN_IF_ERROR(FilterExpr::Parse(filter, opt_.schema, &f));
  Compiler c{&b.leaves, &leaf_keys};
  std::vector<Step> prog;
  c.Node(f->root(), &prog);
  if (c.max_depth > kProgStack) return Status(Status::kNotSupported, "filter too deep for the GPU evaluator");
  b.progs.push_back(std::move(prog));
  std::vector<uint64_t> m;
  VDBGPU_RETURN_IF_ERROR(Bitmaps(ctx, b, {0}, si, 1, &m));
  const uint64_t words = (segs_[si]->rows + 31) / 32;
  if (words > 0)
    VDBGPU_CUDA(cudaMemcpyAsync(out, PairBits(0, 0, 1), words * 4, cudaMemcpyDefault, ctx.stream()));
  if (matches != nullptr) *matches = m[0];
  return ctx.Sync("filter bitmap");
}

Status GpuCollection::SearchGroups(Context& ctx, Batch& b) {
  cudaStream_t st = ctx.stream();
  const size_t S = segs_.size();
  const SearchParams& p = b.r->params;
  const uint32_t G = b.F + 1;
  // ---- unfiltered queries: every segment's index (planner.cc:54-62).
  for (size_t s = 0; s < S && b.goff[b.F + 1] > b.goff[b.F]; ++s) {
    GpuSegment& seg = *segs_[s];
    b.strat[s * G + b.F] = seg.is_mutable ? "scan" : "index";
    b.matches[s * G + b.F] = seg.rows - seg.deleted;
    VDBGPU_RETURN_IF_ERROR(RunIndex(ctx, b, s, b.F, b.k, p, seg.deleted > 0 ? seg.live.as<uint32_t>() : nullptr,
                                    nullptr, 0, nullptr));
  }
  if (b.F == 0 || S == 0) return Status::OK();
  std::vector<uint32_t> fq;  // filters with at least one query
  for (uint32_t f = 0; f < b.F; ++f)
    if (b.goff[f + 1] > b.goff[f]) fq.push_back(f);
  if (fq.empty()) return Status::OK();
  const uint64_t max_words = MaxWords();
  const uint64_t nchunks_w = (max_words + kProgChunkWords - 1) / kProgChunkWords;
  const size_t chunk = SegmentsPerChunk(b, fq.size());
  for (size_t s0 = 0; s0 < S; s0 += chunk) {
    const size_t s1 = std::min(S, s0 + chunk), cs = s1 - s0;
    std::vector<uint64_t> matches;
    uint64_t t0 = NowUs();
    VDBGPU_RETURN_IF_ERROR(Bitmaps(ctx, b, fq, s0, cs, &matches));
    auto pair_ptr = [&](size_t fi, size_t si) -> uint32_t* { return PairBits(fi, si, cs); };

    // ---- plan every (filter, segment) pair (planner.cc:63-123).
    enum { kEmpty, kPre, kGraph, kPost };
    std::vector<int> plan(fq.size() * cs);
    std::vector<SearchParams> pparams(fq.size() * cs, p);
    for (size_t fi = 0; fi < fq.size(); ++fi) {
      for (size_t si = 0; si < cs; ++si) {
        const size_t pi = fi * cs + si;
        GpuSegment& seg = *segs_[s0 + si];
        const uint64_t m = matches[pi];
        const uint64_t live = seg.rows - seg.deleted;
        const double sel = live == 0 ? 0.0 : static_cast<double>(m) / static_cast<double>(live);
        int strat = p.strategy;
        if (strat == 0) {
          constexpr double kGraphCost = 10.0;
          const double sc = std::max(sel, 1e-9);
          const double graph_cost = kGraphCost * static_cast<double>(std::max<uint64_t>(p.ef, b.k)) / sc;
          strat = (m <= p.prefilter_threshold || static_cast<double>(m) <= graph_cost ||
                   seg.index->type() == kIndexFlat)
                      ? 1
                      : 2;
        }
        int pl = m == 0 ? kEmpty : (strat == 1 ? kPre : (strat == 2 ? kGraph : kPost));
        if (seg.is_mutable) pl = m == 0 ? kEmpty : kPre;  // SearchMutable: always exhaustive
        if (pl == kGraph && p.strategy == 0) {
          const double sc = std::max(sel, 1e-9);
          pparams[pi].nprobe = std::max<uint64_t>(
              p.nprobe, static_cast<uint64_t>(std::ceil(static_cast<double>(p.nprobe) / sc)));
        }
        plan[pi] = pl;
        ++stats_[pl == kEmpty ? 6 : pl == kPre ? 3 : pl == kGraph ? 4 : 5];
        if (pl == kPre) stats_[1] += m * (b.goff[fq[fi] + 1] - b.goff[fq[fi]]);
        const size_t gi = (s0 + si) * G + fq[fi];
        b.matches[gi] = m;
        b.strat[gi] = seg.is_mutable ? "scan_filter"
                      : pl == kEmpty ? "empty" : pl == kPre ? "prefilter_exact" : pl == kGraph ? "filtered_index" : "post_filter";
      }
    }

    // ---- exact over the bitmap (ExactOverBitmap, planner.cc:31-38) for prefilter pairs, and
    // for graph pairs whose search came up short (planner.cc:100-105).
    auto run_exact = [&](const std::vector<size_t>& pairs, bool fallback) -> Status {
      if (pairs.empty()) return Status::OK();
      uint64_t total_rows = 0;
      for (size_t pi : pairs) total_rows += matches[pi];
      VDBGPU_RETURN_IF_ERROR(rowlists_.ensure(std::max<uint64_t>(1, total_rows) * 4));
      std::vector<CompactTask> ct;
      std::vector<ExactItem> items;
      uint64_t off = 0;
      for (size_t pi : pairs) {
        const size_t fi = pi / cs, si = pi % cs;
        GpuSegment& seg = *segs_[s0 + si];
        CompactTask c{};
        c.bits = pair_ptr(fi, si);
        c.words = static_cast<uint32_t>(seg.words);
        c.chunk_counts = counts_.as<uint32_t>() + pi * nchunks_w;
        c.rows_out = rowlists_.as<uint32_t>() + off;
        ct.push_back(c);
        const uint32_t f = fq[fi];
        for (uint64_t q = b.goff[f]; q < b.goff[f + 1]; q += 4) {
          ExactItem it{};
          it.rows = seg.index->device_rows();
          it.list = c.rows_out;
          it.count = static_cast<uint32_t>(matches[pi]);
          it.q0 = static_cast<uint32_t>(q);
          it.nq = static_cast<uint32_t>(std::min<uint64_t>(4, b.goff[f + 1] - q));
          it.out = b.keys + ((s0 + si) * b.nq + q) * b.k;
          it.dc = b.dc + (s0 + si) * b.nq + q;
          it.only_if = fallback ? b.shortf + (s0 + si) * b.nq + q : nullptr;
          items.push_back(it);
        }
        off += matches[pi];
      }
      const size_t o_ct = 0;
      const size_t o_it = RoundUp(ct.size() * sizeof(CompactTask), 16);
      VDBGPU_RETURN_IF_ERROR(tasks_.ensure(o_it + items.size() * sizeof(ExactItem) + 16));
      void *dct, *dit;
      VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_ct, ct.data(), ct.size() * sizeof(CompactTask), &dct));
      VDBGPU_CUDA(LaunchCompactRows(static_cast<const CompactTask*>(dct), static_cast<int>(ct.size()),
                                    static_cast<uint32_t>(max_words), st));
      VDBGPU_RETURN_IF_ERROR(Stage(ctx, &tasks_, o_it, items.data(), items.size() * sizeof(ExactItem), &dit));
      ExactArgs ea{};
      ea.items = static_cast<const ExactItem*>(dit);
      ea.nitems = static_cast<int>(items.size());
      ea.queries = b.prepared;
      ea.pd = static_cast<int>(opt_.pd);
      ea.k = static_cast<int>(b.k);
      ea.metric = opt_.metric;
      ea.order = ctx.order();
      ea.out_stride = b.k;
      ea.dc_stride = 1;
      ea.status = ctx.status_word();
      VDBGPU_CUDA(LaunchExactRows(ea, st));
      // The staged tables are reused by the next launch: finish this one first.
      return ctx.Sync("exact over bitmap");
    };
    std::vector<size_t> pre, graph, post;
    for (size_t pi = 0; pi < plan.size(); ++pi) {
      if (plan[pi] == kPre) pre.push_back(pi);
      else if (plan[pi] == kGraph) graph.push_back(pi);
      else if (plan[pi] == kPost) post.push_back(pi);
    }
    stats_[9] += NowUs() - t0;
    t0 = NowUs();
    VDBGPU_RETURN_IF_ERROR(run_exact(pre, false));
    stats_[10] += NowUs() - t0;
    t0 = NowUs();
    // ---- filtered index search (planner.cc:88-105). HNSW segments: every (pair, query) walk of
    // the chunk in batched launches; other index types: one index search per pair.
    bool batched = false;
    if (!graph.empty()) {
      std::vector<const GpuIndex*> idx(cs);
      bool hnsw = true;
      for (size_t si = 0; si < cs; ++si) {
        idx[si] = segs_[s0 + si]->index.get();
        const int t = idx[si]->type();
        hnsw = hnsw && (t == kIndexHnsw || t == kIndexHnswSq8);
      }
      if (hnsw) {
        std::vector<HnswItem> items;
        for (size_t pi : graph) {
          const size_t fi = pi / cs, si = pi % cs;
          const uint32_t f = fq[fi];
          const uint32_t need = p.strategy == 0 ? static_cast<uint32_t>(std::min<uint64_t>(b.k, matches[pi])) : 0u;
          for (uint64_t q = b.goff[f]; q < b.goff[f + 1]; ++q) {
            HnswItem it{};
            it.seg = static_cast<uint32_t>(si);
            it.query = static_cast<uint32_t>(q);
            it.allow = pair_ptr(fi, si);
            it.slot = (s0 + si) * b.nq + q;
            it.need = need;
            items.push_back(it);
          }
        }
        Status st = HnswSearchMulti(ctx, idx, items.data(), items.size(), b.prepared, b.k, p, b.keys, b.dc, b.shortf,
                                    &multi_);
        if (st.ok()) {
          batched = true;
          stats_[8] += items.size();
        } else if (st.code() != Status::kNotSupported) {
          return st;
        }
      }
    }
    for (size_t pi : batched ? std::vector<size_t>() : graph) {
      const size_t fi = pi / cs, si = pi % cs, s = s0 + si;
      const uint32_t f = fq[fi];
      const uint32_t need = p.strategy == 0 ? static_cast<uint32_t>(std::min<uint64_t>(b.k, matches[pi])) : 0u;
      VDBGPU_RETURN_IF_ERROR(RunIndex(ctx, b, s, f, b.k, pparams[pi], pair_ptr(fi, si), nullptr, need,
                                      b.shortf + s * b.nq + b.goff[f]));
    }
    stats_[11] += NowUs() - t0;
    t0 = NowUs();
    if (!graph.empty() && p.strategy == 0) {
      std::vector<int> sh(S * b.nq);
      VDBGPU_CUDA(cudaMemcpyAsync(sh.data(), b.shortf, sh.size() * 4, cudaMemcpyDeviceToHost, st));
      VDBGPU_RETURN_IF_ERROR(ctx.Sync("graph search"));
      std::vector<size_t> fb;
      for (size_t pi : graph) {
        const size_t fi = pi / cs, s = s0 + pi % cs;
        const uint32_t f = fq[fi];
        uint64_t nshort = 0;
        for (uint64_t q = b.goff[f]; q < b.goff[f + 1]; ++q) nshort += sh[s * b.nq + q] != 0 ? 1 : 0;
        if (nshort > 0) fb.push_back(pi);
        stats_[1] += nshort * matches[pi];
      }
      VDBGPU_RETURN_IF_ERROR(run_exact(fb, true));
    }
    stats_[10] += NowUs() - t0;
    // ---- post-filter (planner.cc:106-123).
    for (size_t pi : post) {
      const size_t fi = pi / cs, si = pi % cs, s = s0 + si;
      GpuSegment& seg = *segs_[s];
      const uint64_t live = seg.rows - seg.deleted;
      const uint64_t kk = std::min<uint64_t>(std::max<uint64_t>(live, 1),
                                             static_cast<uint64_t>(b.k) * std::max<uint64_t>(1, p.post_filter_alpha));
      SearchParams pp = p;
      pp.ef = std::max<uint64_t>(p.ef, kk);
      VDBGPU_RETURN_IF_ERROR(RunIndex(ctx, b, s, fq[fi], static_cast<uint32_t>(std::min<uint64_t>(kk, 1u << 20)), pp,
                                      seg.deleted > 0 ? seg.live.as<uint32_t>() : nullptr, pair_ptr(fi, si), 0,
                                      nullptr));
    }
    VDBGPU_RETURN_IF_ERROR(ctx.Sync("segment chunk"));
  }
  return Status::OK();
}

}  // namespace vdbgpu
