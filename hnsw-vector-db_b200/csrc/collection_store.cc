// Host-side reading of a reference-written collection directory (declared in collection_store.h).
#include "collection_store.h"

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <functional>

#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

namespace vdbgpu {

constexpr size_t kBlobHeaderSize = 24;  // src/storage/file_format.h:13

// Whole-file reads as the reference's PosixEnv::read_file (src/storage/posix_env.cc:99-124):
// errors are IOError "<call> <path>: <strerror>". With a limit, only the first `limit` bytes.
static Status ErrnoStatus(const char* what, const std::string& path, int err) {
  return Status(Status::kIOError, std::string(what) + " " + path + ": " + std::strerror(err));
}

static Status ReadFileLimit(const std::string& path, uint64_t limit, std::string* out, uint64_t* size) {
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

// ---- The log replay of Collection::Open (CollectionImpl::Recover step 5,
// src/engine/collection_impl.cc:160-235; ApplyOp, :574-599).

// Log files (src/storage/wal.h:27-37, src/storage/wal.cc): a 16-byte header ("VDBWAL01", u32
// version 1, u32 0), then records [u32 crc32c][u32 payload length][u8 type: 1 upsert, 2 delete]
// [u64 lsn][payload]; the crc covers everything after itself. Upsert payload: u64 id, u32 dim,
// dim floats, u32 metadata length, the metadata row as EncodeMetaRow. Delete payload: u64 id.
constexpr size_t kWalFileHeaderSize = 16, kWalRecordHeaderSize = 17;


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
static Status ParseWalRecords(std::string_view data, const std::function<Status(const WalRecordView&)>& cb, bool* torn) {
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
static bool ParseNumberedName(std::string_view name, std::string_view prefix, std::string_view suffix, uint64_t* num) {
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

static std::vector<std::string> ListDir(const std::string& path) {
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
  const std::string vpath = dir + "/vectors.f32";
  if (file_size < kSegmentHeaderSize) return Status(Status::kCorruption, vpath + ": shorter than its header");
  if (std::memcmp(h, "VDBSEG01", 8) != 0) return Status(Status::kCorruption, vpath + ": bad magic");
  if (GetAt<uint32_t>(h, kSegmentHeaderSize - 4) != Crc32c(h, kSegmentHeaderSize - 4))
    return Status(Status::kCorruption, vpath + ": header checksum mismatch");
  const uint64_t data_len = GetAt<uint64_t>(h, 40);
  if (GetAt<uint32_t>(h, 8) != 1 || GetAt<uint32_t>(h, 12) != static_cast<uint32_t>(opt.metric) ||
      GetAt<uint64_t>(h, 16) != rows || GetAt<uint32_t>(h, 24) != opt.dim || GetAt<uint32_t>(h, 28) != opt.pd ||
      GetAt<uint64_t>(h, 32) != kSegmentHeaderSize || rows > (file_size / 4) ||
      data_len != rows * opt.pd * sizeof(float) || file_size - kSegmentHeaderSize < data_len)
    return Status(Status::kCorruption, vpath + ": header does not match the manifest");
  return Status::OK();
}

// The data checksum of Segment::Open with verify_crc (its default; segment_reader.cc:51-53): the
// crc32c of the rows after the header against the header's field at byte 48, read in chunks.
static Status VerifySegmentData(const std::string& dir, const char* h) {
  const std::string vpath = dir + "/vectors.f32";
  const uint64_t data_len = GetAt<uint64_t>(h, 40);
  const int fd = ::open(vpath.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return ErrnoStatus("open", vpath, errno);
  std::vector<char> buf(std::min<uint64_t>(data_len, uint64_t{64} << 20));
  uint32_t crc = 0;
  uint64_t done = 0;
  while (done < data_len) {
    const size_t want = static_cast<size_t>(std::min<uint64_t>(buf.size(), data_len - done));
    const ssize_t n = ::pread(fd, buf.data(), want, static_cast<off_t>(kSegmentHeaderSize + done));
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0) {
      const int e = n < 0 ? errno : EIO;
      ::close(fd);
      return ErrnoStatus("read", vpath, e);
    }
    crc = Crc32cExtend(crc, buf.data(), static_cast<size_t>(n));
    done += static_cast<uint64_t>(n);
  }
  ::close(fd);
  if (crc != GetAt<uint32_t>(h, 48)) return Status(Status::kCorruption, vpath + ": data checksum mismatch");
  return Status::OK();
}


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




// meta.bin as Segment::Open reads it (segment_reader.cc:71-90): the blob, the row count and
// offsets, then every row decoded as SegmentColumns::Build does (columns.cc:40-50).
static Status CheckMetaBin(const std::string& dir, uint64_t rows, const Schema& schema) {
  std::string f;
  VDBGPU_RETURN_IF_ERROR(ReadFile(dir + "/meta.bin", &f));
  std::string_view p;
  Status st = DecodeBlob(f, "VDBMETA1", &p);
  if (!st.ok()) return Status(Status::kCorruption, dir + "/meta.bin: " + st.message());
  Reader r(p);
  uint64_t n = 0;
  std::string_view offs_bytes;
  if (!r.u64(&n) || n != rows || rows >= p.size() / 8 || !r.bytes((rows + 1) * 8, &offs_bytes))
    return Status(Status::kCorruption, dir + ": bad meta.bin");
  std::vector<uint64_t> offs(rows + 1);
  std::memcpy(offs.data(), offs_bytes.data(), offs_bytes.size());
  std::string_view bytes;
  r.bytes(r.remaining(), &bytes);
  for (uint64_t i = 0; i < rows; ++i)
    if (offs[i] > offs[i + 1] || offs[i + 1] > bytes.size())
      return Status(Status::kCorruption, dir + ": bad meta.bin offsets");
  std::vector<RowValue> row(schema.size());
  for (uint64_t i = 0; i < rows; ++i)
    if (!DecodeMetaRowValues(schema, bytes.substr(offs[i], offs[i + 1] - offs[i]), &row))
      return Status(Status::kCorruption, "bad metadata at row " + std::to_string(i));
  return Status::OK();
}

// The index file's framing as LoadIndex checks it first (src/index/index.cc:46-87): length,
// checksum, a known magic. The body is parsed when the index is loaded onto a GPU.
static Status CheckIndexFraming(const std::string& dir, const char* name) {
  std::string f;
  VDBGPU_RETURN_IF_ERROR(ReadFile(dir + "/" + name, &f));
  std::string_view magic, body;
  Status st = CheckIndexFile(f, &magic, &body);
  if (!st.ok()) return Status(st.code(), dir + ": " + st.message());
  if (IndexTypeForMagic(magic) < 0) return Status(Status::kCorruption, dir + ": unknown index file magic");
  return Status::OK();
}

// Recover step 4: live rows of every segment, oldest segment first.
void LogApplier::Build(const std::vector<SegEntry>& segs) {
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
Status LogApplier::Apply(const WalRecordView& rec, uint64_t skip_below, const CollectionOptions& opt,
                         std::vector<SegEntry>& segs, MutableRows* mut) {
  if (rec.lsn <= skip_below) return Status::OK();
  if (rec.lsn != expected)
    return Status(Status::kCorruption, "log sequence gap: expected LSN " + std::to_string(expected) +
                                           ", found " + std::to_string(rec.lsn));
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
  // The record is sound: it takes its LSN (a refused record leaves the expected LSN unchanged, so
  // a live caller may send it again once corrected).
  ++expected;
  mut->last_lsn = std::max(mut->last_lsn, rec.lsn);
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

// Recover step 5 (collection_impl.cc:160-235): the records after flushed_lsn of every log, in
// order; a torn tail is accepted only at the end of the newest log (recovery truncates it there;
// this loader reads the directory without changing it).
static Status ReplayLogs(const std::vector<std::pair<std::string, std::string>>& logs, uint64_t flushed_lsn,
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

// The directory as Collection::Open recovers it (CollectionImpl::Recover, collection_impl.cc:
// 76-235), on the host: options, segments with their delete bits (those of shard `shard` of
// nshards, or of every segment when the logs hold records or `all`), and the mutable segment
// replayed from the logs. Reads only.
Status RecoverDir(const std::string& path, uint32_t shard, uint32_t nshards, bool all, CollectionOptions* opt,
                  RecoveryState* d) {
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
  // Segment::Open's checks in its order (segment_reader.cc:20-116) for the segments this shard
  // opens: the vectors header and data checksum, ids.u64, meta.bin, the index file's framing, the
  // delete set. Other shards' segments get the header check here and the rest from their owner.
  for (size_t i = 0; i < entries.size(); ++i) {
    SegEntry& e = entries[i];
    std::string h;
    uint64_t size = 0;
    VDBGPU_RETURN_IF_ERROR(ReadPrefix(e.dir + "/vectors.f32", kSegmentHeaderSize, &h, &size));
    VDBGPU_RETURN_IF_ERROR(CheckSegmentHeader(e.dir, h.data(), size, e.rows, *opt));
    if (!all && i % nshards != shard) continue;
    VDBGPU_RETURN_IF_ERROR(VerifySegmentData(e.dir, h.data()));
    VDBGPU_RETURN_IF_ERROR(LoadIds(&e));
    std::vector<uint64_t>().swap(e.ids);
    VDBGPU_RETURN_IF_ERROR(CheckMetaBin(e.dir, e.rows, opt->schema));
    VDBGPU_RETURN_IF_ERROR(CheckIndexFraming(e.dir, IndexFileName(opt->index_type)));
    VDBGPU_RETURN_IF_ERROR(LoadDeletes(&e));
  }
  // Every segment's delete set when the logs hold records (an upsert or delete may name a row of
  // any segment, so the id map needs every segment's ids).
  for (size_t i = 0; i < entries.size(); ++i)
    if (any_records && entries[i].del.empty()) VDBGPU_RETURN_IF_ERROR(LoadDeletes(&entries[i]));
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

Status GpuCollection::Inspect(const std::string& path, std::string* json) {
  RecoveryState d;
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

}  // namespace vdbgpu
