#include "collection.h"
#include "collection_store.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <unordered_map>

#include "formats.h"
#include "hnsw.cuh"

namespace vdbgpu {

namespace {

uint64_t NowUs() {
  return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::microseconds>(
                                   std::chrono::steady_clock::now().time_since_epoch())
                                   .count());
}

constexpr uint64_t kMaxK = 10000;            // include/vdb/collection.h kMaxK
constexpr uint32_t kMaxGpuK = 240;
constexpr uint32_t kScatterChunk = 16384;

uint64_t RoundUp(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

// Memory of the context's device (or managed). Search rejects other GPUs' buffers first, so
// false means host memory, staged through a copy.
bool OnDevice(const void* p, int device) {
  return p != nullptr && WherePointer(p, device) == MemWhere::kDevice;
}

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

Status GpuCollection::Open(Context& ctx, const std::string& path, uint32_t shard, uint32_t nshards,
                           std::unique_ptr<GpuCollection>* out) {
  if (nshards == 0 || shard >= nshards) return Status(Status::kInvalidArgument, "bad shard");
  auto c = std::make_unique<GpuCollection>();
  c->log_ = std::make_shared<RecoveryState>();
  RecoveryState& d = *c->log_;
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
  const RecoveryState& d = *log_;
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
  RecoveryState& d = *log_;
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
  VDBGPU_RETURN_IF_ERROR(RejectOtherDevice(r.queries, ctx.device(), "the query buffer"));
  VDBGPU_RETURN_IF_ERROR(RejectOtherDevice(r.out_ids, ctx.device(), "the id output"));
  VDBGPU_RETURN_IF_ERROR(RejectOtherDevice(r.out_dist, ctx.device(), "the distance output"));
  VDBGPU_RETURN_IF_ERROR(RejectOtherDevice(r.out_records, ctx.device(), "the hit output"));
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
  if (!OnDevice(r.queries, ctx.device())) {
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
  const bool rec_dev = OnDevice(r.out_records, ctx.device()),
             ids_dev_ok = OnDevice(r.out_ids, ctx.device()) && OnDevice(r.out_dist, ctx.device());
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
    // The reference always searches a mutable segment, empty or not (collection_impl.cc:1056-1059;
    // SearchMutable, planner.cc:131-149): with no rows it is explained as a scan of nothing. Shard
    // 0 of a collection opened from a directory reports it the same way.
    const bool has_mutable = std::any_of(segs_.begin(), segs_.end(), [](const auto& x) { return x->is_mutable; });
    if (log_ && log_->shard == 0 && !has_mutable) {
      for (uint64_t i = 0; i < b.nq; ++i) {
        PartExplain e;
        e.segment_id = log_->mutable_id;
        e.is_mutable = true;
        e.strategy = gof[i] < b.F ? "scan_filter" : "scan";
        auto& parts = (*r.explain)[b.perm[i]];
        parts.insert(parts.begin(), e);
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
        // Walks of the rarest filters first: a filtered walk runs until it holds ef allowed rows,
        // so the fewer rows a filter allows the longer its walks are, and starting the long walks
        // first keeps them out of the launch's tail. Each walk writes its own slot, so the order
        // changes no result.
        std::vector<size_t> order(graph);
        std::stable_sort(order.begin(), order.end(), [&](size_t x, size_t y) { return matches[x] < matches[y]; });
        std::vector<HnswItem> items;
        for (size_t pi : order) {
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
