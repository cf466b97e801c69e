// Test infrastructure, not product code.
//
// A C ABI over the reference's Collection (include/vdb/collection.h) for the multi-segment,
// filtered read path: Collection::Create / BulkLoad (src/engine/collection_impl.cc:926-1016) with
// year / tags metadata, Collection::SearchBatch (:1121-1136) and Collection::Search with explain
// (:1036-1119: PrepareQuery, the per-segment planner of src/engine/planner.cc:42-129, and the
// merge by (dist, part, row) with dedupe by external id). Built into oracle/_ref/
// libvdbref_engine.so with shim/roaring.hh standing in for CRoaring (same set semantics).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <nlohmann/json.hpp>
#include <string>
#include <vector>

#include "engine/options_json.h"
#include "meta/columns.h"
#include "meta/filter.h"
#include "meta/schema.h"
#include "storage/env.h"
#include "storage/file_format.h"
#include "storage/segment.h"
#include "util/coding.h"
#include "vdb/collection.h"

namespace {
std::string g_err;
}

struct ref_coll {
  std::unique_ptr<vdb::Collection> c;
  size_t dim = 0;
};

extern "C" {

const char* ref_coll_last_error() { return g_err.c_str(); }

// options_json: the reference's collection options (engine/options_json.cc). Compaction and
// background flushing are off so every bulk load stays its own on-disk segment.
ref_coll* ref_coll_create(const char* path, const char* options_json, int threads) {
  auto j = nlohmann::json::parse(options_json, nullptr, false);
  if (j.is_discarded()) {
    g_err = "options must be JSON";
    return nullptr;
  }
  vdb::CollectionOptions o;
  vdb::Status s = vdb::OptionsFromJson(j, &o);
  if (!s.ok()) {
    g_err = s.ToString();
    return nullptr;
  }
  vdb::OpenOptions oo;
  oo.num_threads = static_cast<size_t>(threads);
  oo.auto_compact = false;
  oo.auto_flush = false;
  auto c = vdb::Collection::Create(path, o, oo);
  if (!c.ok()) {
    g_err = c.status().ToString();
    return nullptr;
  }
  auto* h = new ref_coll;
  h->c = std::move(c).value();
  h->dim = o.dim;
  return h;
}

// Collection::Open of an existing directory (crash recovery: the logs are replayed into the
// mutable segment), without background flushes or compactions.
ref_coll* ref_coll_open(const char* path, int threads) {
  vdb::OpenOptions oo;
  oo.num_threads = static_cast<size_t>(threads);
  oo.auto_compact = false;
  oo.auto_flush = false;
  auto c = vdb::Collection::Open(path, oo);
  if (!c.ok()) {
    g_err = c.status().ToString();
    return nullptr;
  }
  auto* h = new ref_coll;
  h->c = std::move(c).value();
  h->dim = h->c->options().dim;
  return h;
}

void ref_coll_free(ref_coll* h) {
  if (h == nullptr) return;
  if (h->c) (void)h->c->Close();
  delete h;
}

// One segment: n rows (dim floats each), external ids, year (int64) and up to max_tags tags per
// row given as word ids (UINT32_MAX = unused), stored as keyword strings "w<id>".
int ref_coll_bulk_load(ref_coll* h, const uint64_t* ids, const float* vectors, uint64_t n,
                       const int64_t* years, const uint32_t* tags, uint32_t max_tags) {
  std::vector<vdb::Metadata> md;
  if (years != nullptr) {
    md.resize(n);
    for (uint64_t i = 0; i < n; ++i) {
      md[i]["year"] = years[i];
      std::vector<std::string> t;
      for (uint32_t j = 0; j < max_tags; ++j) {
        const uint32_t w = tags[i * max_tags + j];
        if (w != UINT32_MAX) t.push_back("w" + std::to_string(w));
      }
      md[i]["tags"] = t;
    }
  }
  vdb::Status s = h->c->BulkLoad(ids, vectors, n, years != nullptr ? &md : nullptr);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  return 0;
}

// One segment with arbitrary metadata: meta_json is a JSON array of n objects (null = none),
// converted by MetadataFromJson (src/meta/schema.cc:179) against the collection's schema.
int ref_coll_bulk_load_json(ref_coll* h, const uint64_t* ids, const float* vectors, uint64_t n,
                            const char* meta_json) {
  std::vector<vdb::Metadata> md;
  if (meta_json != nullptr) {
    auto j = nlohmann::json::parse(meta_json, nullptr, false);
    if (j.is_discarded() || !j.is_array() || j.size() != n) {
      g_err = "metadata must be a JSON array with one entry per row";
      return 3;
    }
    md.resize(n);
    for (uint64_t i = 0; i < n; ++i) {
      vdb::Status s = vdb::MetadataFromJson(j[i], h->c->options().schema, &md[i]);
      if (!s.ok()) {
        g_err = s.ToString();
        return static_cast<int>(s.code());
      }
    }
  }
  vdb::Status s = h->c->BulkLoad(ids, vectors, n, meta_json != nullptr ? &md : nullptr);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  return 0;
}

// Collection::UpsertBatch of n rows with metadata as ref_coll_bulk_load_json (null = none): one
// log record per row (src/engine/collection_impl.cc:460-540).
int ref_coll_upsert_json(ref_coll* h, const uint64_t* ids, const float* vectors, uint64_t n,
                         const char* meta_json) {
  std::vector<vdb::Metadata> md;
  if (meta_json != nullptr) {
    auto j = nlohmann::json::parse(meta_json, nullptr, false);
    if (j.is_discarded() || !j.is_array() || j.size() != n) {
      g_err = "metadata must be a JSON array with one entry per row";
      return 3;
    }
    md.resize(n);
    for (uint64_t i = 0; i < n; ++i) {
      vdb::Status s = vdb::MetadataFromJson(j[i], h->c->options().schema, &md[i]);
      if (!s.ok()) {
        g_err = s.ToString();
        return static_cast<int>(s.code());
      }
    }
  }
  vdb::Status s = h->c->UpsertBatch(ids, vectors, n, meta_json != nullptr ? &md : nullptr);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  return 0;
}

// Collection::RemoveBatch; *removed = how many ids were live.
int ref_coll_remove(ref_coll* h, const uint64_t* ids, uint64_t n, uint64_t* removed) {
  size_t r = 0;
  vdb::Status s = h->c->RemoveBatch(ids, n, &r);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  if (removed != nullptr) *removed = r;
  return 0;
}

// Collection::Flush (synchronous).
int ref_coll_flush(ref_coll* h) {
  vdb::Status s = h->c->Flush();
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  return 0;
}

// Collection::Stats as JSON (the row and log fields, and per segment id / kind / index / rows /
// deleted / lsn).
int ref_coll_stats(ref_coll* h, char* out, size_t cap) {
  const vdb::CollectionStats st = h->c->Stats();
  nlohmann::json j = {{"live_rows", st.live_rows}, {"total_rows", st.total_rows},
                      {"deleted_rows", st.deleted_rows}, {"last_lsn", st.last_lsn},
                      {"flushed_lsn", st.flushed_lsn}, {"recovery_records", st.last_recovery_records}};
  j["segments"] = nlohmann::json::array();
  for (const auto& s : st.segments)
    j["segments"].push_back({{"id", s.id}, {"kind", s.kind}, {"index", s.index}, {"rows", s.rows},
                             {"deleted", s.deleted}, {"lsn", s.lsn}});
  const std::string text = j.dump();
  if (text.size() + 1 > cap) {
    g_err = "stats buffer too small";
    return 7;
  }
  std::memcpy(out, text.c_str(), text.size() + 1);
  return 0;
}

// The filter bitmap of one segment: SegmentColumns::Build over the segment's meta.bin
// (segment_reader.cc:75-95) then SegmentColumns::Evaluate (columns.cc:185-205). out receives
// (rows + 31) / 32 words, bit r of word r / 32 set for every matching row.
int ref_segment_filter_bitmap(const char* segment_dir, const char* schema_json,
                              const char* filter_json, uint32_t* out, uint64_t rows) {
  auto sj = nlohmann::json::parse(schema_json, nullptr, false);
  vdb::Schema schema;
  vdb::Status s = sj.is_discarded() ? vdb::Status::InvalidArgument("schema must be JSON")
                                    : vdb::SchemaFromJson(sj, &schema);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  std::string storage;
  std::string_view payload;
  s = vdb::ReadBlobFile(vdb::Env::Default(), std::string(segment_dir) + "/meta.bin", vdb::kMetaMagic,
                        &storage, &payload);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  vdb::ByteReader r(payload);
  uint64_t n = 0;
  std::string_view offs_bytes;
  if (!r.GetU64(&n) || n != rows || !r.GetBytes((rows + 1) * sizeof(uint64_t), &offs_bytes)) {
    g_err = "bad meta.bin";
    return 9;
  }
  std::vector<uint64_t> offs(rows + 1);
  std::memcpy(offs.data(), offs_bytes.data(), offs_bytes.size());
  std::string_view bytes(r.position(), r.remaining());
  vdb::SegmentColumns cols;
  s = cols.Build(schema, rows, [&](size_t i) { return bytes.substr(offs[i], offs[i + 1] - offs[i]); });
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  auto f = vdb::FilterExpr::Parse(filter_json, schema);
  if (!f.ok()) {
    g_err = f.status().ToString();
    return static_cast<int>(f.status().code());
  }
  roaring::Roaring bm = cols.Evaluate((*f)->root());
  std::memset(out, 0, (rows + 31) / 32 * 4);
  for (uint32_t row : bm) out[row >> 5] |= 1u << (row & 31);
  return 0;
}

// FilterExpr::Parse alone (src/meta/filter_parser.cc): 0, or the status code with the message
// in ref_coll_last_error().
int ref_filter_parse(const char* schema_json, const char* filter_json) {
  auto sj = nlohmann::json::parse(schema_json, nullptr, false);
  vdb::Schema schema;
  vdb::Status s = sj.is_discarded() ? vdb::Status::InvalidArgument("schema must be JSON")
                                    : vdb::SchemaFromJson(sj, &schema);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  auto f = vdb::FilterExpr::Parse(filter_json, schema);
  if (!f.ok()) {
    g_err = f.status().message();
    return static_cast<int>(f.status().code());
  }
  g_err = (*f)->ToString();
  return 0;
}

// Collection::SearchBatch with an optional JSON filter. Misses: UINT64_MAX / +inf.
// Collection::RemoveBatch then Collection::Flush: the deletes reach the disk segments' persisted
// delete sets (deletes-<n>.roar, CollectionImpl::FlushFrozen).
// RemoveBatch, then UpsertBatch of nup rows (an upsert of an id on disk deletes its old row), then
// Flush. Flush persists the delete sets of disk segments only when the mutable segment holds rows
// (CollectionImpl::FlushOnce, src/engine/collection_impl.cc:649-650), hence the upserts.
int ref_coll_remove_flush(ref_coll* h, const uint64_t* ids, uint64_t n, const uint64_t* up_ids,
                          const float* up_vectors, uint64_t nup, uint64_t* removed) {
  size_t r = 0;
  vdb::Status s = h->c->RemoveBatch(ids, n, &r);
  if (s.ok() && nup > 0) s = h->c->UpsertBatch(up_ids, up_vectors, nup);
  if (s.ok()) s = h->c->Flush();
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  if (removed != nullptr) *removed = r;
  return 0;
}

int ref_coll_search_batch(ref_coll* h, const float* q, uint64_t nq, uint32_t k, uint64_t ef,
                          uint64_t nprobe, int rerank, int strategy, uint64_t prefilter_threshold,
                          uint64_t post_filter_alpha, const char* filter_json, uint64_t* out_ids,
                          float* out_dist) {
  vdb::SearchParams p;
  p.ef = ef;
  p.nprobe = nprobe;
  p.rerank = rerank;
  p.strategy = static_cast<vdb::FilterStrategy>(strategy);
  p.prefilter_threshold = prefilter_threshold;
  p.post_filter_alpha = post_filter_alpha;
  std::unique_ptr<vdb::Filter> f;
  if (filter_json != nullptr) {
    auto pf = h->c->ParseFilter(filter_json);
    if (!pf.ok()) {
      g_err = pf.status().ToString();
      return static_cast<int>(pf.status().code());
    }
    f = std::move(pf).value();
  }
  std::vector<std::vector<vdb::SearchHit>> hits;
  vdb::Status s = h->c->SearchBatch(q, nq, k, p, f.get(), &hits);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  for (uint64_t i = 0; i < nq; ++i)
    for (uint32_t j = 0; j < k; ++j) {
      const bool have = j < hits[i].size();
      out_ids[i * k + j] = have ? hits[i][j].id : UINT64_MAX;
      out_dist[i * k + j] = have ? hits[i][j].distance : INFINITY;
    }
  return 0;
}

// Collection::Search of one query with explain: per part (mutable first, then disk segments in
// snapshot order) the strategy name, matches and distance computations, as JSON.
int ref_coll_explain(ref_coll* h, const float* q, uint32_t k, uint64_t ef, uint64_t nprobe,
                     int rerank, int strategy, uint64_t prefilter_threshold,
                     uint64_t post_filter_alpha, const char* filter_json, char* out, size_t cap) {
  vdb::SearchRequest req;
  req.vector = q;
  req.k = k;
  req.params.ef = ef;
  req.params.nprobe = nprobe;
  req.params.rerank = rerank;
  req.params.strategy = static_cast<vdb::FilterStrategy>(strategy);
  req.params.prefilter_threshold = prefilter_threshold;
  req.params.post_filter_alpha = post_filter_alpha;
  std::unique_ptr<vdb::Filter> f;
  if (filter_json != nullptr) {
    auto pf = h->c->ParseFilter(filter_json);
    if (!pf.ok()) {
      g_err = pf.status().ToString();
      return static_cast<int>(pf.status().code());
    }
    f = std::move(pf).value();
    req.filter = f.get();
  }
  std::vector<vdb::SearchHit> hits;
  vdb::SearchExplain ex;
  vdb::Status s = h->c->Search(req, &hits, &ex);
  if (!s.ok()) {
    g_err = s.ToString();
    return static_cast<int>(s.code());
  }
  nlohmann::json j = nlohmann::json::array();
  for (const auto& e : ex.segments)
    j.push_back({{"id", e.segment_id}, {"kind", e.kind}, {"strategy", e.strategy}, {"index", e.index},
                 {"matches", e.matches}, {"live_rows", e.live_rows}, {"ef", e.ef},
                 {"distance_computations", e.distance_computations}, {"results", e.results}});
  const std::string str = j.dump();
  if (str.size() + 1 > cap) return -1;
  std::memcpy(out, str.c_str(), str.size() + 1);
  return 0;
}

}  // extern "C"
