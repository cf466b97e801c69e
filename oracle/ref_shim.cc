// Test infrastructure, not product code.
//
// A C ABI over the reference's own index layer (vdb, compiled in place from its sources by
// oracle/Makefile into oracle/_ref/libvdbref.so). Tests use it to produce ground truth and
// golden fixtures, and bench.py's cpu_baseline leg times it. Nothing in the product links it.
//
// Every entry point forwards to the reference's public classes and functions:
//   CreateIndex / Index::build / Index::save / LoadIndex   src/index/index.h:58-62, index.cc:16-87
//   Index::search (concurrently, one query per task)         src/index/index.h:44-45
//   FlatSearchBatch                                          src/index/flat_index.cc:41-68
//   Sq8Quantizer train/encode/serialize                      src/index/quant/sq8.cc:9-64
//   MetricDistance / MetricSq8Distance / Kernels()           src/distance/cpu_features.cc:62-73
//   TopK / Rerank                                            src/util/topk.h:13-54, src/index/index.cc:89-95
//   NormalizeVector                                          src/util/dataset.cc:33-40
// The only composition of our own is ref_sq8_scan_search: the exhaustive SQ8 scan with an fp32
// re-rank has no reference index type, so it is built from the reference primitives above.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "distance/distance.h"
#include "index/flat_index.h"
#include "index/index.h"
#include "index/quant/sq8.h"
#include "storage/env.h"
#include "util/aligned_buffer.h"
#include "util/dataset.h"
#include "util/thread_pool.h"
#include "util/topk.h"
#include "vdb/options.h"
#include "vdb/types.h"

namespace {

class StringFile final : public vdb::WritableFile {
 public:
  using vdb::WritableFile::append;
  vdb::Status append(std::span<const std::byte> d) override {
    data.append(reinterpret_cast<const char*>(d.data()), d.size());
    return vdb::Status::OK();
  }
  vdb::Status sync() override { return vdb::Status::OK(); }
  vdb::Status close() override { return vdb::Status::OK(); }
  uint64_t size() const override { return data.size(); }
  std::string data;
};

// Rows allowed by a dense bitset (bit r of word r/64).
class BitsetFilter final : public vdb::RowFilter {
 public:
  explicit BitsetFilter(const uint64_t* bits) : bits_(bits) {}
  bool allowed(vdb::InternalId id) const override { return (bits_[id >> 6] >> (id & 63)) & 1u; }

 private:
  const uint64_t* bits_;
};

std::string g_error;

}  // namespace

struct ref_index {
  vdb::AlignedBuffer rows;
  vdb::VectorView view;
  vdb::Metric metric = vdb::Metric::L2;
  vdb::IndexOptions opts;
  std::unique_ptr<vdb::Index> index;
};

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

const char* ref_kernel_set() { return vdb::Kernels().name; }

// One distance with the runtime-selected reference kernels. which: 0 = l2, 1 = dot, 2 = ip.
float ref_distance(int which, const float* a, const float* b, size_t d) {
  const vdb::KernelSet& k = vdb::Kernels();
  return which == 0 ? k.l2(a, b, d) : which == 1 ? k.dot(a, b, d) : k.ip(a, b, d);
}

float ref_sq8_distance(int metric, const float* q, const uint8_t* code, const float* vmin,
                       const float* scale, size_t d) {
  return vdb::MetricSq8Distance(static_cast<vdb::Metric>(metric))(q, code, vmin, scale, d);
}

// vdb::NormalizeVector on every row (rows of `stride` floats, first `dim` used). Returns the
// number of rows that could not be normalized.
uint64_t ref_normalize_rows(float* rows, uint64_t n, uint32_t dim, uint32_t stride) {
  uint64_t bad = 0;
  for (uint64_t i = 0; i < n; ++i) bad += vdb::NormalizeVector(rows + i * stride, dim) ? 0 : 1;
  return bad;
}

static ref_index* MakeHandle(int metric, const float* rows, uint64_t n, uint32_t dim, uint32_t pd) {
  auto* h = new ref_index;
  h->rows.reset(static_cast<size_t>(n) * pd * sizeof(float));
  if (n > 0) std::memcpy(h->rows.data(), rows, static_cast<size_t>(n) * pd * sizeof(float));
  h->view = vdb::VectorView{h->rows.floats(), static_cast<size_t>(n), dim, pd};
  h->metric = static_cast<vdb::Metric>(metric);
  return h;
}

// CreateIndex + build. threads == 1 builds on the calling thread (deterministic HNSW);
// threads == 0 uses every core.
ref_index* ref_index_build(int type, int metric, const float* rows, uint64_t n, uint32_t dim,
                           uint32_t pd, uint32_t M, uint32_t efc, uint32_t pq_m, uint32_t nlist,
                           uint32_t max_train_ppc, uint64_t seed, int threads) {
  ref_index* h = MakeHandle(metric, rows, n, dim, pd);
  h->opts.type = static_cast<vdb::IndexType>(type);
  h->opts.M = M;
  h->opts.ef_construction = efc;
  h->opts.pq_m = pq_m;
  h->opts.nlist = nlist;
  h->opts.max_train_points_per_centroid = max_train_ppc;
  h->opts.seed = seed;
  auto idx = vdb::CreateIndex(h->opts, h->metric, h->view);
  if (!idx.ok()) {
    g_error = idx.status().ToString();
    delete h;
    return nullptr;
  }
  h->index = std::move(idx).value();
  vdb::Status st;
  if (threads == 1) {
    st = h->index->build(nullptr);
  } else {
    vdb::ThreadPool pool(static_cast<size_t>(threads));
    st = h->index->build(&pool);
  }
  if (!st.ok()) {
    g_error = st.ToString();
    delete h;
    return nullptr;
  }
  return h;
}

// LoadIndex over a copy of `rows`.
ref_index* ref_index_load(const void* bytes, size_t nbytes, int metric, const float* rows,
                          uint64_t n, uint32_t dim, uint32_t pd, uint32_t pq_m) {
  ref_index* h = MakeHandle(metric, rows, n, dim, pd);
  h->opts.pq_m = pq_m;
  auto idx = vdb::LoadIndex(std::string_view(static_cast<const char*>(bytes), nbytes), h->opts,
                            h->metric, h->view);
  if (!idx.ok()) {
    g_error = idx.status().ToString();
    delete h;
    return nullptr;
  }
  h->index = std::move(idx).value();
  return h;
}

// Index::extend (src/index/index.h:53-54) over a copy of `rows` (n rows, the first ones the
// index's own); threads as in ref_index_build. A new handle, or null with ref_last_error.
ref_index* ref_index_extend(const ref_index* h, const float* rows, uint64_t n, int threads) {
  ref_index* e = MakeHandle(static_cast<int>(h->metric), rows, n, static_cast<uint32_t>(h->view.dim),
                            static_cast<uint32_t>(h->view.padded_dim));
  e->opts = h->opts;
  vdb::StatusOr<std::unique_ptr<vdb::Index>> r = vdb::Status::Internal("unreached");
  if (threads == 1) {
    r = h->index->extend(e->view, nullptr);
  } else {
    vdb::ThreadPool pool(static_cast<size_t>(threads));
    r = h->index->extend(e->view, &pool);
  }
  if (!r.ok()) {
    g_error = r.status().ToString();
    delete e;
    return nullptr;
  }
  e->index = std::move(r).value();
  return e;
}

void ref_index_free(ref_index* h) { delete h; }

int ref_index_type(const ref_index* h) { return static_cast<int>(h->index->type()); }

// Index::save into a malloc'ed buffer (free with ref_free). Returns the size, 0 on error.
size_t ref_index_save(const ref_index* h, void** out) {
  StringFile f;
  vdb::Status st = h->index->save(f);
  if (!st.ok()) {
    g_error = st.ToString();
    *out = nullptr;
    return 0;
  }
  void* p = std::malloc(f.data.size());
  std::memcpy(p, f.data.data(), f.data.size());
  *out = p;
  return f.data.size();
}

void ref_free(void* p) { std::free(p); }

// Index::search for nq queries (nq x pd floats), threads as in ref_index_build. Missing results
// are written as (+inf, UINT32_MAX). out_count[q] = hits returned, out_dc[q] = distance
// computations (IndexSearchStats). allow_bits may be null.
void ref_index_search(const ref_index* h, const float* q, uint64_t nq, uint32_t k, uint64_t ef,
                      uint64_t nprobe, int rerank, const uint64_t* allow_bits, int threads,
                      float* out_dist, uint32_t* out_id, uint32_t* out_count, uint64_t* out_dc) {
  vdb::SearchParams p;
  p.ef = ef;
  p.nprobe = nprobe;
  p.rerank = rerank;
  BitsetFilter bf(allow_bits);
  const vdb::RowFilter* filter = allow_bits != nullptr ? &bf : nullptr;
  const size_t pd = h->view.padded_dim;
  auto one = [&](size_t i) {
    std::vector<vdb::Neighbor> out;
    vdb::IndexSearchStats st;
    h->index->search(q + i * pd, k, p, filter, out, &st);
    for (uint32_t j = 0; j < k; ++j) {
      bool have = j < out.size();
      out_dist[i * k + j] = have ? out[j].dist : INFINITY;
      out_id[i * k + j] = have ? out[j].id : UINT32_MAX;
    }
    if (out_count != nullptr) out_count[i] = static_cast<uint32_t>(out.size());
    if (out_dc != nullptr) out_dc[i] = st.distance_computations;
  };
  if (threads == 1) {
    for (size_t i = 0; i < nq; ++i) one(i);
  } else {
    vdb::ThreadPool pool(static_cast<size_t>(threads));
    pool.parallel_for(0, nq, one, 16);
  }
}

// FlatSearchBatch (the reference's ground-truth producer).
void ref_flat_search_batch(int metric, const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                           const float* q, uint64_t nq, uint32_t k, int threads, float* out_dist,
                           uint32_t* out_id) {
  vdb::VectorView v{rows, static_cast<size_t>(n), dim, pd};
  std::vector<std::vector<vdb::Neighbor>> out;
  vdb::DistFn fn = vdb::MetricDistance(static_cast<vdb::Metric>(metric));
  if (threads == 1) {
    vdb::FlatSearchBatch(v, fn, q, nq, k, out, nullptr);
  } else {
    vdb::ThreadPool pool(static_cast<size_t>(threads));
    vdb::FlatSearchBatch(v, fn, q, nq, k, out, &pool);
  }
  for (size_t i = 0; i < nq; ++i)
    for (uint32_t j = 0; j < k; ++j) {
      bool have = j < out[i].size();
      out_dist[i * k + j] = have ? out[i][j].dist : INFINITY;
      out_id[i * k + j] = have ? out[i][j].id : UINT32_MAX;
    }
}

// Sq8Quantizer::train on all rows, then encode every row (padded_dim bytes per row).
// vmin/scale receive padded_dim floats each.
void ref_sq8_train_encode(const float* rows, uint64_t n, uint32_t dim, uint32_t pd, float* vmin,
                          float* scale, uint8_t* codes, int threads) {
  vdb::VectorView v{rows, static_cast<size_t>(n), dim, pd};
  vdb::Sq8Quantizer sq;
  sq.train(v);
  std::memcpy(vmin, sq.vmin(), pd * sizeof(float));
  std::memcpy(scale, sq.scale(), pd * sizeof(float));
  auto enc = [&](size_t b, size_t e) {
    for (size_t i = b; i < e; ++i) sq.encode(v.row(i), codes + i * pd);
  };
  if (threads == 1) {
    enc(0, n);
  } else {
    vdb::ThreadPool pool(static_cast<size_t>(threads));
    vdb::ParallelForRange(&pool, 0, n, enc, 4096);
  }
}

// The exhaustive SQ8 scan with an fp32 re-rank, composed from reference primitives:
// MetricSq8Distance over every code -> TopK(depth) -> Rerank(MetricDistance) -> k.
// out_pre (nullable, nq x depth) receives the pre-rank top-`depth` (dist, id), closest first.
void ref_sq8_scan_search(int metric, const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                         const uint8_t* codes, const float* vmin, const float* scale,
                         const float* q, uint64_t nq, uint32_t k, uint32_t depth, int threads,
                         float* out_dist, uint32_t* out_id, float* out_pre_dist,
                         uint32_t* out_pre_id) {
  vdb::VectorView v{rows, static_cast<size_t>(n), dim, pd};
  const vdb::Metric m = static_cast<vdb::Metric>(metric);
  vdb::Sq8DistFn sfn = vdb::MetricSq8Distance(m);
  vdb::DistFn fn = vdb::MetricDistance(m);
  auto one = [&](size_t i) {
    const float* qi = q + i * pd;
    vdb::TopK top(depth);
    for (size_t r = 0; r < n; ++r)
      top.push(sfn(qi, codes + r * pd, vmin, scale, pd), static_cast<vdb::InternalId>(r));
    std::vector<vdb::Neighbor> cands = top.sorted(), out;
    if (out_pre_dist != nullptr) {
      for (uint32_t j = 0; j < depth; ++j) {
        bool have = j < cands.size();
        out_pre_dist[i * depth + j] = have ? cands[j].dist : INFINITY;
        out_pre_id[i * depth + j] = have ? cands[j].id : UINT32_MAX;
      }
    }
    vdb::Rerank(v, fn, qi, cands, k, out, nullptr);
    for (uint32_t j = 0; j < k; ++j) {
      bool have = j < out.size();
      out_dist[i * k + j] = have ? out[j].dist : INFINITY;
      out_id[i * k + j] = have ? out[j].id : UINT32_MAX;
    }
  };
  if (threads == 1) {
    for (size_t i = 0; i < nq; ++i) one(i);
  } else {
    vdb::ThreadPool pool(static_cast<size_t>(threads));
    pool.parallel_for(0, nq, one, 1);
  }
}

// TopK over (dist, id) pairs pushed in order, result closest first (src/util/topk.h:13-54).
uint32_t ref_topk(const float* dist, const uint32_t* id, uint64_t n, uint32_t k, float* out_dist,
                  uint32_t* out_id) {
  vdb::TopK top(k);
  for (uint64_t i = 0; i < n; ++i) top.push(dist[i], id[i]);
  std::vector<vdb::Neighbor> s = top.sorted();
  for (size_t j = 0; j < s.size(); ++j) {
    out_dist[j] = s[j].dist;
    out_id[j] = s[j].id;
  }
  return static_cast<uint32_t>(s.size());
}

}  // extern "C"
