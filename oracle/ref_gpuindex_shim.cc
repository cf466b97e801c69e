// Test infrastructure (not shipped): the reference's own segment search path driven over two copies
// of a collection directory's disk segments, one opened by Segment::Open as the reference does
// (its CPU index loaded from index.<type>), the other with vdb::GpuIndex handed to Segment::Open as
// the segment's prebuilt index (src/storage/segment_reader.cc:20-27). Both are searched by the
// reference's SearchDiskSegment (src/engine/planner.cc:42-129): same planner, same filter bitmaps,
// same exact search over bitmaps; only Index::search differs. Built by `make -C oracle gpuindex`
// against the reference sources and lib/libvdbgpu.so.
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include <nlohmann/json.hpp>

#include "engine/planner.h"
#include "gpu_index.h"
#include "meta/filter.h"
#include "storage/env.h"
#include "storage/manifest.h"
#include "storage/segment.h"
#include "util/dataset.h"
#include "vdbgpu.h"

namespace {

std::string g_err;

struct gi_coll {
  vdb::Manifest manifest;
  std::vector<std::shared_ptr<vdb::Segment>> cpu;  // owns the rows the GPU copies were loaded from
  std::vector<std::shared_ptr<vdb::Segment>> segs; // the segments searched
  vdbgpu_ctx* ctx = nullptr;
  ~gi_coll() {
    segs.clear();
    cpu.clear();
    if (ctx != nullptr) vdbgpu_close(ctx);
  }
};

}  // namespace

extern "C" {

const char* gi_last_error() { return g_err.c_str(); }

// Opens every disk segment of the collection at `dir`. use_gpu: each segment's index is a
// vdb::GpuIndex on `device` loaded from the segment's own index file.
gi_coll* gi_open(const char* dir, int use_gpu, int device) {
  auto h = std::make_unique<gi_coll>();
  vdb::Env* env = vdb::Env::Default();
  vdb::Status s = vdb::ReadCurrentManifest(env, dir, &h->manifest);
  if (!s.ok()) {
    g_err = s.ToString();
    return nullptr;
  }
  const vdb::CollectionOptions& opts = h->manifest.options;
  if (use_gpu && vdbgpu_open(device, &h->ctx) != VDBGPU_OK) {
    g_err = "vdbgpu_open failed";
    return nullptr;
  }
  const std::string seg_dir = vdb::JoinPath(dir, "segments");
  for (const vdb::SegmentMeta& sm : h->manifest.segments) {
    const std::string sdir = vdb::JoinPath(seg_dir, vdb::SegmentDirName(sm.id));
    auto cpu = vdb::Segment::Open(env, sdir, sm, opts, true);
    if (!cpu.ok()) {
      g_err = cpu.status().ToString();
      return nullptr;
    }
    if (!use_gpu) {
      h->segs.push_back(*cpu);
      continue;
    }
    std::string bytes;
    s = env->read_file(vdb::JoinPath(sdir, vdb::IndexFileName(opts.index.type)), &bytes);
    if (!s.ok()) {
      g_err = s.ToString();
      return nullptr;
    }
    auto gi = vdb::GpuIndex::Load(h->ctx, bytes, opts.metric, (*cpu)->vectors());
    if (!gi.ok()) {
      g_err = gi.status().ToString();
      return nullptr;
    }
    auto seg = vdb::Segment::Open(env, sdir, sm, opts, true, nullptr, nullptr, std::move(gi).value());
    if (!seg.ok()) {
      g_err = seg.status().ToString();
      return nullptr;
    }
    h->cpu.push_back(*cpu);
    h->segs.push_back(*seg);
  }
  return h.release();
}

void gi_close(gi_coll* h) { delete h; }

uint32_t gi_segments(const gi_coll* h) { return static_cast<uint32_t>(h->segs.size()); }

// One query through SearchDiskSegment on every segment: PrepareQuery's padding and cosine
// normalisation (collection_impl.cc:1023-1034), then per segment its hits (segment-local rows,
// closest first; out_* hold k slots per segment, out_count the hits) and its explain as JSON.
int gi_search(gi_coll* h, const float* v, uint32_t k, uint64_t ef, uint64_t nprobe, int rerank, int strategy,
              uint64_t prefilter_threshold, uint64_t post_filter_alpha, const char* filter_json, float* out_dist,
              uint32_t* out_row, uint32_t* out_count, char* explain, size_t cap) {
  const vdb::CollectionOptions& opts = h->manifest.options;
  std::vector<float> q(vdb::PaddedDim(opts.dim), 0.f);
  std::memcpy(q.data(), v, opts.dim * sizeof(float));
  if (opts.metric == vdb::Metric::Cosine && !vdb::NormalizeVector(q.data(), opts.dim)) {
    g_err = "zero query";
    return 1;
  }
  std::unique_ptr<vdb::FilterExpr> filter;
  if (filter_json != nullptr) {
    auto f = vdb::FilterExpr::Parse(filter_json, opts.schema);
    if (!f.ok()) {
      g_err = f.status().ToString();
      return static_cast<int>(f.status().code());
    }
    filter = std::move(f).value();
  }
  vdb::SearchParams p;
  p.ef = ef;
  p.nprobe = nprobe;
  p.rerank = rerank;
  p.strategy = static_cast<vdb::FilterStrategy>(strategy);
  p.prefilter_threshold = prefilter_threshold;
  p.post_filter_alpha = post_filter_alpha;
  const vdb::DistFn fn = vdb::MetricDistance(opts.metric);
  nlohmann::json ex = nlohmann::json::array();
  for (size_t i = 0; i < h->segs.size(); ++i) {
    vdb::SegmentHits sh;
    vdb::SearchDiskSegment(*h->segs[i], q.data(), k, p, filter.get(), fn, &sh);
    out_count[i] = static_cast<uint32_t>(std::min<size_t>(sh.hits.size(), k));
    for (uint32_t j = 0; j < k; ++j) {
      const bool have = j < sh.hits.size();
      out_dist[i * k + j] = have ? sh.hits[j].dist : INFINITY;
      out_row[i * k + j] = have ? sh.hits[j].id : UINT32_MAX;
    }
    const vdb::SegmentExplain& e = sh.explain;
    ex.push_back({{"id", e.segment_id}, {"strategy", e.strategy}, {"matches", e.matches},
                  {"live_rows", e.live_rows}, {"ef", e.ef}, {"distance_computations", e.distance_computations},
                  {"results", e.results}});
  }
  const std::string text = ex.dump();
  if (text.size() + 1 > cap) {
    g_err = "explain buffer too small";
    return 7;
  }
  std::memcpy(explain, text.c_str(), text.size() + 1);
  return 0;
}

}  // extern "C"
