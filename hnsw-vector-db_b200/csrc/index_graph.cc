// GPU indexes loaded from the reference's graph and list index files:
//   HnswIndex     (src/index/hnsw/hnsw_index.h:12-41, file body hnsw_index.cc:36-48)
//   HnswSq8Index  (hnsw_index.h:63-96, file body hnsw_index.cc:104-129)
//   PqFlatIndex / IvfPqIndex (src/index/quant/ivf_pq.h) in index_ivfpq.cc
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "formats.h"
#include "hnsw.cuh"
#include "runtime.h"

namespace vdbgpu {

Status LoadIvfPqIndex(Context& ctx, int type, std::string_view body, int metric, const float* rows,
                      uint64_t n, uint32_t dim, uint32_t pd, std::unique_ptr<GpuIndex>* out);

namespace {

template <class T>
Status Upload(Context& ctx, const std::vector<T>& v, DeviceBuffer* out) {
  VDBGPU_RETURN_IF_ERROR(out->alloc(std::max<size_t>(1, v.size()) * sizeof(T)));
  if (!v.empty())
    VDBGPU_CUDA(cudaMemcpyAsync(out->get(), v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice,
                                ctx.stream()));
  return Status::OK();
}

int Log2Ceil(uint64_t x) {
  int b = 0;
  while ((uint64_t{1} << b) < x) ++b;
  return b;
}

class HnswGpuIndex final : public GpuIndex {
 public:
  explicit HnswGpuIndex(bool sq8) : sq8_(sq8) {}
  int type() const override { return sq8_ ? kIndexHnswSq8 : kIndexHnsw; }
  uint64_t rows() const override { return n_; }
  const float* device_rows() const override { return rows_.as<float>(); }
  uint64_t device_bytes() const override {
    return rows_.size() + codes_.size() + links0_.size() + upper_.size() + upper_off_.size() +
           level_.size() + vmin_.size() + scale_.size();
  }

  Status Load(Context& ctx, std::string_view body, const float* rows, uint64_t n) {
    n_ = n;
    Reader r(body);
    if (!sq8_) {
      uint32_t fpd = 0;
      if (!r.u32(&fpd) || fpd != pd) return Status(Status::kCorruption, "hnsw dim mismatch");
    } else {
      uint64_t fn = 0;
      if (!r.u64(&fn) || fn != n) return Status(Status::kCorruption, "hnsw-sq8 index does not match the segment");
      Sq8Data q;
      // HnswSq8Index::load (hnsw_index.cc:117-122) reports any quantizer fault as a mismatch.
      if (!ParseSq8(r, &q).ok() || q.pd != pd)
        return Status(Status::kCorruption, "hnsw-sq8 index does not match the segment");
      std::string_view codes;
      if (!r.bytes(n * pd, &codes)) return Status(Status::kCorruption, "truncated sq8 codes");
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, q.vmin, &vmin_));
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, q.scale, &scale_));
      VDBGPU_RETURN_IF_ERROR(codes_.alloc(std::max<uint64_t>(1, n * pd)));
      if (n > 0)
        VDBGPU_CUDA(cudaMemcpyAsync(codes_.get(), codes.data(), n * pd, cudaMemcpyHostToDevice, ctx.stream()));
    }
    VDBGPU_RETURN_IF_ERROR(ParseHnswGraph(r, n, &g_));
    // The walk gives every link of a list its own lane: at most 32 links on layer 0 (M0 = 2M).
    if (g_.M > 16)
      return Status(Status::kNotSupported, "HNSW graphs with M above 16 are not supported on the GPU");
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, g_.links0, &links0_));
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, g_.upper, &upper_));
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, g_.upper_off, &upper_off_));
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, g_.level, &level_));
    VDBGPU_RETURN_IF_ERROR(rows_.alloc(std::max<uint64_t>(1, n * pd) * sizeof(float)));
    if (n > 0)
      VDBGPU_CUDA(cudaMemcpyAsync(rows_.get(), rows, n * pd * sizeof(float), cudaMemcpyDefault, ctx.stream()));
    // The graph arrays on the host are no longer needed.
    g_.links0 = {};
    g_.upper = {};
    g_.upper_off = {};
    g_.level = {};
    return ctx.Sync("hnsw index load");
  }

  // HnswIndex::search (hnsw_index.cc:22-34) / HnswSq8Index::search (hnsw_index.cc:82-102).
  Status Search(Context& ctx, const SearchBatch& b) override {
    const uint64_t k = b.k;
    const uint64_t pef = b.params.ef;
    uint64_t depth = 0, kg = k, ef = std::max(pef, k);
    if (sq8_) {
      depth = b.params.rerank < 0 ? std::max(pef, k) : static_cast<uint64_t>(b.params.rerank);
      ef = std::max({pef, k, depth});
      kg = depth == 0 ? k : std::max(depth, k);
      ef = std::max(ef, kg);
    }
    if (ef > 4096) return Status(Status::kNotSupported, "ef above 4096 is not supported on the GPU");
    HnswArgs a{};
    a.nq = static_cast<int>(b.nq);
    a.pd = static_cast<int>(pd);
    a.k = static_cast<int>(k);
    a.k_graph = static_cast<int>(kg);
    a.ef = static_cast<int>(ef);
    a.depth = static_cast<int>(depth);
    a.metric = metric;
    a.order = ctx.order();
    a.queries = b.queries;
    a.rows = rows_.as<float>();
    a.codes = sq8_ ? codes_.as<uint8_t>() : nullptr;
    a.vmin = sq8_ ? vmin_.as<float>() : nullptr;
    a.scale = sq8_ ? scale_.as<float>() : nullptr;
    a.links0 = links0_.as<uint32_t>();
    a.M0 = g_.M0;
    a.upper = upper_.as<uint32_t>();
    a.upper_off = upper_off_.as<uint64_t>();
    a.level = level_.as<uint8_t>();
    a.M = g_.M;
    a.max_level = g_.size > 0 ? g_.max_level : -1;
    a.entry = g_.entry;
    a.n = n_;
    a.allow = b.allow;
    a.step_limit = 1 << 22;
    a.out_dist = b.out_dist;
    a.out_row = b.out_row;
    a.out_dc = b.dist_comps;
    a.status = ctx.status_word();
    // Work counters of the walk while timing is on (HnswArgs::counters).
    a.counters = ctx.timing() ? ctx.counters() : nullptr;
    if (a.counters != nullptr)
      VDBGPU_CUDA(cudaMemsetAsync(a.counters, 0, 8 * sizeof(unsigned long long), ctx.stream()));
    // Unfiltered walks keep their state in shared memory: a visited hash and a candidate array
    // sized for the walk; one that overflows reruns the batch with that structure doubled (and
    // fewer queries per block once four no longer fit). Filtered walks keep every reached node
    // as a candidate until they hold ef allowed rows (the reference's unbounded heap), so they
    // run pooled: visited bits and candidates beyond a sorted front in global memory, the pool
    // growing fourfold on overflow.
    // Walks run pooled by default (measured faster at every ef: the sorted shared-memory arrays
    // cost O(ef) per insert). VDB_HNSW_POOLED_EF=<n> keeps unfiltered walks with ef <= n in shared
    // memory (read on every call).
    const char* pe = std::getenv("VDB_HNSW_POOLED_EF");
    const uint64_t pooled_ef = pe != nullptr ? std::strtoull(pe, nullptr, 10) : 0ull;
    const bool pooled = b.allow != nullptr || ef > pooled_ef;
    int bits = std::max(11, Log2Ceil(32 * ef));
    int cap = static_cast<int>(2 * ef + 64);
    int pool_cap = static_cast<int>(std::max<uint64_t>(4096, 32 * ef));
    for (;;) {
      a.pooled = pooled ? 1 : 0;
      a.hash_bits = pooled ? 1 : bits;  // pooled walks mark visits in global memory
      a.cand_cap = pooled ? kPoolFrontSlots : cap;
      a.warps = 0;
      for (int w = 4; w >= 1; w /= 2)
        if (static_cast<size_t>(w) * HnswWarpSmemBytes(a.pd, a.hash_bits, a.ef, a.cand_cap) <= 227 * 1024) {
          a.warps = w;
          break;
        }
      if (a.warps == 0)
        return Status(Status::kNotSupported,
                      "the graph walk's state exceeds the GPU's shared memory; use a smaller ef");
      ctx.Mark(0);
      ctx.Mark(1);
      if (pooled) {
        // Queries per launch: their visited bitmaps and candidate pools within ~8 GiB.
        a.vwords = (n_ + 31) / 32;
        const uint64_t per = a.vwords * 4 + static_cast<uint64_t>(pool_cap) * 8;
        const uint64_t chunk = std::max<uint64_t>(1, std::min<uint64_t>(b.nq, (8ull << 30) / per));
        VDBGPU_RETURN_IF_ERROR(visited_.ensure(chunk * a.vwords * 4));
        VDBGPU_RETURN_IF_ERROR(pool_.ensure(chunk * static_cast<uint64_t>(pool_cap) * 8));
        a.visited = visited_.as<uint32_t>();
        a.pool = pool_.as<uint64_t>();
        a.pool_cap = pool_cap;
        for (uint64_t q0 = 0; q0 < b.nq; q0 += chunk) {
          const uint64_t nqc = std::min(chunk, b.nq - q0);
          VDBGPU_CUDA(cudaMemsetAsync(visited_.get(), 0, nqc * a.vwords * 4, ctx.stream()));
          HnswArgs ac = a;
          ac.nq = static_cast<int>(nqc);
          ac.queries = b.queries + q0 * pd;
          ac.out_dist = b.out_dist + q0 * k;
          ac.out_row = b.out_row + q0 * k;
          ac.out_dc = b.dist_comps != nullptr ? b.dist_comps + q0 : nullptr;
          VDBGPU_CUDA(LaunchHnswSearch(ac, ctx.stream()));
        }
      } else {
        VDBGPU_CUDA(LaunchHnswSearch(a, ctx.stream()));
      }
      ctx.Mark(2);
      ctx.Mark(3);
      Status s = ctx.Sync("hnsw search");
      if (s.ok()) return s;
      const bool hash_full = s.message().find("code 6") != std::string::npos;
      const bool cand_full = s.message().find("code 9") != std::string::npos;
      if (pooled && cand_full && pool_cap < (1 << 24)) {
        pool_cap *= 4;
      } else if (!pooled && hash_full && bits < 16) {
        ++bits;
      } else if (!pooled && cand_full && cap < (1 << 16)) {
        cap *= 2;
      } else {
        return s;
      }
    }
  }

  bool sq8() const { return sq8_; }
  uint32_t graph_m() const { return g_.M; }
  // The device arrays a multi-segment walk reads.
  void Describe(HnswSegment* d) const {
    d->rows = rows_.as<float>();
    d->codes = sq8_ ? codes_.as<uint8_t>() : nullptr;
    d->vmin = sq8_ ? vmin_.as<float>() : nullptr;
    d->scale = sq8_ ? scale_.as<float>() : nullptr;
    d->links0 = links0_.as<uint32_t>();
    d->upper = upper_.as<uint32_t>();
    d->upper_off = upper_off_.as<uint64_t>();
    d->level = level_.as<uint8_t>();
    d->n = n_;
    d->entry = g_.entry;
    d->max_level = g_.size > 0 ? g_.max_level : -1;
  }

 private:
  bool sq8_;
  uint64_t n_ = 0;
  HnswGraphData g_;
  DeviceBuffer rows_, codes_, vmin_, scale_, links0_, upper_, upper_off_, level_;
  DeviceBuffer visited_, pool_;  // pooled walks' scratch (grow-only)
};

}  // namespace

Status HnswSearchMulti(Context& ctx, const std::vector<const GpuIndex*>& indexes, const HnswItem* items,
                       size_t nitems, const float* queries, uint32_t k, const SearchParams& p, uint64_t* out_keys,
                       uint64_t* out_dc, int* out_short, MultiScratch* sc) {
  if (nitems == 0) return Status::OK();
  std::vector<HnswSegment> segs(indexes.size());
  const HnswGpuIndex* first = nullptr;
  uint64_t max_n = 1;
  for (size_t i = 0; i < indexes.size(); ++i) {
    const auto* h = dynamic_cast<const HnswGpuIndex*>(indexes[i]);
    if (h == nullptr) return Status(Status::kNotSupported, "not an HNSW index");
    if (first == nullptr) first = h;
    if (h->sq8() != first->sq8() || h->graph_m() != first->graph_m() || h->pd != first->pd || h->metric != first->metric)
      return Status(Status::kNotSupported, "segments with different graph parameters");
    h->Describe(&segs[i]);
    max_n = std::max<uint64_t>(max_n, segs[i].n);
  }
  // Search parameters exactly as HnswGpuIndex::Search derives them.
  const uint64_t pef = p.ef;
  uint64_t depth = 0, kg = k, ef = std::max<uint64_t>(pef, k);
  if (first->sq8()) {
    depth = p.rerank < 0 ? std::max<uint64_t>(pef, k) : static_cast<uint64_t>(p.rerank);
    ef = std::max({pef, static_cast<uint64_t>(k), depth});
    kg = depth == 0 ? k : std::max<uint64_t>(depth, k);
    ef = std::max(ef, kg);
  }
  if (ef > 4096) return Status(Status::kNotSupported, "ef above 4096 is not supported on the GPU");
  VDBGPU_RETURN_IF_ERROR(sc->segs.ensure(segs.size() * sizeof(HnswSegment)));
  VDBGPU_CUDA(cudaMemcpyAsync(sc->segs.get(), segs.data(), segs.size() * sizeof(HnswSegment), cudaMemcpyHostToDevice,
                              ctx.stream()));
  HnswArgs a{};
  a.pd = static_cast<int>(first->pd);
  a.k = static_cast<int>(k);
  a.k_graph = static_cast<int>(kg);
  a.ef = static_cast<int>(ef);
  a.depth = static_cast<int>(depth);
  a.metric = first->metric;
  a.order = ctx.order();
  a.queries = queries;
  a.M0 = 2 * first->graph_m();
  a.M = first->graph_m();
  a.step_limit = 1 << 22;
  a.status = ctx.status_word();
  a.pooled = 1;
  a.hash_bits = 1;
  a.cand_cap = kPoolFrontSlots;
  a.vwords = (max_n + 31) / 32;
  a.segs = sc->segs.as<HnswSegment>();
  a.out_keys = out_keys;
  a.out_dc = out_dc;
  a.out_short = out_short;
  a.codes = first->sq8() ? segs[0].codes : nullptr;  // selects the SQ8 kernel
  a.counters = ctx.timing() ? ctx.counters() : nullptr;
  if (a.counters != nullptr)
    VDBGPU_CUDA(cudaMemsetAsync(a.counters, 0, 8 * sizeof(unsigned long long), ctx.stream()));
  a.warps = 4;
  // Walks per launch: their visited bitmaps and candidate pools within the scratch budget below.
  // Filtered walks at a few percent selectivity reach ~10^4 candidates: size the pools for that so
  // a launch rarely reruns.
  int pool_cap = static_cast<int>(std::max<uint64_t>(32768, 64 * ef));
  // Scratch for the walks of one launch: half the free device memory, between 16 and 64 GiB. The
  // fewer launches, the fewer launch tails (each launch waits for its longest walk).
  size_t free_b = 0, total_b = 0;
  VDBGPU_CUDA(cudaMemGetInfo(&free_b, &total_b));
  const uint64_t budget = std::clamp<uint64_t>(free_b / 2 + sc->visited.size() + sc->pool.size(), 16ull << 30,
                                               64ull << 30);
  size_t done = 0;
  while (done < nitems) {
    const uint64_t per = a.vwords * 4 + static_cast<uint64_t>(pool_cap) * 8;
    const size_t chunk = static_cast<size_t>(std::max<uint64_t>(1, std::min<uint64_t>(nitems - done, budget / per)));
    VDBGPU_RETURN_IF_ERROR(sc->items.ensure(chunk * sizeof(HnswItem)));
    VDBGPU_RETURN_IF_ERROR(sc->visited.ensure(chunk * a.vwords * 4));
    VDBGPU_RETURN_IF_ERROR(sc->pool.ensure(chunk * static_cast<uint64_t>(pool_cap) * 8));
    VDBGPU_CUDA(cudaMemcpyAsync(sc->items.get(), items + done, chunk * sizeof(HnswItem), cudaMemcpyHostToDevice,
                                ctx.stream()));
    VDBGPU_CUDA(cudaMemsetAsync(sc->visited.get(), 0, chunk * a.vwords * 4, ctx.stream()));
    a.nq = static_cast<int>(chunk);
    a.items = sc->items.as<HnswItem>();
    a.visited = sc->visited.as<uint32_t>();
    a.pool = sc->pool.as<uint64_t>();
    a.pool_cap = pool_cap;
    VDBGPU_CUDA(LaunchHnswSearch(a, ctx.stream()));
    Status s = ctx.Sync("hnsw multi-segment search");
    if (!s.ok()) {
      if (s.message().find("code 9") != std::string::npos && pool_cap < (1 << 22)) {
        pool_cap *= 4;  // a walk's candidate pool overflowed: rerun this chunk with larger pools
        continue;
      }
      return s;
    }
    done += chunk;
  }
  return Status::OK();
}

Status LoadGraphOrListIndex(Context& ctx, int type, std::string_view body, int metric,
                            const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                            std::unique_ptr<GpuIndex>* out) {
  if (type == kIndexHnsw || type == kIndexHnswSq8) {
    auto idx = std::make_unique<HnswGpuIndex>(type == kIndexHnswSq8);
    idx->metric = metric;
    idx->dim = dim;
    idx->pd = pd;
    VDBGPU_RETURN_IF_ERROR(idx->Load(ctx, body, rows, n));
    *out = std::move(idx);
    return Status::OK();
  }
  return LoadIvfPqIndex(ctx, type, body, metric, rows, n, dim, pd, out);
}

}  // namespace vdbgpu
