// An HNSW graph built on the GPU and written in the reference's index.hnsw format
// (HnswIndex::save, src/index/hnsw/hnsw_index.cc:36-41; HnswGraph::serialize,
// src/index/hnsw/hnsw_graph.h:387-401; WriteIndexFile, src/index/index.cc:38-44), so that the GPU
// path, the reference's LoadIndex and vdbgpu_collection_add_segment all read it.
//
// The reference inserts nodes one at a time (HnswGraph::insert, hnsw_graph.h:231-283): a greedy
// descent, an ef_construction beam per layer, select_neighbors down to M links and back links
// re-pruned to M0 (layer 0) / M. Sequential insertion does not map to a GPU, so this builder
// applies the same per-layer rules to all nodes at once:
//   levels     level_for's distribution (hnsw_graph.h:470-474): floor(-ln(1 - u) / ln M) with
//              u from SplitMix64 of (seed, id), capped at 15
//   candidates the layer's nodes in a seeded random insertion order; in doubling rounds each
//              node's exact nearest neighbours among the nodes up to its own round (the
//              tensor-core flat scan), standing in for the ef_construction beam over the nodes
//              inserted before it
//   forward    select_neighbors(candidates, M) (hnsw_graph.h:569-590)
//   back links every forward link u -> v also offered to v; a list above M0 / M is sorted by
//              distance and re-pruned with the same heuristic (add_link, hnsw_graph.h:593-616)
// The result is a valid graph of the same shape (degree bounds, heuristic links, layers), not
// the reference's graph: parity of search is tested on graphs both sides load from one file.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "formats.h"
#include "hnsw_build.cuh"
#include "runtime.h"

namespace vdbgpu {
namespace {

uint64_t SplitMix64(uint64_t x) {  // Steele, Lea & Flood (2014), the SplitMix64 finalizer
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

double UnitDouble(uint64_t x) { return static_cast<double>(x >> 11) * (1.0 / 9007199254740992.0); }

template <class T>
void Put(std::string* s, T v) {
  s->append(reinterpret_cast<const char*>(&v), sizeof(T));
}

// Links one layer. `nodes` lists the layer's nodes by row id: the first n_old are already linked
// (old_lists holds their lists, count + layer positions, stride 1 + maxc), the rest are inserted
// in the given order. Each inserted node takes its exact nearest neighbours among the old nodes and
// the inserted nodes up to its own doubling round as candidates, keeps select_neighbors(.., M) of
// them, and offers each kept link back; every list that grew past maxc is re-pruned with the
// heuristic. lists (out): every position's list, count + layer positions, stride 1 + maxc.
Status LinkLayer(Context& ctx, int metric, const float* dr, uint32_t dim, uint32_t pd,
                 const std::vector<uint32_t>& nodes, uint64_t n_old, const std::vector<uint32_t>* old_lists,
                 uint32_t M, uint32_t maxc, uint32_t kcand, std::vector<uint32_t>* lists) {
  cudaStream_t st = ctx.stream();
  const uint64_t m = nodes.size();
  const uint64_t n_new = m - n_old;
  lists->assign(m * (1 + maxc), 0);
  if (n_new == 0) {
    if (old_lists != nullptr) *lists = *old_lists;
    return Status::OK();
  }
  // The layer's rows in position order.
  DeviceBuffer lrows_buf, ids_dev;
  VDBGPU_RETURN_IF_ERROR(lrows_buf.alloc(m * pd * sizeof(float)));
  VDBGPU_RETURN_IF_ERROR(ids_dev.alloc(m * 4));
  VDBGPU_CUDA(cudaMemcpyAsync(ids_dev.get(), nodes.data(), m * 4, cudaMemcpyHostToDevice, st));
  VDBGPU_CUDA(LaunchGatherRows(dr, ids_dev.as<uint32_t>(), m, static_cast<int>(pd), lrows_buf.as<float>(), st));
  const float* lrows = lrows_buf.as<float>();
  // Candidates: in doubling rounds, the inserted positions [a, b) take their exact nearest
  // neighbours among positions [0, b) -- the old nodes, the nodes inserted before them and beside
  // them -- so early nodes get the long links sequential insertion gives them (self included in
  // the search, dropped by the select step).
  const uint32_t kq = static_cast<uint32_t>(std::min<uint64_t>(kcand + 1, m));
  DeviceBuffer cid, cd;
  VDBGPU_RETURN_IF_ERROR(cid.alloc(n_new * kq * 4));
  VDBGPU_RETURN_IF_ERROR(cd.alloc(n_new * kq * 4));
  const uint64_t first = n_old + std::max<uint64_t>(256, kq);
  for (uint64_t a = n_old, b = std::min<uint64_t>(m, first); a < m; a = b, b = std::min<uint64_t>(m, 2 * b)) {
    std::unique_ptr<GpuIndex> flat;
    VDBGPU_RETURN_IF_ERROR(CreateFlatIndex(ctx, metric == 2 ? 1 : metric, lrows, b, dim, pd, &flat));
    const uint64_t chunk = 65536;
    for (uint64_t q0 = a; q0 < b; q0 += chunk) {
      SearchBatch sb{};
      sb.queries = lrows + q0 * pd;
      sb.nq = std::min(chunk, b - q0);
      sb.k = kq;
      sb.allow = nullptr;
      sb.out_dist = cd.as<float>() + (q0 - n_old) * kq;
      sb.out_row = cid.as<uint32_t>() + (q0 - n_old) * kq;
      sb.dist_comps = nullptr;
      VDBGPU_RETURN_IF_ERROR(flat->Search(ctx, sb));
    }
    VDBGPU_RETURN_IF_ERROR(ctx.Sync("hnsw build: neighbours"));
  }
  // Forward links of the inserted nodes: select_neighbors(candidates, M).
  DeviceBuffer fwd_new, fwd, cnt, off, cursor, rev, out;
  VDBGPU_RETURN_IF_ERROR(fwd_new.alloc(n_new * (1 + M) * 4));
  PruneArgs pa{};
  pa.rows = lrows;
  pa.pd = static_cast<int>(pd);
  pa.metric = metric == 0 ? 0 : 1;
  pa.n = m;
  pa.node_base = n_old;
  pa.n_select = n_new;
  pa.cand_ids = cid.as<uint32_t>();
  pa.cand_d = cd.as<float>();
  pa.kc = static_cast<int>(kq);
  pa.maxm = static_cast<int>(M);
  pa.out = fwd_new.as<uint32_t>();
  pa.out_stride = static_cast<int>(1 + M);
  VDBGPU_CUDA(LaunchSelect(pa, st));
  // Reverse adjacency of the new forward links only (old lists were settled when they were made).
  VDBGPU_RETURN_IF_ERROR(cnt.alloc(m * 4));
  VDBGPU_CUDA(cudaMemsetAsync(cnt.get(), 0, m * 4, st));
  VDBGPU_CUDA(LaunchReverse(fwd_new.as<uint32_t>(), static_cast<int>(1 + M), n_new, cnt.as<uint32_t>(), st));
  std::vector<uint32_t> hc(m);
  VDBGPU_CUDA(cudaMemcpyAsync(hc.data(), cnt.get(), m * 4, cudaMemcpyDeviceToHost, st));
  VDBGPU_RETURN_IF_ERROR(ctx.Sync("hnsw build: reverse counts"));
  std::vector<uint64_t> ho(m + 1, 0);
  for (uint64_t i = 0; i < m; ++i) ho[i + 1] = ho[i] + hc[i];
  VDBGPU_RETURN_IF_ERROR(off.alloc((m + 1) * 8));
  VDBGPU_RETURN_IF_ERROR(cursor.alloc(m * 4));
  VDBGPU_RETURN_IF_ERROR(rev.alloc(std::max<uint64_t>(1, ho[m]) * 4));
  VDBGPU_CUDA(cudaMemcpyAsync(off.get(), ho.data(), (m + 1) * 8, cudaMemcpyHostToDevice, st));
  VDBGPU_CUDA(cudaMemsetAsync(cursor.get(), 0, m * 4, st));
  VDBGPU_CUDA(LaunchFillReverse(fwd_new.as<uint32_t>(), static_cast<int>(1 + M), n_new, off.as<uint64_t>(),
                                cursor.as<uint32_t>(), rev.as<uint32_t>(), st, static_cast<uint32_t>(n_old)));
  // Every position's own list (an old node's current list, an inserted node's forward links),
  // plus its back links, re-pruned to maxc.
  const uint32_t* own = fwd_new.as<uint32_t>();
  int own_stride = static_cast<int>(1 + M);
  if (n_old > 0) {
    VDBGPU_RETURN_IF_ERROR(fwd.alloc(m * (1 + maxc) * 4));
    VDBGPU_CUDA(cudaMemcpyAsync(fwd.get(), old_lists->data(), n_old * (1 + maxc) * 4, cudaMemcpyHostToDevice, st));
    VDBGPU_CUDA(cudaMemsetAsync(fwd.as<uint32_t>() + n_old * (1 + maxc), 0, n_new * (1 + maxc) * 4, st));
    VDBGPU_CUDA(cudaMemcpy2DAsync(fwd.as<uint32_t>() + n_old * (1 + maxc), (1 + maxc) * 4, fwd_new.get(),
                                  (1 + M) * 4, (1 + M) * 4, n_new, cudaMemcpyDeviceToDevice, st));
    own = fwd.as<uint32_t>();
    own_stride = static_cast<int>(1 + maxc);
  }
  VDBGPU_RETURN_IF_ERROR(out.alloc(m * (1 + maxc) * 4));
  pa.node_base = 0;
  pa.n_select = 0;
  pa.fwd = own;
  pa.fwd_stride = own_stride;
  pa.rev_off = off.as<uint64_t>();
  pa.rev_ids = rev.as<uint32_t>();
  pa.maxm = static_cast<int>(maxc);
  pa.out = out.as<uint32_t>();
  pa.out_stride = static_cast<int>(1 + maxc);
  VDBGPU_CUDA(LaunchMergeLinks(pa, st));
  VDBGPU_CUDA(cudaMemcpyAsync(lists->data(), out.get(), lists->size() * 4, cudaMemcpyDeviceToHost, st));
  return ctx.Sync("hnsw build: links");
}

// Node levels from level_for's law (hnsw_graph.h:470-474).
int LevelFor(uint64_t seed, double mult, uint64_t i) {
  const double u = UnitDouble(SplitMix64(seed ^ (i * 0x9E3779B97F4A7C15ull)));
  return std::min(static_cast<int>(-std::log(1.0 - u) * mult), 15);
}

// HnswIndex::save + HnswGraph::serialize + WriteIndexFile for a graph of n nodes.
std::string SerializeHnsw(uint32_t pd, uint64_t n, uint32_t M, uint32_t efc, uint64_t seed, int max_level,
                          uint32_t entry, const std::vector<uint8_t>& level, const std::vector<uint32_t>& links0,
                          const std::vector<std::vector<uint32_t>>& upper) {
  std::string out = "VDBHNSW1";
  Put<uint32_t>(&out, pd);
  Put<uint64_t>(&out, n);
  Put<uint64_t>(&out, n);
  Put<uint32_t>(&out, M);
  Put<uint32_t>(&out, efc);
  Put<uint64_t>(&out, seed);
  Put<uint32_t>(&out, static_cast<uint32_t>(max_level));
  Put<uint32_t>(&out, entry);
  out.append(reinterpret_cast<const char*>(level.data()), level.size());
  out.append(reinterpret_cast<const char*>(links0.data()), links0.size() * 4);
  for (uint64_t i = 0; i < n; ++i)
    if (!upper[i].empty()) out.append(reinterpret_cast<const char*>(upper[i].data()), upper[i].size() * 4);
  Put<uint32_t>(&out, Crc32c(out.data(), out.size()));
  return out;
}

// Rows on the device (a copy when they are host memory).
Status DeviceRows(Context& ctx, const float* rows, uint64_t n, uint32_t pd, DeviceBuffer* buf, const float** dr) {
  *dr = rows;
  if (n == 0 || WherePointer(rows, ctx.device()) == MemWhere::kDevice) return Status::OK();
  VDBGPU_RETURN_IF_ERROR(buf->alloc(n * pd * sizeof(float)));
  VDBGPU_CUDA(cudaMemcpyAsync(buf->get(), rows, n * pd * sizeof(float), cudaMemcpyDefault, ctx.stream()));
  *dr = buf->as<float>();
  return Status::OK();
}

// A seeded insertion order (Fisher-Yates over SplitMix64) of nodes[from, end) for layer l.
void ShuffleTail(std::vector<uint32_t>* nodes, size_t from, uint64_t seed, int l) {
  const uint64_t cnt = nodes->size() - from;
  if (cnt <= 1) return;
  uint64_t rs = SplitMix64(seed + 0x51ED27ull * static_cast<uint64_t>(l + 1));
  for (uint64_t i = cnt - 1; i > 0; --i) {
    rs = SplitMix64(rs);
    std::swap((*nodes)[from + i], (*nodes)[from + rs % (i + 1)]);
  }
}

}  // namespace

Status BuildHnswFile(Context& ctx, int metric, const float* rows, uint64_t n, uint32_t dim, uint32_t pd, uint32_t M,
                     uint32_t kcand, uint64_t seed, std::string* file) {
  if (M < 2 || M > 16) return Status(Status::kInvalidArgument, "M must be in 2..16 for the GPU builder");
  if (n >= (uint64_t{1} << 32) - 1) return Status(Status::kInvalidArgument, "too many rows");
  const uint32_t M0 = 2 * M;
  if (kcand == 0) kcand = std::min<uint32_t>(2 * M0, 127);
  kcand = std::max<uint32_t>(std::min<uint32_t>(kcand, 127), M0);
  // ---- levels (hnsw_graph.h:470-474) and the entry point (first node on the top layer)
  std::vector<uint8_t> level(n, 0);
  const double mult = 1.0 / std::log(static_cast<double>(M));
  int max_level = -1;
  uint32_t entry = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const int l = LevelFor(seed, mult, i);
    level[i] = static_cast<uint8_t>(l);
    if (l > max_level) {
      max_level = l;
      entry = static_cast<uint32_t>(i);
    }
  }
  DeviceBuffer drows;
  const float* dr = nullptr;
  VDBGPU_RETURN_IF_ERROR(DeviceRows(ctx, rows, n, pd, &drows, &dr));
  std::vector<uint32_t> links0(n * (1 + M0), 0);
  std::vector<std::vector<uint32_t>> upper(n);
  for (uint64_t i = 0; i < n; ++i)
    if (level[i] > 0) upper[i].assign(static_cast<size_t>(level[i]) * (1 + M), 0);
  for (int l = 0; l <= max_level; ++l) {
    std::vector<uint32_t> nodes;
    for (uint64_t i = 0; i < n; ++i)
      if (level[i] >= l) nodes.push_back(static_cast<uint32_t>(i));
    const uint64_t m = nodes.size();
    if (m <= 1) continue;
    const uint32_t maxc = l == 0 ? M0 : M;
    ShuffleTail(&nodes, 0, seed, l);
    std::vector<uint32_t> lists;
    VDBGPU_RETURN_IF_ERROR(LinkLayer(ctx, metric, dr, dim, pd, nodes, 0, nullptr, M, maxc, kcand, &lists));
    // Layer positions back to row ids.
    for (uint64_t i = 0; i < m; ++i) {
      const uint32_t* src = lists.data() + i * (1 + maxc);
      const uint32_t c = std::min(src[0], maxc);
      uint32_t* dst = l == 0 ? links0.data() + static_cast<uint64_t>(nodes[i]) * (1 + M0)
                             : upper[nodes[i]].data() + static_cast<size_t>(l - 1) * (1 + M);
      dst[0] = c;
      for (uint32_t j = 0; j < c; ++j) dst[1 + j] = nodes[src[1 + j]];
    }
  }
  *file = SerializeHnsw(pd, n, M, kcand, seed, max_level, entry, level, links0, upper);
  return Status::OK();
}

Status ExtendHnswFile(Context& ctx, int metric, const HnswGraphData& g, uint32_t pd, const float* rows, uint64_t n,
                      uint32_t dim, std::string* file) {
  const uint64_t n0 = g.cap;
  if (n < n0) return Status(Status::kInvalidArgument, "extend needs a superset of the indexed rows");
  if (n >= (uint64_t{1} << 32) - 1) return Status(Status::kInvalidArgument, "too many rows");
  if (g.M < 2 || g.M > 16 || g.M0 != 2 * g.M)
    return Status(Status::kNotSupported, "the GPU extends graphs with M in 2..16 (M0 = 2M)");
  const uint32_t M = g.M, M0 = g.M0;
  const uint32_t kcand = std::max<uint32_t>(std::min<uint32_t>(g.efc == 0 ? 2 * M0 : g.efc, 127), M0);
  // Levels: the old nodes keep theirs; new ones follow level_for with the graph's seed, and the
  // first node above the top layer becomes the entry point (HnswGraph::insert).
  std::vector<uint8_t> level(g.level.begin(), g.level.end());
  level.resize(n, 0);
  const double mult = 1.0 / std::log(static_cast<double>(M));
  int max_level = g.max_level;
  uint32_t entry = g.entry;
  for (uint64_t i = n0; i < n; ++i) {
    const int l = LevelFor(g.seed, mult, i);
    level[i] = static_cast<uint8_t>(l);
    if (l > max_level) {
      max_level = l;
      entry = static_cast<uint32_t>(i);
    }
  }
  DeviceBuffer drows;
  const float* dr = nullptr;
  VDBGPU_RETURN_IF_ERROR(DeviceRows(ctx, rows, n, pd, &drows, &dr));
  std::vector<uint32_t> links0(n * (1 + M0), 0);
  std::copy(g.links0.begin(), g.links0.begin() + n0 * (1 + M0), links0.begin());
  std::vector<std::vector<uint32_t>> upper(n);
  for (uint64_t i = 0; i < n; ++i) {
    if (level[i] == 0) continue;
    upper[i].assign(static_cast<size_t>(level[i]) * (1 + M), 0);
    if (i < n0)
      std::copy(g.upper.begin() + g.upper_off[i], g.upper.begin() + g.upper_off[i] + upper[i].size(),
                upper[i].begin());
  }
  std::vector<uint32_t> pos(n, 0);
  for (int l = 0; l <= max_level; ++l) {
    // Old nodes first (already linked), then the new ones in a seeded insertion order.
    std::vector<uint32_t> nodes;
    for (uint64_t i = 0; i < n0; ++i)
      if (level[i] >= l) nodes.push_back(static_cast<uint32_t>(i));
    const uint64_t n_old = nodes.size();
    for (uint64_t i = n0; i < n; ++i)
      if (level[i] >= l) nodes.push_back(static_cast<uint32_t>(i));
    const uint64_t m = nodes.size();
    if (m == n_old || m <= 1) continue;
    ShuffleTail(&nodes, n_old, g.seed, l);
    const uint32_t maxc = l == 0 ? M0 : M;
    for (uint64_t p = 0; p < m; ++p) pos[nodes[p]] = static_cast<uint32_t>(p);
    auto list_of = [&](uint32_t id) {
      return l == 0 ? links0.data() + static_cast<uint64_t>(id) * (1 + M0)
                    : upper[id].data() + static_cast<size_t>(l - 1) * (1 + M);
    };
    // The old nodes' current lists in layer positions.
    std::vector<uint32_t> old_lists(n_old * (1 + maxc), 0);
    for (uint64_t p = 0; p < n_old; ++p) {
      const uint32_t* src = list_of(nodes[p]);
      const uint32_t c = std::min(src[0], maxc);
      old_lists[p * (1 + maxc)] = c;
      for (uint32_t j = 0; j < c; ++j) old_lists[p * (1 + maxc) + 1 + j] = pos[src[1 + j]];
    }
    std::vector<uint32_t> lists;
    VDBGPU_RETURN_IF_ERROR(LinkLayer(ctx, metric, dr, dim, pd, nodes, n_old, &old_lists, M, maxc, kcand, &lists));
    for (uint64_t p = 0; p < m; ++p) {
      const uint32_t* src = lists.data() + p * (1 + maxc);
      const uint32_t c = std::min(src[0], maxc);
      uint32_t* dst = list_of(nodes[p]);
      dst[0] = c;
      for (uint32_t j = 0; j < c; ++j) dst[1 + j] = nodes[src[1 + j]];
    }
  }
  *file = SerializeHnsw(pd, n, M, g.efc, g.seed, max_level, entry, level, links0, upper);
  return Status::OK();
}

}  // namespace vdbgpu
