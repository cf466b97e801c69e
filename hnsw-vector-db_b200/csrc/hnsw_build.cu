// Kernels of the GPU HNSW builder (hnsw_build.cc): the neighbour heuristic of
// HnswGraph::select_neighbors (src/index/hnsw/hnsw_graph.h:569-590) over exact nearest-neighbour
// candidates, the reverse adjacency, and the merge of forward and back links with the re-prune
// of HnswGraph::add_link (hnsw_graph.h:593-616). One warp per node; distances in fp32 (the
// graph's shape, not its bits, is what matters here).
#include "common.cuh"
#include "hnsw_build.cuh"
#include "warp_ops.cuh"

namespace vdbgpu {
namespace {

constexpr int kListCap = 256;  // candidates a merge considers per node

struct PruneSmem {
  float* cr;       // candidate row (pd)
  float* kr;       // kept rows, maxm x (pd + 1) (padded: lane j reads row j conflict-free)
  uint64_t* keys;  // kListCap sorted (dist, id) keys
  uint32_t* kept;  // maxm ids
  uint32_t* list;  // kListCap ids (merge)
};

__host__ __device__ inline size_t PruneWarpBytes(int pd, int maxm) {
  const size_t b = static_cast<size_t>(pd) * 4 + static_cast<size_t>(maxm) * (pd + 1) * 4 +
                   static_cast<size_t>(kListCap) * 8 + static_cast<size_t>(maxm) * 4 + kListCap * 4;
  return (b + 15) / 16 * 16;
}

__device__ __forceinline__ float pair_dist(const float* a, const float* b, int pd, bool l2) {
  float s = 0.f;
  if (l2) {
    for (int e = 0; e < pd; ++e) {
      const float d = a[e] - b[e];
      s = fmaf(d, d, s);
    }
    return s;
  }
  for (int e = 0; e < pd; ++e) s = fmaf(a[e], b[e], s);
  return -s;
}

// HnswGraph::select_neighbors: walk the sorted candidates and keep one only when it is closer to
// the base node than to every neighbour kept so far; fewer candidates than maxm are all kept.
__device__ int heuristic(const PruneArgs& a, PruneSmem& s, int nc, int maxm) {
  const int lane = threadIdx.x & 31;
  const bool l2 = a.metric == 0;
  if (nc < maxm) {
    for (int i = lane; i < nc; i += 32) s.kept[i] = neighbor_id(s.keys[i]);
    __syncwarp();
    return nc;
  }
  int kept = 0;
  for (int i = 0; i < nc && kept < maxm; ++i) {
    const uint64_t key = s.keys[i];
    const uint32_t c = neighbor_id(key);
    const float cd = neighbor_dist(key);
    const float* row = a.rows + static_cast<uint64_t>(c) * a.pd;
    for (int e = lane; e < a.pd; e += 32) s.cr[e] = row[e];
    __syncwarp();
    bool bad = false;
    if (lane < kept) bad = pair_dist(s.cr, s.kr + static_cast<size_t>(lane) * (a.pd + 1), a.pd, l2) < cd;
    if (!__any_sync(0xFFFFFFFFu, bad)) {
      float* dst = s.kr + static_cast<size_t>(kept) * (a.pd + 1);
      for (int e = lane; e < a.pd; e += 32) dst[e] = s.cr[e];
      if (lane == 0) s.kept[kept] = c;
      ++kept;
    }
    __syncwarp();
  }
  return kept;
}

__device__ PruneSmem carve(uint8_t* base, int pd, int maxm) {
  PruneSmem s;
  s.keys = reinterpret_cast<uint64_t*>(base);
  s.cr = reinterpret_cast<float*>(s.keys + kListCap);
  s.kr = s.cr + pd;
  s.kept = reinterpret_cast<uint32_t*>(s.kr + static_cast<size_t>(maxm) * (pd + 1));
  s.list = s.kept + maxm;
  return s;
}

// Forward links: the heuristic over each node's nearest candidates (sorted, self excluded).
__global__ void select_kernel(const PruneArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t local = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  const uint64_t nsel = a.n_select != 0 ? a.n_select : a.n;
  if (local >= nsel) return;
  const uint64_t node = a.node_base + local;  // the node's position in the layer
  PruneSmem s = carve(sm + static_cast<size_t>(warp) * PruneWarpBytes(a.pd, a.maxm), a.pd, a.maxm);
  // Candidates arrive sorted by (dist, id); keep order, drop self and misses.
  int nc = 0;
  for (int b = 0; b < a.kc; b += 32) {
    const int j = b + lane;
    uint32_t id = UINT32_MAX;
    float d = 0.f;
    if (j < a.kc) {
      id = a.cand_ids[local * a.kc + j];
      d = a.cand_d[local * a.kc + j];
    }
    const bool ok = id != UINT32_MAX && id != static_cast<uint32_t>(node) && id < a.n;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, ok);
    if (ok) s.keys[nc + __popc(m & ((1u << lane) - 1u))] = pack_neighbor(d, id);
    nc += __popc(m);
  }
  __syncwarp();
  const int kept = heuristic(a, s, nc, a.maxm);
  uint32_t* out = a.out + local * a.out_stride;
  for (int i = lane; i < kept; i += 32) out[1 + i] = s.kept[i];
  if (lane == 0) out[0] = static_cast<uint32_t>(kept);
}

__global__ void count_reverse_kernel(const uint32_t* fwd, int stride, uint64_t n, uint32_t* cnt) {
  const uint64_t u = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  if (u >= n) return;
  const uint32_t* l = fwd + u * stride;
  for (uint32_t j = 0; j < l[0]; ++j) atomicAdd(&cnt[l[1 + j]], 1u);
}

// Source u's back links name it as src_base + u (its position in the layer).
__global__ void fill_reverse_kernel(const uint32_t* fwd, int stride, uint64_t n, const uint64_t* off,
                                    uint32_t* cursor, uint32_t* rev, uint32_t src_base) {
  const uint64_t u = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  if (u >= n) return;
  const uint32_t* l = fwd + u * stride;
  for (uint32_t j = 0; j < l[0]; ++j) {
    const uint32_t v = l[1 + j];
    rev[off[v] + atomicAdd(&cursor[v], 1u)] = src_base + static_cast<uint32_t>(u);
  }
}

// Final lists: forward links plus back links (no duplicates); a list longer than maxm is sorted
// by distance to the node and re-pruned with the heuristic (add_link's rule).
__global__ void merge_kernel(const PruneArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t node = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (node >= a.n) return;
  PruneSmem s = carve(sm + static_cast<size_t>(warp) * PruneWarpBytes(a.pd, a.maxm), a.pd, a.maxm);
  const uint32_t* f = a.fwd + node * a.fwd_stride;
  const int nf = static_cast<int>(f[0]);
  for (int i = lane; i < nf; i += 32) s.list[i] = f[1 + i];
  __syncwarp();
  int nl = nf;
  const uint64_t r0 = a.rev_off[node], r1 = a.rev_off[node + 1];
  for (uint64_t b = r0; b < r1 && nl < kListCap; b += 32) {
    const uint64_t j = b + lane;
    uint32_t id = UINT32_MAX;
    if (j < r1) id = a.rev_ids[j];
    bool dup = id == UINT32_MAX;
    for (int i = 0; i < nf && !dup; ++i) dup = s.list[i] == id;
    const bool ok = !dup;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, ok);
    const int pos = nl + __popc(m & ((1u << lane) - 1u));
    if (ok && pos < kListCap) s.list[pos] = id;
    nl = min(kListCap, nl + __popc(m));
    __syncwarp();
  }
  uint32_t* out = a.out + node * a.out_stride;
  if (nl <= a.maxm) {
    for (int i = lane; i < nl; i += 32) out[1 + i] = s.list[i];
    if (lane == 0) out[0] = static_cast<uint32_t>(nl);
    return;
  }
  // Distances to the node, then sort (dist, id) and prune.
  const bool l2 = a.metric == 0;
  const float* nrow = a.rows + node * a.pd;
  for (int e = lane; e < a.pd; e += 32) s.cr[e] = nrow[e];
  __syncwarp();
  uint64_t x[kListCap / 32];
#pragma unroll
  for (int e = 0; e < kListCap / 32; ++e) {
    const int i = e * 32 + lane;
    x[e] = ~0ull;
    if (i < nl) {
      const uint32_t id = s.list[i];
      x[e] = pack_neighbor(pair_dist(s.cr, a.rows + static_cast<uint64_t>(id) * a.pd, a.pd, l2), id);
    }
  }
  __syncwarp();
  warp_sort<kListCap / 32>(x);
#pragma unroll
  for (int e = 0; e < kListCap / 32; ++e) s.keys[e * 32 + lane] = x[e];
  __syncwarp();
  const int kept = heuristic(a, s, nl, a.maxm);
  for (int i = lane; i < kept; i += 32) out[1 + i] = s.kept[i];
  if (lane == 0) out[0] = static_cast<uint32_t>(kept);
}

__global__ void gather_rows_kernel(const float* rows, const uint32_t* ids, uint64_t n, int pd, float* out) {
  const uint64_t i = blockIdx.x;
  if (i >= n) return;
  const float* src = rows + static_cast<uint64_t>(ids[i]) * pd;
  for (int e = threadIdx.x; e < pd; e += blockDim.x) out[i * pd + e] = src[e];
}

int WarpsFor(int pd, int maxm) {
  const size_t per = PruneWarpBytes(pd, maxm);
  int w = 4;
  while (w > 1 && static_cast<size_t>(w) * per > 200 * 1024) w /= 2;
  return w;
}

}  // namespace

size_t PruneSmemBytes(int pd, int maxm) { return PruneWarpBytes(pd, maxm); }

cudaError_t LaunchSelect(const PruneArgs& a, cudaStream_t st) {
  if (a.n == 0) return cudaSuccess;
  const int w = WarpsFor(a.pd, a.maxm);
  const size_t smem = static_cast<size_t>(w) * PruneWarpBytes(a.pd, a.maxm);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  NoteLaunch();
  const uint64_t nsel = a.n_select != 0 ? a.n_select : a.n;
  select_kernel<<<static_cast<unsigned>((nsel + w - 1) / w), w * 32, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchReverse(const uint32_t* fwd, int stride, uint64_t n, uint32_t* cnt, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  NoteLaunch();
  count_reverse_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(fwd, stride, n, cnt);
  return cudaGetLastError();
}

cudaError_t LaunchFillReverse(const uint32_t* fwd, int stride, uint64_t n, const uint64_t* off, uint32_t* cursor,
                              uint32_t* rev, cudaStream_t st, uint32_t src_base) {
  if (n == 0) return cudaSuccess;
  NoteLaunch();
  fill_reverse_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(fwd, stride, n, off, cursor, rev,
                                                                              src_base);
  return cudaGetLastError();
}

cudaError_t LaunchMergeLinks(const PruneArgs& a, cudaStream_t st) {
  if (a.n == 0) return cudaSuccess;
  const int w = WarpsFor(a.pd, a.maxm);
  const size_t smem = static_cast<size_t>(w) * PruneWarpBytes(a.pd, a.maxm);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  NoteLaunch();
  merge_kernel<<<static_cast<unsigned>((a.n + w - 1) / w), w * 32, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchGatherRows(const float* rows, const uint32_t* ids, uint64_t n, int pd, float* out, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  NoteLaunch();
  gather_rows_kernel<<<static_cast<unsigned>(n), 128, 0, st>>>(rows, ids, n, pd, out);
  return cudaGetLastError();
}

}  // namespace vdbgpu
