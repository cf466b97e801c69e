// Selection, exact re-rank and operand preparation kernels for flat and SQ8 search.
//
//   finalize_kernel  one warp per query: merges the candidate buffers that the tensor-core scan
//                    left for that query (every row slice), keeps the C best by (pre-rank key,
//                    row), recomputes their distances exactly in fp32 in the reference kernel
//                    set's summation order, and writes the k best by (dist, id). For SQ8 the
//                    exact SQ8 distances pick the re-rank depth first, then the fp32 rows decide
//                    (Rerank, src/index/index.cc:89-95; TopK order, src/util/topk.h:13-54).
//   prep_queries     fp32 queries -> fp16/bf16 tensor-core operand with a per-query power-of-two
//                    scale, plus the per-query key multiplier.
//   rows/codes prep  fp32 rows -> fp16/bf16 operand (+ squared norms); SQ8 codes -> fp16.
//   sq8 train/encode Sq8Quantizer::train / encode (src/index/quant/sq8.cc:9-37), bit-exact.
#include <cuda_runtime.h>

#include "common.cuh"
#include "ivfpq.cuh"
#include "kernels.cuh"
#include "scan_mma.cuh"
#include "warp_ops.cuh"

namespace vdbgpu {
namespace {

constexpr int kFinWarps = 4;
constexpr int kMaxSurvivors = 1024;
constexpr uint64_t kNoNeighbor = ~0ull;  // packs (+NaN-ordered, UINT32_MAX): sorts last

template <int E>
__device__ void sort_into_smem(uint64_t* s, int n) {
  const int lane = threadIdx.x & 31;
  uint64_t x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    x[e] = i < n ? s[i] : kNoNeighbor;
  }
  warp_sort<E>(x);
  __syncwarp();
#pragma unroll
  for (int e = 0; e < E; ++e) s[e * 32 + lane] = x[e];
  __syncwarp();
}

// Sorts s[0..n) (n <= 256) ascending in place, padding to the sort size with kNoNeighbor.
__device__ void sort_small(uint64_t* s, int n) {
  if (n <= 32) sort_into_smem<1>(s, n);
  else if (n <= 64) sort_into_smem<2>(s, n);
  else if (n <= 128) sort_into_smem<4>(s, n);
  else sort_into_smem<8>(s, n);
}

// The c-th smallest (1-based) of the n distinct packed keys s[0..n), c <= n: the c-th smallest
// 32-bit key K by a bitwise search from the top bit over keys held in registers (E per lane),
// then, only when the entries whose key is K do not all fit, the row among them by a search on
// the low word.
template <int E>
__device__ uint64_t kth_packed_regs(const uint64_t* s, int n, int c) {
  const int lane = threadIdx.x & 31;
  uint32_t k[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    k[e] = i < n ? static_cast<uint32_t>(s[i] >> 32) : 0xFFFFFFFFu;
  }
  uint32_t key = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = key | (1u << bit);
    int cnt = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) cnt += k[e] < cand ? 1 : 0;
    if (__reduce_add_sync(0xFFFFFFFFu, cnt) < c) key = cand;
  }
  // key = the largest value with fewer than c keys below it, so the c-th key itself.
  int below = 0, at = 0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    below += k[e] < key ? 1 : 0;
    at += (k[e] == key && e * 32 + lane < n) ? 1 : 0;
  }
  below = __reduce_add_sync(0xFFFFFFFFu, below);
  at = __reduce_add_sync(0xFFFFFFFFu, at);
  const int r = c - below;  // rank among the entries whose key is K
  if (r == at) return (static_cast<uint64_t>(key) << 32) | 0xFFFFFFFFull;
  uint32_t row = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = row | (1u << bit);
    int cnt = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = e * 32 + lane;
      cnt += (k[e] == key && i < n && static_cast<uint32_t>(s[i]) < cand) ? 1 : 0;
    }
    if (__reduce_add_sync(0xFFFFFFFFu, cnt) < r) row = cand;
  }
  return (static_cast<uint64_t>(key) << 32) | row;
}

// Keeps the c smallest of the n distinct packed keys s[0..n) (c < n <= kMaxSurvivors) in
// s[0..c), unordered: the c-th smallest (in registers up to 512 keys, else by a bitwise search
// over shared memory from the top bit), then a stable in-place compaction of the keys at or
// below it.
__device__ void keep_smallest(uint64_t* s, int n, int c) {
  const int lane = threadIdx.x & 31;
  uint64_t ans = 0;
  if (n <= 256) {
    ans = kth_packed_regs<8>(s, n, c);
  } else if (n <= 512) {
    ans = kth_packed_regs<16>(s, n, c);
  } else {
    for (int bit = 63; bit >= 0; --bit) {
      const uint64_t cand = ans | (1ull << bit);
      int cnt = 0;
      for (int i = lane; i < n; i += 32) cnt += s[i] < cand ? 1 : 0;
      cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
      if (cnt < c) ans = cand;
    }
  }
  const uint32_t lt = (1u << lane) - 1u;
  int w = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t x = i < n ? s[i] : kNoNeighbor;
    const bool keep = i < n && x <= ans;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
    if (keep) s[w + __popc(m & lt)] = x;  // every read of this pass precedes the ballot
    w += __popc(m);
  }
  __syncwarp();
}

// Candidate slot of (query tile, list, query row). A query has `wgs` lists per row slice (one
// per epilogue warpgroup of the scan): list p = wgs * slice + warpgroup. Units are numbered
// slice-major (scan_mma.cu unit_rows), so unit = slice * qtiles + qtile.
__device__ __forceinline__ size_t unit_slot(const FinalizeArgs& a, int qtile, int p,
                                            int row_in_tile) {
  const size_t qtiles = (static_cast<size_t>(a.nq) + kScanBM - 1) / kScanBM;
  const size_t unit = static_cast<size_t>(p / a.wgs) * qtiles + qtile;
  return (unit * a.wgs + (p % a.wgs)) * kScanBM + row_in_tile;
}

// The c-th smallest packed key (1-based) among the query's entries below `thr`, in four passes
// over its lists: a radix select on the pre-rank key (8-bit digits, a per-warp histogram of the
// keys that still match) finds the c-th key K and its rank r among the entries whose key is K;
// only when r leaves some of those out does a 32-pass search on their rows follow. Reached when a query's lists hold more than
// kMaxSurvivors entries below its bound (unseeded scans of few queries over many row slices).
__device__ uint64_t global_kth_radix(const FinalizeArgs& a, int qtile, int row_in_tile, uint32_t thr, int c,
                                     uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  const int lists = a.wgs * a.units_per_qtile;
  uint32_t prefix = 0, mask = 0, at_k = 0;
  int r = c;  // rank (1-based) of the c-th key among the keys that match the prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int b = 0; b < 8; ++b) hist[lane * 8 + b] = 0;
    __syncwarp();
    for (int p = 0; p < lists; ++p) {
      const size_t slot = unit_slot(a, qtile, p, row_in_tile);
      const int n = a.cand_count[slot];
      const uint2* bp = a.cand + slot * kScanCap;
      for (int e = lane; e < n; e += 32) {
        const uint32_t key = float_key(__uint_as_float(bp[e].x));
        if (key < thr && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
    }
    __syncwarp();
    uint32_t h[8], tot = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      h[b] = hist[lane * 8 + b];
      tot += h[b];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += v;
    }
    const uint32_t excl = incl - tot;
    const uint32_t owner =
        __ballot_sync(0xFFFFFFFFu, excl < static_cast<uint32_t>(r) && static_cast<uint32_t>(r) <= incl);
    const int src = __ffs(owner) - 1;
    uint32_t digit = 0, before = 0, cnt = 0;
    if (lane == src) {
      uint32_t run = excl;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (cnt == 0 && static_cast<uint32_t>(r) <= run + h[b]) {
          digit = static_cast<uint32_t>(lane * 8 + b);
          before = run;
          cnt = h[b];
        }
        run += h[b];
      }
    }
    digit = __shfl_sync(0xFFFFFFFFu, digit, src);
    before = __shfl_sync(0xFFFFFFFFu, before, src);
    at_k = __shfl_sync(0xFFFFFFFFu, cnt, src);
    r -= static_cast<int>(before);
    prefix |= digit << shift;
    mask |= 255u << shift;
    __syncwarp();
  }
  if (static_cast<uint32_t>(r) == at_k) return (static_cast<uint64_t>(prefix) << 32) | 0xFFFFFFFFull;
  // Ties on the key K: the r-th smallest row among the entries whose key is K.
  uint32_t ans = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = ans | (1u << bit);
    int cnt = 0;
    for (int p = 0; p < lists; ++p) {
      const size_t slot = unit_slot(a, qtile, p, row_in_tile);
      const int n = a.cand_count[slot];
      const uint2* bp = a.cand + slot * kScanCap;
      for (int e = lane; e < n; e += 32) {
        const uint2 v = bp[e];
        cnt += (float_key(__uint_as_float(v.x)) == prefix && v.y < cand) ? 1 : 0;
      }
    }
    cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
    if (cnt < r) ans = cand;
  }
  return (static_cast<uint64_t>(prefix) << 32) | ans;
}

__global__ void __launch_bounds__(kFinWarps * 32)
    finalize_kernel(const FinalizeArgs a) {
  extern __shared__ __align__(16) uint8_t fsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pd = a.pd;
  // Block-shared: vmin, scale (SQ8). Per warp: query, survivors / candidates.
  float* vmin_s = reinterpret_cast<float*>(fsm);
  float* scale_s = vmin_s + pd;
  uint8_t* wbase = fsm + 2 * pd * sizeof(float) +
                   warp * (pd * sizeof(float) + kMaxSurvivors * sizeof(uint64_t));
  float* q_s = reinterpret_cast<float*>(wbase);
  uint64_t* surv = reinterpret_cast<uint64_t*>(wbase + pd * sizeof(float));
  // The overflow path's histogram borrows the survivors' last 1 KB: that path selects before it
  // writes survivors, and then writes at most cpre <= 256 of them.
  uint32_t* hist = reinterpret_cast<uint32_t*>(surv + kMaxSurvivors - 128);
  if (a.codes != nullptr) {
    for (int i = threadIdx.x; i < pd; i += blockDim.x) {
      vmin_s[i] = a.vmin[i];
      scale_s[i] = a.scale[i];
    }
  }
  __syncthreads();
  const int q = blockIdx.x * kFinWarps + warp;
  if (q >= a.nq) return;
  for (int i = lane; i < pd; i += 32) q_s[i] = a.queries[static_cast<size_t>(q) * pd + i];
  const int qtile = q / kScanBM, row_in_tile = q % kScanBM;
  const uint32_t thr = a.qtau[q];  // keep key < thr (ordered); 0xFFFFFFFF keeps all
  const uint32_t lt = (1u << lane) - 1u;

  // 1. Gather the entries that can still be among the C best: lane p reads list p of each group
  // of 32, eight entries at a time in 16-byte loads (a list's slots are 16-byte aligned and
  // kScanCap is even, so the pair past an odd count stays inside the list), all issued before
  // any entry is filed.
  int nsurv = 0;
  const int lists = a.wgs * a.units_per_qtile;
  auto file = [&](uint32_t kx, uint32_t row, bool valid) {
    const uint32_t key = float_key(__uint_as_float(kx));
    const bool pass = valid && key < thr;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, pass);
    const int pos = nsurv + __popc(m & lt);
    if (pass && pos < kMaxSurvivors) surv[pos] = (static_cast<uint64_t>(key) << 32) | row;
    nsurv += __popc(m);
  };
  static_assert(kScanCap % 2 == 0, "pairs of list slots");
  for (int p0 = 0; p0 < lists; p0 += 32) {
    const int p = p0 + lane;
    int my_cnt = 0;
    const uint4* lp = nullptr;
    if (p < lists) {
      const size_t slot = unit_slot(a, qtile, p, row_in_tile);
      my_cnt = a.cand_count[slot];
      lp = reinterpret_cast<const uint4*>(a.cand + slot * kScanCap);
    }
    const int maxc = __reduce_max_sync(0xFFFFFFFFu, static_cast<uint32_t>(my_cnt));
    for (int e0 = 0; e0 < maxc; e0 += 8) {
      uint4 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        w[u] = e0 + 2 * u < my_cnt ? __ldg(&lp[(e0 >> 1) + u]) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        file(w[u].x, w[u].y, e0 + 2 * u < my_cnt);
        file(w[u].z, w[u].w, e0 + 2 * u + 1 < my_cnt);
      }
    }
  }
  __syncwarp();
  // With a seeded bound, fewer than cpre keys below it means some of the query's C best may
  // lie above the seed: the query is rescanned without one.
  if (a.fb_count != nullptr && nsurv < a.cpre) {
    if (lane == 0) a.fb_list[atomicAdd(a.fb_count, 1)] = static_cast<uint32_t>(q);
    return;
  }
  int ncand;
  if (nsurv <= kMaxSurvivors) {
    ncand = nsurv < a.cpre ? nsurv : a.cpre;
    if (nsurv > a.cpre) keep_smallest(surv, nsurv, a.cpre);
    sort_small(surv, ncand);
  } else {
    // Rare: select the cpre-th key over all entries, then gather exactly those <= it.
    const uint64_t kth = global_kth_radix(a, qtile, row_in_tile, thr, a.cpre, hist);
    int w = 0;
    for (int p = 0; p < a.wgs * a.units_per_qtile; ++p) {
      const size_t slot = unit_slot(a, qtile, p, row_in_tile);
      const int n = a.cand_count[slot];
      const uint2* b = a.cand + slot * kScanCap;
      for (int e0 = 0; e0 < n; e0 += 32) {
        const int e = e0 + lane;
        uint64_t pk = kNoNeighbor;
        bool pass = false;
        if (e < n) {
          const uint2 v = b[e];
          const uint32_t key = float_key(__uint_as_float(v.x));
          pk = (static_cast<uint64_t>(key) << 32) | v.y;
          pass = key < thr && pk <= kth;
        }
        const uint32_t m = __ballot_sync(0xFFFFFFFFu, pass);
        const int pos = w + __popc(m & lt);
        if (pass && pos < a.cpre) surv[pos] = pk;
        w += __popc(m);
      }
    }
    __syncwarp();
    ncand = w < a.cpre ? w : a.cpre;
    sort_small(surv, ncand);
  }

  // 2. Exact distances of the candidates (stored back as packed (dist, row)).
  const bool l2 = a.metric == 0;
  // Exact fp32 distances of surv[0..n) on the float rows, 4 gathers in flight at a time.
  const bool packed128 = pd == 128 && a.order == kOrderAvx512;
  auto exact_rows = [&](int n) {
    if (packed128) {
      warp_dists128_f32(a.rows, q_s, n, l2, [&](int i) { return neighbor_id(surv[i]); },
                        [&](int i, float v) { surv[i] = pack_neighbor(v, neighbor_id(surv[i])); });
      return;
    }
    for (int i = 0; i < n; i += 4) {
      uint32_t r[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = neighbor_id(surv[i + c < n ? i + c : i]);
      float d[4];
      if (a.order == kOrderAvx512 && pd <= 8 * 32 + 16) {
        warp_exact_dist4_avx512<8>(q_s, a.rows, r, n - i, pd, l2, d);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          d[c] = warp_exact_dist(q_s, a.rows + static_cast<size_t>(r[c]) * pd, pd, l2, a.order);
      }
      __syncwarp();
      if (lane < 4 && i + lane < n) {
        float dl = d[0];
        uint32_t rl = r[0];
#pragma unroll
        for (int c = 1; c < 4; ++c) {
          dl = lane == c ? d[c] : dl;
          rl = lane == c ? r[c] : rl;
        }
        surv[i + lane] = pack_neighbor(dl, rl);
      }
      __syncwarp();
    }
  };
  if (a.codes == nullptr) {
    exact_rows(ncand);
    sort_small(surv, ncand);
  } else if (packed128) {
    warp_dists128_sq8(a.codes, q_s, vmin_s, scale_s, ncand, l2, [&](int i) { return neighbor_id(surv[i]); },
                      [&](int i, float v) { surv[i] = pack_neighbor(v, neighbor_id(surv[i])); });
    sort_small(surv, ncand);
    if (a.depth > 0) {
      const int nr = ncand < a.depth ? ncand : a.depth;
      exact_rows(nr);
      ncand = nr;
      sort_small(surv, ncand);
    }
  } else {
    for (int i = 0; i < ncand; i += 8) {
      // Four pairs of codes per iteration: half-warp h takes candidates i+2c+h, c = 0..3.
      float d[4];
      uint32_t row[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int my = i + 2 * c + (lane >> 4);
        row[c] = neighbor_id(surv[my < ncand ? my : i]);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        d[c] = halfwarp_sq8_dist(q_s, a.codes + static_cast<size_t>(row[c]) * pd, vmin_s, scale_s,
                                 pd, l2, a.order);
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int my = i + 2 * c + (lane >> 4);
        if ((lane & 15) == 0 && my < ncand) surv[my] = pack_neighbor(d[c], row[c]);
      }
      __syncwarp();
    }
    sort_small(surv, ncand);
    if (a.depth > 0) {
      const int nr = ncand < a.depth ? ncand : a.depth;
      exact_rows(nr);
      ncand = nr;
      sort_small(surv, ncand);
    }
  }

  // 3. The k best, closest first; missing slots are (+inf, UINT32_MAX).
  for (int i = lane; i < a.k; i += 32) {
    const size_t o = static_cast<size_t>(q) * a.k + i;
    if (i < ncand) {
      a.out_dist[o] = neighbor_dist(surv[i]);
      a.out_row[o] = neighbor_id(surv[i]);
    } else {
      a.out_dist[o] = INFINITY;
      a.out_row[o] = UINT32_MAX;
    }
  }
}

// ------------------------------------------------------------------ IVF-PQ exact stage (list mode)

constexpr int kIvfFinWarps = 4;

// L2SqAny(q - c, b) over d elements with the residual formed on the fly: l2_any's arithmetic on
// the values the reference stores first (r = q - c, src/index/quant/ivf_pq.cc:206-208).
__device__ __forceinline__ float l2_any_resid(const float* q, const float* c, const float* b, int d) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= d; i += 4) {
    const float t0 = __fsub_rn(__fsub_rn(q[i], c[i]), b[i]);
    const float t1 = __fsub_rn(__fsub_rn(q[i + 1], c[i + 1]), b[i + 1]);
    const float t2 = __fsub_rn(__fsub_rn(q[i + 2], c[i + 2]), b[i + 2]);
    const float t3 = __fsub_rn(__fsub_rn(q[i + 3], c[i + 3]), b[i + 3]);
    s0 = __fadd_rn(s0, __fmul_rn(t0, t0));
    s1 = __fadd_rn(s1, __fmul_rn(t1, t1));
    s2 = __fadd_rn(s2, __fmul_rn(t2, t2));
    s3 = __fadd_rn(s3, __fmul_rn(t3, t3));
  }
  for (; i < d; ++i) {
    const float t = __fsub_rn(__fsub_rn(q[i], c[i]), b[i]);
    s0 = __fadd_rn(s0, __fmul_rn(t, t));
  }
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

__global__ void __launch_bounds__(kIvfFinWarps * 32) ivf_finalize_kernel(const IvfFinalizeArgs a) {
  extern __shared__ __align__(16) uint8_t ivsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pd = a.pd;
  uint8_t* wbase = ivsm + warp * (pd * sizeof(float) + kMaxSurvivors * sizeof(uint64_t));
  float* q_s = reinterpret_cast<float*>(wbase);
  uint64_t* surv = reinterpret_cast<uint64_t*>(wbase + pd * sizeof(float));
  const int q = static_cast<int>(blockIdx.x) * kIvfFinWarps + warp;
  if (q >= a.nq) return;
  for (int i = lane; i < pd; i += 32) q_s[i] = a.queries[static_cast<size_t>(q) * pd + i];
  const uint32_t thr = a.qtau[q];
  const uint32_t lt = (1u << lane) - 1u;
  __syncwarp();
  long long t_mark = clock64();
  auto stage = [&](int i) {
    if (a.counters == nullptr) return;
    const long long t = clock64();
    if (lane == 0) atomicAdd(&a.counters[i], static_cast<unsigned long long>(t - t_mark));
    t_mark = t;
  };

  // 1. The entries below the bound: lane j reads list j (probe j / wgs, epilogue warpgroup
  // j % wgs of the probe's tile), eight entries at a time; each entry is offered as (ordered
  // pre-rank key, probe << 24 | row within the list). walk(f) calls f(key, tag, valid) in lockstep
  // over the warp.
  const int lists = a.nprobe * a.wgs;
  uint32_t scanned = 0;  // rows of the probed lists
  auto walk = [&](auto&& f, bool count_rows) {
    for (int j0 = 0; j0 < lists; j0 += 32) {
      const int j = j0 + lane;
      int cnt = 0;
      const uint4* lp = nullptr;
      uint32_t p = 0;
      uint64_t pb = 0;
      if (j < lists) {
        p = static_cast<uint32_t>(j / a.wgs);
        const int wg = j % a.wgs;
        const size_t pair = static_cast<size_t>(q) * a.nprobe + p;
        const uint32_t l = a.probe_ids[pair];
        const uint32_t slot = a.pair_slot[pair];
        const size_t cs = (static_cast<size_t>(slot / 128) * a.wgs + wg) * 128 + slot % 128;
        cnt = a.cand_count[cs];
        lp = reinterpret_cast<const uint4*>(a.cand + cs * kScanCap);
        pb = a.poff[l];
        if (count_rows && wg == 0) scanned += static_cast<uint32_t>(a.list_off[l + 1] - a.list_off[l]);
      }
      const int maxc = static_cast<int>(__reduce_max_sync(0xFFFFFFFFu, static_cast<uint32_t>(cnt)));
      for (int e0 = 0; e0 < maxc; e0 += 8) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = e0 + 2 * u < cnt ? __ldg(&lp[(e0 >> 1) + u]) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          f(float_key(__uint_as_float(w[u].x)), (p << 24) | static_cast<uint32_t>(w[u].y - pb), e0 + 2 * u < cnt);
          f(float_key(__uint_as_float(w[u].z)), (p << 24) | static_cast<uint32_t>(w[u].w - pb), e0 + 2 * u + 1 < cnt);
        }
      }
    }
  };
  int nsurv = 0;
  auto file = [&](uint32_t key, uint32_t tag, bool valid) {
    const bool pass = valid && key < thr;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, pass);
    const int pos = nsurv + __popc(m & lt);
    if (pass && pos < kMaxSurvivors) surv[pos] = (static_cast<uint64_t>(key) << 32) | tag;
    nsurv += __popc(m);
  };
  walk(file, true);
  scanned = __reduce_add_sync(0xFFFFFFFFu, scanned);
  __syncwarp();
  if (a.counters != nullptr && lane == 0) {
    atomicAdd(&a.counters[0], static_cast<unsigned long long>(nsurv));
    if (nsurv > kMaxSurvivors) atomicAdd(&a.counters[1], 1ull);
  }
  if (nsurv > kMaxSurvivors) {
    // More entries below the bound than shared memory holds: the cpre-th (key, tag) over the
    // lists by a radix select on the key (8-bit digits, a per-warp histogram in the survivors'
    // last 1 KB) and, when the entries at that key do not all fit, a search on the tag; then
    // exactly the cpre entries at or below it are gathered.
    uint32_t* hist = reinterpret_cast<uint32_t*>(surv + kMaxSurvivors - 128);
    uint32_t prefix = 0, mask = 0, at_k = 0;
    int r = a.cpre;
    for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) hist[lane * 8 + bb] = 0;
      __syncwarp();
      walk([&](uint32_t key, uint32_t, bool valid) {
        if (valid && key < thr && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }, false);
      __syncwarp();
      uint32_t h[8], tot = 0;
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) {
        h[bb] = hist[lane * 8 + bb];
        tot += h[bb];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += v;
      }
      const uint32_t excl = incl - tot;
      const uint32_t owner =
          __ballot_sync(0xFFFFFFFFu, excl < static_cast<uint32_t>(r) && static_cast<uint32_t>(r) <= incl);
      const int src = __ffs(owner) - 1;
      uint32_t digit = 0, before = 0, cnt = 0;
      if (lane == src) {
        uint32_t run = excl;
#pragma unroll
        for (int bb = 0; bb < 8; ++bb) {
          if (cnt == 0 && static_cast<uint32_t>(r) <= run + h[bb]) {
            digit = static_cast<uint32_t>(lane * 8 + bb);
            before = run;
            cnt = h[bb];
          }
          run += h[bb];
        }
      }
      digit = __shfl_sync(0xFFFFFFFFu, digit, src);
      before = __shfl_sync(0xFFFFFFFFu, before, src);
      at_k = __shfl_sync(0xFFFFFFFFu, cnt, src);
      r -= static_cast<int>(before);
      prefix |= digit << shift;
      mask |= 255u << shift;
      __syncwarp();
    }
    uint32_t tag_cut = 0xFFFFFFFFu;
    if (static_cast<uint32_t>(r) != at_k) {
      tag_cut = 0;
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = tag_cut | (1u << bit);
        int c = 0;
        walk([&](uint32_t key, uint32_t tag, bool valid) { c += (valid && key == prefix && tag < cand) ? 1 : 0; },
             false);
        if (__reduce_add_sync(0xFFFFFFFFu, static_cast<uint32_t>(c)) < static_cast<uint32_t>(r)) tag_cut = cand;
      }
    }
    const uint64_t kth = (static_cast<uint64_t>(prefix) << 32) | tag_cut;
    nsurv = 0;
    walk([&](uint32_t key, uint32_t tag, bool valid) {
      file(key, tag, valid && ((static_cast<uint64_t>(key) << 32) | tag) <= kth);
    }, false);
    __syncwarp();
  }
  int ncand = nsurv < a.cpre ? nsurv : a.cpre;
  if (nsurv > a.cpre) keep_smallest(surv, nsurv, a.cpre);

  stage(2);
  // 2. The reference's ADC of each candidate (one lane per candidate): its table entries
  // term2 + 2 * (-<q_j, C_j[c]>) (precomputed) or L2SqAny(q_j - c_j, C_j[c]) (residual), summed in
  // four partial sums, plus the coarse distance (precomputed tables).
  const int m = a.m, ds = a.dsub;
  const size_t ts = static_cast<size_t>(m) * 256;
  const bool fast_adc = a.mode == kIvfPrecomputed && ds == 2 && m % 16 == 0 && m <= 64 &&
                        (reinterpret_cast<uintptr_t>(a.codes) & 15u) == 0;
  for (int i = lane; i < ncand; i += 32) {
    const uint32_t tag = static_cast<uint32_t>(surv[i]);
    const uint32_t p = tag >> 24;
    const size_t pair = static_cast<size_t>(q) * a.nprobe + p;
    const uint32_t l = a.probe_ids[pair];
    const uint64_t pos = a.list_off[l] + (tag & 0xFFFFFFu);
    const uint8_t* code = a.codes + pos * m;
    const float* t2 = a.mode == kIvfPrecomputed ? a.term2 + l * ts : nullptr;
    const float* cl = a.coarse + static_cast<size_t>(l) * pd;
    auto entry = [&](int j) {
      const int c = code[j];
      const float* cen = a.centroids + (static_cast<size_t>(j) * 256 + c) * ds;
      if (a.mode == kIvfPrecomputed)
        return __fadd_rn(__ldg(&t2[j * 256 + c]), __fmul_rn(-dot_any(q_s + j * ds, cen, ds), 2.f));
      return l2_any_resid(q_s + j * ds, cl + j * ds, cen, ds);
    };
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    if (fast_adc) {
      // The code in registers (16-byte loads), then per chunk of 8 sub-quantizers every term2
      // entry and centroid pair requested before any is used; entries are added to the partial
      // sums in ascending j, as the reference's loop does.
      uint32_t w[16];
      const uint4* cp = reinterpret_cast<const uint4*>(code);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint4 v = t * 16 < m ? __ldg(&cp[t]) : make_uint4(0, 0, 0, 0);
        w[4 * t] = v.x;
        w[4 * t + 1] = v.y;
        w[4 * t + 2] = v.z;
        w[4 * t + 3] = v.w;
      }
      const float2* cen2 = reinterpret_cast<const float2*>(a.centroids);
#pragma unroll
      for (int j0 = 0; j0 < 64; j0 += 8) {
        if (j0 < m) {
          float tv[8];
          float2 cv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int j = j0 + u;
            const uint32_t c = (w[j >> 2] >> (8 * (j & 3))) & 255u;
            tv[u] = __ldg(&t2[j * 256 + c]);
            cv[u] = __ldg(&cen2[j * 256 + c]);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int j = j0 + u;
            const float dq = dot_any(q_s + 2 * j, reinterpret_cast<const float*>(&cv[u]), 2);
            s[j & 3] = __fadd_rn(s[j & 3], __fadd_rn(tv[u], __fmul_rn(-dq, 2.f)));
          }
        }
      }
    } else {
      int j = 0;
      for (; j + 4 <= m; j += 4) {
        s[0] = __fadd_rn(s[0], entry(j));
        s[1] = __fadd_rn(s[1], entry(j + 1));
        s[2] = __fadd_rn(s[2], entry(j + 2));
        s[3] = __fadd_rn(s[3], entry(j + 3));
      }
      for (; j < m; ++j) s[0] = __fadd_rn(s[0], entry(j));
    }
    // The coarse distance is the offset of the precomputed tables only (the residual tables
    // already measure from the query).
    const float off = a.mode == kIvfPrecomputed ? a.probe_dist[pair] : 0.f;
    const float d = __fadd_rn(off, __fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3])));
    surv[i] = pack_neighbor(d, __ldg(&a.ids[pos]));
  }
  __syncwarp();
  stage(3);
  // 3. TopK(R) by (dist, id), then the re-rank on fp32 rows (exact, reference kernel-set order).
  sort_small(surv, ncand);
  const int R = a.depth > a.k ? a.depth : a.k;
  ncand = ncand < R ? ncand : R;
  uint32_t dc = static_cast<uint32_t>(a.nlist) + scanned;
  if (a.depth > 0 && a.order == kOrderAvx512 && (pd == 96 || pd == 128)) {
    auto id_at = [&](int i) { return neighbor_id(surv[i]); };
    auto put = [&](int i, float v) { surv[i] = pack_neighbor(v, neighbor_id(surv[i])); };
    if (pd == 96) warp_dists_f32x2<3>(a.rows, q_s, ncand, true, id_at, put);
    else warp_dists_f32x2<4>(a.rows, q_s, ncand, true, id_at, put);
    sort_small(surv, ncand);
    dc += static_cast<uint32_t>(ncand);
  } else if (a.depth > 0) {
    for (int i = 0; i < ncand; i += 4) {
      uint32_t r[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = neighbor_id(surv[i + c < ncand ? i + c : i]);
      float d[4];
      if (a.order == kOrderAvx512 && pd <= 8 * 32 + 16) {
        warp_exact_dist4_avx512<8>(q_s, a.rows, r, ncand - i, pd, true, d);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) d[c] = warp_exact_dist(q_s, a.rows + static_cast<size_t>(r[c]) * pd, pd, true, a.order);
      }
      __syncwarp();
      if (lane < 4 && i + lane < ncand) {
        float dl = d[0];
        uint32_t rl = r[0];
#pragma unroll
        for (int c = 1; c < 4; ++c) {
          dl = lane == c ? d[c] : dl;
          rl = lane == c ? r[c] : rl;
        }
        surv[i + lane] = pack_neighbor(dl, rl);
      }
      __syncwarp();
    }
    sort_small(surv, ncand);
    dc += static_cast<uint32_t>(ncand);
  }
  for (int i = lane; i < a.k; i += 32) {
    const size_t o = static_cast<size_t>(q) * a.k + i;
    if (i < ncand) {
      a.out_dist[o] = neighbor_dist(surv[i]);
      a.out_row[o] = neighbor_id(surv[i]);
    } else {
      a.out_dist[o] = INFINITY;
      a.out_row[o] = UINT32_MAX;
    }
  }
  if (lane == 0 && a.out_dc != nullptr) a.out_dc[q] = dc;
  stage(4);
}

// ------------------------------------------------------------------ seeded scans

// One warp per query: the m-th smallest ordered key over the query's lists. Keys at or above the
// bound the pass itself left in qtau_out[q] cannot be among the m smallest (a slice that compacted
// kept m keys below it; without compactions every list holds all keys below it), so only keys
// below it are gathered, once, into shared memory, and searched bit by bit from the top (the
// largest v with fewer than m keys below it). Fewer than m keys below the bound: no estimate.
constexpr int kSeedWarps = 4;
constexpr int kSeedCap = 1024;

__global__ void __launch_bounds__(kSeedWarps * 32) scan_seed_kernel(const SeedArgs a) {
  __shared__ uint32_t keys_s[kSeedWarps][kSeedCap];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = static_cast<int>(blockIdx.x) * kSeedWarps + warp;
  if (q >= a.nq) return;
  const size_t qtiles = (static_cast<size_t>(a.nq) + kScanBM - 1) / kScanBM;
  const int qtile = q / kScanBM, row_in_tile = q % kScanBM;
  const int lists = a.units_per_qtile * a.wgs;
  const uint32_t thr = a.qtau_out[q];
  const uint32_t lt = (1u << lane) - 1u;
  uint32_t* ks = keys_s[warp];
  auto list_of = [&](int p, int* n) {
    const size_t unit = static_cast<size_t>(p / a.wgs) * qtiles + qtile;
    const size_t slot = (unit * a.wgs + (p % a.wgs)) * kScanBM + row_in_tile;
    *n = a.cand_count[slot];
    return a.cand + slot * kScanCap;
  };
  int n = 0;
  for (int p = 0; p < lists; ++p) {
    int cnt;
    const uint2* b = list_of(p, &cnt);
    for (int e0 = 0; e0 < cnt; e0 += 32) {
      const int e = e0 + lane;
      uint32_t key = 0xFFFFFFFFu;
      if (e < cnt) key = float_key(__uint_as_float(b[e].x));
      const bool pass = e < cnt && key < thr;
      const uint32_t mk = __ballot_sync(0xFFFFFFFFu, pass);
      const int pos = n + __popc(mk & lt);
      if (pass && pos < kSeedCap) ks[pos] = key;
      n += __popc(mk);
    }
  }
  __syncwarp();
  uint32_t ans = 0xFFFFFFFFu;
  if (n >= a.m) {
    ans = 0;
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t cand = ans | (1u << bit);
      int c = 0;
      if (n <= kSeedCap) {
        for (int i = lane; i < n; i += 32) c += ks[i] < cand ? 1 : 0;
      } else {  // rare: too many keys below the bound for shared memory
        for (int p = 0; p < lists; ++p) {
          int cnt;
          const uint2* b = list_of(p, &cnt);
          for (int e = lane; e < cnt; e += 32) {
            const uint32_t key = float_key(__uint_as_float(b[e].x));
            c += (key < thr && key < cand) ? 1 : 0;
          }
        }
      }
      c = __reduce_add_sync(0xFFFFFFFFu, c);
      if (c < a.m) ans = cand;
    }
  }
  if (lane == 0) a.qtau_out[q] = ans;
}

__global__ void scatter_results_kernel(const float* src_dist, const uint32_t* src_row,
                                       const uint32_t* list, uint32_t n, int k, float* out_dist,
                                       uint32_t* out_row) {
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<uint64_t>(n) * k) return;
  const uint64_t r = i / k, j = i % k;
  const uint64_t o = static_cast<uint64_t>(list[r]) * k + j;
  out_dist[o] = src_dist[i];
  out_row[o] = src_row[i];
}

// ------------------------------------------------------------------ operand preparation

__global__ void prep_queries_kernel(const PrepArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.nq_pad) return;
  const int q = warp;
  const bool valid = q < a.nq;
  // Operand values a_i of this query.
  float amax = 0.f;
  for (int i = lane; i < a.pd; i += 32) {
    float v = 0.f;
    if (valid) {
      const float x = a.queries[static_cast<size_t>(q) * a.pd + i];
      if (a.kind == kPrepFlat) v = x;
      else if (a.kind == kPrepSq8Ip) v = x * a.scale[i];
      else v = (x - a.vmin[i]) * a.scale[i];
    }
    amax = fmaxf(amax, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  // Power-of-two scale bringing max|a| into [2^14, 2^15) for fp16 (exact rescaling).
  int s = 0;
  if (a.ab_format == 0 && amax > 0.f) {
    s = 14 - ilogbf(amax);
    s = s < -100 ? -100 : (s > 100 ? 100 : s);
  }
  const float up = ldexpf(1.f, s);
  for (int i = lane; i < a.kpad; i += 32) {
    float v = 0.f;
    if (valid && i < a.pd) {
      const float x = a.queries[static_cast<size_t>(q) * a.pd + i];
      if (a.kind == kPrepFlat) v = x;
      else if (a.kind == kPrepSq8Ip) v = x * a.scale[i];
      else v = (x - a.vmin[i]) * a.scale[i];
      v *= up;
    }
    const size_t o = static_cast<size_t>(q) * a.kpad + i;
    if (a.ab_format == 0) reinterpret_cast<__half*>(a.operand)[o] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(a.operand)[o] = __float2bfloat16_rn(v);
  }
  if (lane == 0 && valid) {
    // key = qscale * acc (+ row term): acc = 2^s * <a, b>.
    const float down = ldexpf(1.f, -s - a.row_scale_log2);
    a.qscale[q] = (a.key_factor == 2 ? -2.f : -1.f) * down;
  }
}

__global__ void prep_rows_kernel(const float* __restrict__ rows, uint64_t n, int pd, int kpad,
                                 int ab_format, int scale_log2, void* operand, float* norms) {
  const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const float up = ldexpf(1.f, scale_log2);
  float ss = 0.f;
  for (int i = lane; i < kpad; i += 32) {
    const float x = i < pd ? rows[warp * pd + i] : 0.f;
    ss = fmaf(x, x, ss);
    const size_t o = warp * kpad + i;
    if (ab_format == 0) reinterpret_cast<__half*>(operand)[o] = __float2half_rn(x * up);
    else reinterpret_cast<__nv_bfloat16*>(operand)[o] = __float2bfloat16_rn(x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  if (norms != nullptr && lane == 0) norms[warp] = ss;
}

__global__ void absmax_kernel(const float* __restrict__ x, uint64_t count, uint32_t* out) {
  float m = 0.f;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// Per-dimension min/max over all rows (Sq8Quantizer::train, sq8.cc:9-26), in ordered-key space.
__global__ void sq8_minmax_kernel(const float* __restrict__ rows, uint64_t n, int dim, int pd,
                                  uint32_t* kmin, uint32_t* kmax) {
  const int d = threadIdx.x;
  if (d >= dim) return;
  uint32_t lo = 0xFFFFFFFFu, hi = 0u;
  for (uint64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const uint32_t k = float_key(rows[r * pd + d]);
    lo = k < lo ? k : lo;
    hi = k > hi ? k : hi;
  }
  atomicMin(&kmin[d], lo);
  atomicMax(&kmax[d], hi);
}

// Sq8Quantizer::encode (sq8.cc:28-37): nearbyint((x - vmin) / scale) with IEEE division,
// clamped to [0, 255]; padding dimensions and scale <= 0 encode 0. Also writes the fp16 operand
// copy of the code and, for L2, the row term sum_i (scale_i * code_i)^2.
__global__ void sq8_encode_kernel(const float* __restrict__ rows, uint64_t n, int dim, int pd,
                                  int kpad, const float* __restrict__ vmin,
                                  const float* __restrict__ scale, uint8_t* codes,
                                  __half* operand, float* rowterm) {
  const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  float ss = 0.f;
  for (int i = lane; i < kpad; i += 32) {
    uint8_t c = 0;
    if (i < pd && i < dim && scale[i] > 0.f) {
      float v = rintf(__fdiv_rn(__fsub_rn(rows[warp * pd + i], vmin[i]), scale[i]));
      v = v < 0.f ? 0.f : (255.f < v ? 255.f : v);
      c = static_cast<uint8_t>(v);
    }
    if (i < pd) codes[warp * pd + i] = c;
    const float cf = static_cast<float>(c);
    operand[warp * kpad + i] = __float2half_rn(cf);
    if (i < pd) {
      const float t = scale[i] * cf;
      ss = fmaf(t, t, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  if (rowterm != nullptr && lane == 0) rowterm[warp] = ss;
}

// fp16 operand and row term from existing codes (codes loaded from an index file).
__global__ void sq8_operand_kernel(const uint8_t* __restrict__ codes, uint64_t n, int pd, int kpad,
                                   const float* __restrict__ scale, __half* operand,
                                   float* rowterm) {
  const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  float ss = 0.f;
  for (int i = lane; i < kpad; i += 32) {
    const float cf = i < pd ? static_cast<float>(codes[warp * pd + i]) : 0.f;
    operand[warp * kpad + i] = __float2half_rn(cf);
    if (i < pd) {
      const float t = scale[i] * cf;
      ss = fmaf(t, t, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  if (rowterm != nullptr && lane == 0) rowterm[warp] = ss;
}

}  // namespace

size_t FinalizeSmemBytes(int pd) {
  return 2 * pd * sizeof(float) + kFinWarps * (pd * sizeof(float) + kMaxSurvivors * sizeof(uint64_t));
}

cudaError_t LaunchFinalize(const FinalizeArgs& a, cudaStream_t stream) {
  const size_t smem = FinalizeSmemBytes(a.pd);
  cudaError_t e = cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int blocks = (a.nq + kFinWarps - 1) / kFinWarps;
  NoteLaunch();
  finalize_kernel<<<blocks, kFinWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchIvfFinalize(const IvfFinalizeArgs& a, cudaStream_t stream) {
  if (a.nq <= 0) return cudaSuccess;
  if (a.cpre > 256 || a.k > 256 || a.depth > 256 || a.nprobe > 128 || a.pd > 8 * 32 + 16)
    return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(kIvfFinWarps) * (a.pd * sizeof(float) + kMaxSurvivors * sizeof(uint64_t));
  cudaError_t e = cudaFuncSetAttribute(ivf_finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  NoteLaunch();
  ivf_finalize_kernel<<<(a.nq + kIvfFinWarps - 1) / kIvfFinWarps, kIvfFinWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchScanSeed(const SeedArgs& a, cudaStream_t stream) {
  if (a.nq <= 0) return cudaSuccess;
  const int blocks = (a.nq + kSeedWarps - 1) / kSeedWarps;
  NoteLaunch();
  scan_seed_kernel<<<blocks, kSeedWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchScatterResults(const float* src_dist, const uint32_t* src_row, const uint32_t* list,
                                 uint32_t n, int k, float* out_dist, uint32_t* out_row,
                                 cudaStream_t stream) {
  const uint64_t total = static_cast<uint64_t>(n) * k;
  if (total == 0) return cudaSuccess;
  NoteLaunch();
  scatter_results_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      src_dist, src_row, list, n, k, out_dist, out_row);
  return cudaGetLastError();
}

cudaError_t LaunchPrepQueries(const PrepArgs& a, cudaStream_t stream) {
  const int threads = 256;
  const int blocks = (a.nq_pad * 32 + threads - 1) / threads;
  NoteLaunch();
  prep_queries_kernel<<<blocks, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchPrepRows(const float* rows, uint64_t n, int pd, int kpad, int ab_format,
                           int scale_log2, void* operand, float* norms, cudaStream_t stream) {
  const int threads = 256;
  const uint64_t blocks = (n * 32 + threads - 1) / threads;
  NoteLaunch();
  prep_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      rows, n, pd, kpad, ab_format, scale_log2, operand, norms);
  return cudaGetLastError();
}

cudaError_t LaunchAbsMax(const float* x, uint64_t count, uint32_t* out, cudaStream_t stream) {
  NoteLaunch();
  absmax_kernel<<<1184, 256, 0, stream>>>(x, count, out);
  return cudaGetLastError();
}

cudaError_t LaunchSq8MinMax(const float* rows, uint64_t n, int dim, int pd, uint32_t* kmin,
                            uint32_t* kmax, cudaStream_t stream) {
  if (dim > 1024) return cudaErrorInvalidValue;
  uint64_t blocks = n < 4096 ? (n == 0 ? 1 : n) : 4096;
  NoteLaunch();
  sq8_minmax_kernel<<<static_cast<unsigned>(blocks), dim, 0, stream>>>(rows, n, dim, pd, kmin, kmax);
  return cudaGetLastError();
}

cudaError_t LaunchSq8Encode(const float* rows, uint64_t n, int dim, int pd, int kpad,
                            const float* vmin, const float* scale, uint8_t* codes, __half* operand,
                            float* rowterm, cudaStream_t stream) {
  const int threads = 256;
  const uint64_t blocks = (n * 32 + threads - 1) / threads;
  NoteLaunch();
  sq8_encode_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      rows, n, dim, pd, kpad, vmin, scale, codes, operand, rowterm);
  return cudaGetLastError();
}

cudaError_t LaunchSq8Operand(const uint8_t* codes, uint64_t n, int pd, int kpad, const float* scale,
                             __half* operand, float* rowterm, cudaStream_t stream) {
  const int threads = 256;
  const uint64_t blocks = (n * 32 + threads - 1) / threads;
  NoteLaunch();
  sq8_operand_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(codes, n, pd, kpad,
                                                                            scale, operand, rowterm);
  return cudaGetLastError();
}

}  // namespace vdbgpu
