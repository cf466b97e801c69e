// Batched HNSW search over the reference's own graphs (sm_100a), one warp per query.
//
// Follows HnswGraph::search (src/index/hnsw/hnsw_graph.h:286-309) step for step: greedy descent
// over the upper layers (greedy<false>, :482-508), then the ef-beam on layer 0
// (search_layer<false, filtered>, :513-567), then HnswSq8Index's fp32 re-rank
// (src/index/hnsw/hnsw_index.cc:82-102). Distances are summed in the order of the reference's
// runtime kernel set, so for the same graph and inputs the walk takes the same path and returns
// the same neighbours, distances and distance-computation counts.
//
// Parallel where the reference is sequential, without changing the result:
//   * the distances of a node's neighbours are independent: four quarter-warps compute four rows
//     at a time (8 lanes emulate one 16-lane AVX-512 accumulator pair, same adds in the same tree);
//   * visited marks go to a per-warp open-addressing hash in shared memory (the reference's
//     tag array, visited_pool.h:16-41; a list never holds a node twice, so marking a whole list at
//     once is equivalent);
//   * the heaps are sorted arrays. (dist, id) is a total order, so popping the least candidate and
//     evicting the greatest result pick the same elements a binary heap picks. Heap updates are
//     applied one neighbour at a time, in list order, with the reference's
//     "results.size() < ef || d < lower" rule.
//   * once the result set holds ef entries its worst distance can only fall, so a candidate
//     farther than it can never be expanded and is dropped when the candidate array is full.
#include <cuda_runtime.h>

#include "common.cuh"
#include "hnsw.cuh"
#include "warp_ops.cuh"

namespace vdbgpu {
namespace {

constexpr int kHnswWarps = 4;
constexpr uint32_t kEmpty = 0u;

struct WarpSmem {
  float* q;           // pd floats
  uint32_t* hash;     // 1 << hash_bits slots (id + 1, 0 = empty)
  uint64_t* res;      // ef sorted ascending packed (dist, id)
  uint64_t* cand;     // cand_cap, ascending from index head
  uint32_t* nb_id;    // 32 neighbour ids of the current expansion (new ones, compacted)
  float* nb_d;        // their distances
};

__device__ __forceinline__ uint32_t hash_slot(uint32_t id, int bits) {
  return (id * 2654435761u) >> (32 - bits);
}

// Marks `id` visited; true when it was not visited before. Sets *full when the table has no
// free slot left on the probe path (the caller reports an overflow).
__device__ __forceinline__ bool visit(uint32_t* hash, int bits, uint32_t id, bool* full) {
  const uint32_t mask = (1u << bits) - 1u;
  uint32_t s = hash_slot(id, bits);
  const uint32_t key = id + 1u;
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    const uint32_t prev = atomicCAS(&hash[s], kEmpty, key);
    if (prev == kEmpty) return true;
    if (prev == key) return false;
    s = (s + 1u) & mask;
  }
  *full = true;
  return false;
}

// Distance of the query (shared memory) to 4 rows at once: lanes 8g..8g+7 take row r[g].
// Float rows: the reference kernel set's order. Returns the distance of this lane's group.
template <bool kSq8>
__device__ __forceinline__ float group_dist(const HnswArgs& a, const float* q_s, uint32_t row,
                                            bool l2) {
  const int j = threadIdx.x & 7;
  const int pd = a.pd;
  float r;
  if (!kSq8) {
    const float* x = a.rows + static_cast<size_t>(row) * pd;
    if (a.order == kOrderAvx512) {
      const int nb = pd >> 5;
      float a0 = 0.f, a0b = 0.f, a1 = 0.f, a1b = 0.f;
      for (int t = 0; t < nb; ++t) {
        const int e = 32 * t + j;
        const float x0 = __ldg(&x[e]), x1 = __ldg(&x[e + 8]), x2 = __ldg(&x[e + 16]), x3 = __ldg(&x[e + 24]);
        if (l2) {
          const float d0 = __fsub_rn(q_s[e], x0), d1 = __fsub_rn(q_s[e + 8], x1);
          const float d2 = __fsub_rn(q_s[e + 16], x2), d3 = __fsub_rn(q_s[e + 24], x3);
          a0 = __fmaf_rn(d0, d0, a0);
          a0b = __fmaf_rn(d1, d1, a0b);
          a1 = __fmaf_rn(d2, d2, a1);
          a1b = __fmaf_rn(d3, d3, a1b);
        } else {
          a0 = __fmaf_rn(q_s[e], x0, a0);
          a0b = __fmaf_rn(q_s[e + 8], x1, a0b);
          a1 = __fmaf_rn(q_s[e + 16], x2, a1);
          a1b = __fmaf_rn(q_s[e + 24], x3, a1b);
        }
      }
      if ((pd & 31) != 0) {
        const int e = 32 * nb + j;
        const float x0 = __ldg(&x[e]), x1 = __ldg(&x[e + 8]);
        if (l2) {
          const float d0 = __fsub_rn(q_s[e], x0), d1 = __fsub_rn(q_s[e + 8], x1);
          a0 = __fmaf_rn(d0, d0, a0);
          a0b = __fmaf_rn(d1, d1, a0b);
        } else {
          a0 = __fmaf_rn(q_s[e], x0, a0);
          a0b = __fmaf_rn(q_s[e + 8], x1, a0b);
        }
      }
      // s[j] = acc0[j] + acc1[j]; T3[j] = s[j+8] + s[j]; then lanes +4, +2, +1.
      float t3 = __fadd_rn(__fadd_rn(a0b, a1b), __fadd_rn(a0, a1));
      t3 = __fadd_rn(t3, __shfl_xor_sync(0xFFFFFFFFu, t3, 4));
      t3 = __fadd_rn(t3, __shfl_xor_sync(0xFFFFFFFFu, t3, 2));
      t3 = __fadd_rn(t3, __shfl_xor_sync(0xFFFFFFFFu, t3, 1));
      r = t3;
    } else if (a.order == kOrderAvx2) {
      float a0 = 0.f, a1 = 0.f;
      for (int i = 0; i < pd; i += 16) {
        const float x0 = __ldg(&x[i + j]), x1 = __ldg(&x[i + 8 + j]);
        if (l2) {
          const float d0 = __fsub_rn(q_s[i + j], x0), d1 = __fsub_rn(q_s[i + 8 + j], x1);
          a0 = __fmaf_rn(d0, d0, a0);
          a1 = __fmaf_rn(d1, d1, a1);
        } else {
          a0 = __fmaf_rn(q_s[i + j], x0, a0);
          a1 = __fmaf_rn(q_s[i + 8 + j], x1, a1);
        }
      }
      float v = __fadd_rn(a0, a1);                               // v[j]
      v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));      // s[j] = v[j] + v[j+4]
      v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));      // s0+s1, s2+s3
      v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
      r = v;
    } else {
      float s = 0.f;
      if (j == 0) {
        for (int e = 0; e < pd; ++e) {
          const float xv = __ldg(&x[e]);
          if (l2) {
            const float d = __fsub_rn(q_s[e], xv);
            s = __fadd_rn(s, __fmul_rn(d, d));
          } else {
            s = __fadd_rn(s, __fmul_rn(q_s[e], xv));
          }
        }
      }
      r = __shfl_sync(0xFFFFFFFFu, s, threadIdx.x & 24);
    }
  } else {
    const uint8_t* c = a.codes + static_cast<size_t>(row) * pd;
    if (a.order == kOrderAvx512 || a.order == kOrderAvx2) {
      float a0 = 0.f, a1 = 0.f;  // avx512: acc[j], acc[j+8]; avx2: acc0[j], acc1[j]
      for (int i = 0; i < pd; i += 16) {
        const int e0 = i + j, e1 = i + 8 + j;
        const float x0 = __fmaf_rn(static_cast<float>(c[e0]), a.scale[e0], a.vmin[e0]);
        const float x1 = __fmaf_rn(static_cast<float>(c[e1]), a.scale[e1], a.vmin[e1]);
        if (l2) {
          const float d0 = __fsub_rn(q_s[e0], x0), d1 = __fsub_rn(q_s[e1], x1);
          a0 = __fmaf_rn(d0, d0, a0);
          a1 = __fmaf_rn(d1, d1, a1);
        } else {
          a0 = __fmaf_rn(q_s[e0], x0, a0);
          a1 = __fmaf_rn(q_s[e1], x1, a1);
        }
      }
      float v = __fadd_rn(a0, a1);
      if (a.order == kOrderAvx512) {
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
      } else {
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
      }
      r = v;
    } else {
      float s = 0.f;
      if (j == 0) {
        for (int e = 0; e < pd; ++e) {
          const float xv = __fadd_rn(a.vmin[e], __fmul_rn(static_cast<float>(c[e]), a.scale[e]));
          if (l2) {
            const float d = __fsub_rn(q_s[e], xv);
            s = __fadd_rn(s, __fmul_rn(d, d));
          } else {
            s = __fadd_rn(s, __fmul_rn(q_s[e], xv));
          }
        }
      }
      r = __shfl_sync(0xFFFFFFFFu, s, threadIdx.x & 24);
    }
  }
  return l2 ? r : -r;
}

// pd == 128, AVX-512 order: 8 rows per pass, packed pairs (warp_ops.cuh).
__device__ __forceinline__ void dists_of_128(const HnswArgs& a, const float* q_s, const uint32_t* ids, float* d,
                                             int n, bool l2) {
  warp_dists128_f32(a.rows, q_s, n, l2, [&](int i) { return ids[i]; }, [&](int i, float v) { d[i] = v; });
}
__device__ __forceinline__ void sq8_dists_of_128(const HnswArgs& a, const float* q_s, const uint32_t* ids, float* d,
                                                 int n, bool l2) {
  warp_dists128_sq8(a.codes, q_s, a.vmin, a.scale, n, l2, [&](int i) { return ids[i]; },
                    [&](int i, float v) { d[i] = v; });
}

// Distances of ids[0..n) (n <= 32) into d[0..n), four rows per pass.
template <bool kSq8>
__device__ void dists_of(const HnswArgs& a, const float* q_s, const uint32_t* ids, float* d, int n,
                         bool l2) {
  if (a.pd == 128 && a.order == kOrderAvx512) {
    if (kSq8) sq8_dists_of_128(a, q_s, ids, d, n, l2);
    else dists_of_128(a, q_s, ids, d, n, l2);
    return;
  }
  const int lane = threadIdx.x & 31, g = lane >> 3;
  for (int i = 0; i < n; i += 4) {
    const int my = i + g;
    const uint32_t row = ids[my < n ? my : i];
    const float v = group_dist<kSq8>(a, q_s, row, l2);
    if ((lane & 7) == 0 && my < n) d[my] = v;
  }
  __syncwarp();
}

// Number of elements of the ascending arr[b..b+n) strictly below key (warp-cooperative).
__device__ __forceinline__ int count_below(const uint64_t* arr, int b, int n, uint64_t key) {
  const int lane = threadIdx.x & 31;
  int c = 0;
  for (int i = lane; i < n; i += 32) c += arr[b + i] < key ? 1 : 0;
  return __reduce_add_sync(0xFFFFFFFFu, c);
}

// Inserts key into the ascending arr[b..b+n) keeping order; arr must have room at b + n.
__device__ __forceinline__ void insert_sorted(uint64_t* arr, int b, int n, uint64_t key) {
  const int lane = threadIdx.x & 31;
  const int p = count_below(arr, b, n, key);
  // Shift arr[b+p .. b+n) up by one, top chunk first.
  for (int hi = n; hi > p; hi -= 32) {
    const int i = hi - 1 - lane;
    uint64_t v = 0;
    const bool mv = i >= p;
    if (mv) v = arr[b + i];
    __syncwarp();
    if (mv) arr[b + i + 1] = v;
    __syncwarp();
  }
  if (lane == 0) arr[b + p] = key;
  __syncwarp();
}

// ------------------------------------------------------------------ pooled candidates
//
// Large walks (a filtered walk keeps every reached node as a candidate until it holds ef allowed
// rows) keep the kPoolFront smallest candidates sorted in shared memory and the rest unsorted in a
// per-query pool in global memory, with every pool key above every front key (pmin = the pool's
// smallest key). The front's head is then the least candidate overall: the pop order of the
// reference's heap. The visited set is a per-query bitmap in global memory.

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// Merges one candidate key per lane (where want) into the candidates. Returns false when the pool
// is full.
// Removes the dead slots (~0: moved to the front or pruned) from the pool.
__device__ void pool_compact(uint64_t* pool, int& npool) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  int nkeep = 0;
  // Four chunks of 32 are read before any is written (loads in flight together); a chunk's
  // entries move to nkeep <= its own start, never ahead of unread entries.
  for (int base = 0; base < npool; base += 128) {
    uint64_t kk[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + 32 * u + lane;
      kk[u] = i < npool ? pool[i] : ~0ull;
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const bool kp = kk[u] != ~0ull;
      const uint32_t mk = __ballot_sync(0xFFFFFFFFu, kp);
      if (kp) pool[nkeep + __popc(mk & lt)] = kk[u];
      nkeep += __popc(mk);
    }
    __syncwarp();
  }
  npool = nkeep;
}

__device__ bool pool_merge(uint64_t key, bool want, uint64_t* front, int& chead, int& ncand, uint64_t* pool,
                           int& npool, int pool_cap, uint64_t& pmin) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const bool to_pool = want && key >= pmin;
  const bool to_front = want && key < pmin;
  const uint32_t mp = __ballot_sync(0xFFFFFFFFu, to_pool);
  const int np = __popc(mp);
  if (npool + np + 32 > pool_cap) pool_compact(pool, npool);
  if (npool + np + 32 > pool_cap) return false;
  if (to_pool) pool[npool + __popc(mp & lt)] = key;
  npool += np;
  const uint32_t mf = __ballot_sync(0xFFFFFFFFu, to_front);
  if (mf == 0) return true;
  // Merge path: only the m <= 32 new keys are sorted; every key's place in the merged order is
  // its index in its own sorted run plus the number of keys of the other run below it (keys are
  // unique: a fresh node's id is in neither run). The front occupies [chead, chead + ncand) within
  // [0, kPoolFront), so front[kPoolFront, kPoolFront + 32) holds the sorted new keys for searching.
  uint64_t b[1] = {to_front ? key : ~0ull};
  warp_sort<1>(b);
  uint64_t* bs = front + kPoolFront;
  bs[lane] = b[0];
  uint64_t av[3];
#pragma unroll
  for (int e = 0; e < 3; ++e) {
    const int i = e * 32 + lane;
    av[e] = i < ncand ? front[chead + i] : ~0ull;
  }
  __syncwarp();
  const int m = __popc(mf);
  int pos_b = 0;
  if (lane < m) {  // new key: its rank plus the front keys below it
    int lo = 0, hi = ncand;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (front[chead + mid] < b[0]) lo = mid + 1; else hi = mid;
    }
    pos_b = lane + lo;
  }
  int pos_a[3];
#pragma unroll
  for (int e = 0; e < 3; ++e) {  // front key: its rank plus the new keys below it
    int lo = 0, hi = m;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (bs[mid] < av[e]) lo = mid + 1; else hi = mid;
    }
    pos_a[e] = e * 32 + lane + lo;
  }
  __syncwarp();
  const int total = ncand + m;
  const int keep = total < kPoolFront ? total : kPoolFront;
  const int nover = total - keep;  // <= 32: room was reserved above
  uint64_t over_min = ~0ull;
  auto place = [&](int pos, uint64_t v) {
    if (pos < keep) {
      front[pos] = v;
    } else {
      pool[npool + (pos - keep)] = v;
      over_min = v < over_min ? v : over_min;
    }
  };
  if (lane < m) place(pos_b, b[0]);
#pragma unroll
  for (int e = 0; e < 3; ++e)
    if (e * 32 + lane < ncand) place(pos_a[e], av[e]);
  if (nover > 0) pmin = warp_min_u64(over_min);  // overflow keys lie below the old pmin
  npool += nover;
  chead = 0;
  ncand = keep;
  __syncwarp();
  return true;
}

// Refills the empty front with every live pool key at or below a threshold (live: not dead and
// not prunable, i.e. nres < ef or dist <= lower). Any threshold keeps every front key below every
// pool key; the threshold is picked so the keys fit in the front: pass 1 finds the live minimum,
// pass 2 counts live keys under eight thresholds min + delta * 4^j, pass 3 moves the keys under
// the largest one that fits (their pool slots become dead, ~0) and finds the new pool minimum.
// delta adapts from refill to refill. When even the smallest threshold holds more keys than fit
// (many equal distances), an exact radix select over the 64-bit keys picks kPoolRefill keys.
__device__ void pool_refill(uint64_t* front, int& chead, int& ncand, uint64_t* pool, int& npool, uint64_t& pmin,
                            uint32_t* hist, bool prune, float lower, float& delta) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  auto live = [&](uint64_t k) { return k != ~0ull && (!prune || !(neighbor_dist(k) > lower)); };
  // Every pool scan reads four chunks of 32 keys per step, so a lane has four loads in flight.
  auto load4 = [&](int base, uint64_t (&kk)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + 32 * u + lane;
      kk[u] = i < npool ? pool[i] : ~0ull;
    }
  };
  uint64_t m = ~0ull;
  int nlive = 0;
  for (int base = 0; base < npool; base += 128) {
    uint64_t kk[4];
    load4(base, kk);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (live(kk[u])) {
        ++nlive;
        m = kk[u] < m ? kk[u] : m;
      }
  }
  m = warp_min_u64(m);
  nlive = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(nlive)));
  chead = 0;
  ncand = 0;
  if (nlive == 0) {
    npool = 0;
    pmin = ~0ull;
    return;
  }
  uint64_t thr = ~0ull;  // move live keys <= thr
  if (nlive > kPoolFront) {
    const float base = neighbor_dist(m);
    bool found = false;
    for (int attempt = 0; attempt < 4 && !found; ++attempt) {
      int c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int b0 = 0; b0 < npool; b0 += 128) {
        uint64_t kk[4];
        load4(b0, kk);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (!live(kk[u])) continue;
          const float d = neighbor_dist(kk[u]);
          float t = base + delta;
#pragma unroll
          for (int j = 0; j < 8; ++j, t = base + (t - base) * 4.f) c[j] += d <= t ? 1 : 0;
        }
      }
      int best = -1;
      float t = base + delta;
#pragma unroll
      for (int j = 0; j < 8; ++j, t = base + (t - base) * 4.f) {
        const int cj = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c[j])));
        if (cj <= kPoolFront) {
          best = j;
          thr = (static_cast<uint64_t>(float_key(t)) << 32) | 0xFFFFFFFFull;
        }
        if (j == 0 && cj > kPoolFront) break;
      }
      if (best >= 0) {
        found = true;
        if (best == 7) delta *= 16.f;  // thresholds too tight: widen next time
        if (best < 3) delta *= 0.25f;
      } else {
        delta *= 1.0f / 64.f;  // even the smallest threshold holds too many keys
      }
    }
    if (!found) {
      // Exact: the kPoolRefill-th smallest live key by a 4-bit radix select.
      uint64_t prefix = 0, pmask = 0;
      int need = kPoolRefill;
      for (int shift = 60; shift >= 0; shift -= 4) {
        if (lane < 16) hist[lane] = 0;
        __syncwarp();
        for (int i = lane; i < npool; i += 32) {
          const uint64_t k = pool[i];
          if (live(k) && (k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 15ull], 1u);
        }
        __syncwarp();
        const int cc = lane < 16 ? static_cast<int>(hist[lane]) : 0;
        int incl = cc;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
          const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += v;
        }
        const uint32_t hit = __ballot_sync(0xFFFFFFFFu, lane < 16 && incl >= need);
        if (hit == 0) {  // cannot happen for a consistent pool
          prefix = m;
          break;
        }
        const int d = __ffs(hit) - 1;
        const int before = __shfl_sync(0xFFFFFFFFu, incl - cc, d);
        prefix |= static_cast<uint64_t>(d) << shift;
        pmask |= 15ull << shift;
        need -= before;
        __syncwarp();
      }
      thr = prefix;  // keys are unique: exactly kPoolRefill live keys are <= thr
    }
  }
  int nsel = 0;
  uint64_t kmin = ~0ull;
  bool any_left = false;
  for (int b0 = 0; b0 < npool; b0 += 128) {
    uint64_t kk[4];
    load4(b0, kk);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = b0 + 32 * u + lane;
      const uint64_t k = kk[u];
      const bool lv = i < npool && live(k);
      const bool sel = lv && k <= thr;
      const uint32_t ms = __ballot_sync(0xFFFFFFFFu, sel);
      if (sel) {
        const int at = nsel + __popc(ms & lt);
        if (at < 128) front[at] = k;
      }
      if (i < npool && !lv && k != ~0ull) pool[i] = ~0ull;  // pruned: dead
      if (sel) pool[i] = ~0ull;                              // moved to the front
      if (lv && !sel) {
        kmin = k < kmin ? k : kmin;
        any_left = true;
      }
      nsel += __popc(ms);
    }
  }
  __syncwarp();
  kmin = warp_min_u64(kmin);
  any_left = __any_sync(0xFFFFFFFFu, any_left);
  if (!any_left) npool = 0;  // every slot is dead
  pmin = any_left ? kmin : ~0ull;
  nsel = nsel < kPoolFront ? nsel : kPoolFront;
  uint64_t x[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int i = e * 32 + lane;
    x[e] = i < nsel ? front[i] : ~0ull;
  }
  __syncwarp();
  warp_sort<4>(x);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int i = e * 32 + lane;
    if (i < nsel) front[i] = x[e];
  }
  __syncwarp();
  ncand = nsel;
}

template <bool kSq8>
__global__ void __launch_bounds__(kHnswWarps * 32, 6) hnsw_search_kernel(const HnswArgs a0) {
  extern __shared__ __align__(16) uint8_t hsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = blockIdx.x * (blockDim.x >> 5) + warp;
  if (q >= a0.nq) return;
  // The walk's graph: the launch's index, or in multi-segment mode this warp's item's segment.
  HnswArgs a = a0;
  const float* qsrc = a0.queries + static_cast<size_t>(q) * a0.pd;
  uint64_t slot = static_cast<uint64_t>(q);
  uint32_t need = 0;
  if (a0.segs != nullptr) {
    const HnswItem it = a0.items[q];
    const HnswSegment sg = a0.segs[it.seg];
    a.rows = sg.rows;
    a.codes = sg.codes;
    a.vmin = sg.vmin;
    a.scale = sg.scale;
    a.links0 = sg.links0;
    a.upper = sg.upper;
    a.upper_off = sg.upper_off;
    a.level = sg.level;
    a.n = sg.n;
    a.entry = sg.entry;
    a.max_level = sg.max_level;
    a.allow = it.allow;
    qsrc = a0.queries + static_cast<size_t>(it.query) * a0.pd;
    slot = it.slot;
    need = it.need;
  }
  const int pd = a.pd;
  const size_t per_warp = HnswWarpSmemBytes(pd, a.hash_bits, a.ef, a.cand_cap);
  uint8_t* base = hsm + warp * per_warp;
  WarpSmem s;
  s.q = reinterpret_cast<float*>(base);
  s.hash = reinterpret_cast<uint32_t*>(base + static_cast<size_t>(pd) * 4);
  const uint32_t hash_slots = a.hash_bits < 1 ? 2u : (1u << a.hash_bits);  // even: keeps res 8-aligned
  s.res = reinterpret_cast<uint64_t*>(s.hash + hash_slots);
  s.cand = s.res + a.ef;
  s.nb_id = reinterpret_cast<uint32_t*>(s.cand + a.cand_cap);
  s.nb_d = reinterpret_cast<float*>(s.nb_id + 32);
  for (int i = lane; i < pd; i += 32) s.q[i] = qsrc[i];
  for (int i = lane; i < static_cast<int>(hash_slots); i += 32) s.hash[i] = kEmpty;
  __syncwarp();
  const bool l2 = a.metric == 0;
  const uint64_t n = a.n;
  uint64_t dc = 0;
  int nres = 0;
  bool bad = false;

  if (a.max_level >= 0 && n > 0) {
    // Entry point and greedy descent over layers max_level..1.
    uint32_t cur = a.entry;
    if (lane == 0) s.nb_id[0] = cur;
    __syncwarp();
    dists_of<kSq8>(a, s.q, s.nb_id, s.nb_d, 1, l2);
    float curd = s.nb_d[0];
    dc = 1;
    for (int layer = a.max_level; layer > 0 && !bad; --layer) {
      for (int iter = 0; iter < a.step_limit; ++iter) {
        const uint32_t* ll = a.upper + a.upper_off[cur] + static_cast<size_t>(layer - 1) * (1 + a.M);
        const uint32_t cnt = ll[0];
        __syncwarp();
        if (lane < static_cast<int>(cnt)) {
          const uint32_t e = ll[1 + lane];
          // A valid graph only links nodes present on this layer (HnswGraph::check).
          const bool ok_e = e < n && a.level[e] >= layer;
          s.nb_id[lane] = ok_e ? e : 0u;
          if (!ok_e) bad = true;
        }
        bad = __any_sync(0xFFFFFFFFu, bad);
        __syncwarp();
        if (bad) {
          if (lane == 0) set_error(a.status, kDevBadIndex);
          break;
        }
        dists_of<kSq8>(a, s.q, s.nb_id, s.nb_d, static_cast<int>(cnt), l2);
        dc += cnt;
        // Strict improvements in list order end at the first occurrence of the minimum.
        float m = lane < static_cast<int>(cnt) ? s.nb_d[lane] : INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fminf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        if (!(m < curd)) break;
        const uint32_t at = __ballot_sync(0xFFFFFFFFu, lane < static_cast<int>(cnt) && s.nb_d[lane] == m);
        cur = s.nb_id[__ffs(at) - 1];
        curd = m;
      }
    }

    // Layer 0: ef-beam.
    const int ef = a.ef;
    const bool filtered = a.allow != nullptr;
    auto allowed = [&](uint32_t id) { return !filtered || ((a.allow[id >> 5] >> (id & 31)) & 1u); };
    if (a.pooled) {
      // Pooled walk: visited bits and overflow candidates in global memory (see pool_merge).
      uint32_t* vis = a.visited + static_cast<uint64_t>(q) * a.vwords;
      uint64_t* pool = a.pool + static_cast<uint64_t>(q) * a.pool_cap;
      uint32_t* hist = reinterpret_cast<uint32_t*>(s.cand + 128);
      int npool = 0;
      uint64_t pmin = ~0ull;
      float delta = fmaxf(fabsf(curd), 1e-3f) * 1e-3f;  // refill threshold step (adapts)
      unsigned long long c_exp = 0, c_ref = 0, c_scan = 0, c_merge = 0, c_ins = 0;
      if (lane == 0) atomicOr(&vis[cur >> 5], 1u << (cur & 31));
      float lower = INFINITY;
      int chead = 0, ncand = 0;
      if (allowed(cur)) {
        if (lane == 0) s.res[0] = pack_neighbor(curd, cur);
        nres = 1;
        lower = curd;
      }
      if (lane == 0) s.cand[0] = pack_neighbor(curd, cur);
      ncand = 1;
      __syncwarp();
      int steps = 0;
      while (!bad) {
        if (ncand == 0) {
          if (npool == 0) break;
          // Candidates beyond a full result set's worst can never be expanded (lower only falls).
          ++c_ref;
          c_scan += static_cast<unsigned long long>(npool);
          pool_refill(s.cand, chead, ncand, pool, npool, pmin, hist, nres >= ef, lower, delta);
          if (ncand == 0) break;
        }
        const uint64_t c = s.cand[chead];
        const float cd = neighbor_dist(c);
        if (cd > lower && (!filtered || nres >= ef)) break;
        ++chead;
        --ncand;
        ++c_exp;
        if (++steps > a.step_limit) {
          if (lane == 0) set_error(a.status, kDevStepLimit);
          bad = true;
          break;
        }
        const uint32_t cid = neighbor_id(c);
        const uint32_t* ll = a.links0 + static_cast<size_t>(cid) * (1 + a.M0);
        // The list's count and its slots load together (a block always holds M0 slots).
        const uint32_t cnt = ll[0];
        const uint32_t e_raw = lane < static_cast<int>(a.M0) ? ll[1 + lane] : 0u;
        // The next expansion most often takes the current front head: its link block starts
        // towards L2 now and lands while this expansion runs.
        if (ncand > 0 && lane < 2)
          prefetch_l2(a.links0 + static_cast<size_t>(neighbor_id(s.cand[chead])) * (1 + a.M0) + 32 * lane);
        uint32_t e = 0;
        bool fresh = false, al = false;
        if (lane < static_cast<int>(cnt)) {
          e = e_raw;
          if (e >= n) {
            bad = true;
          } else {
            // Unfiltered walks: the neighbour's vector starts towards L2 beside its visited mark,
            // so the distance pass below finds it there (a visited neighbour's vector is fetched
            // for nothing). Filtered walks revisit most neighbours, so they skip this.
            if (!filtered) {
              if (kSq8) {
                const uint8_t* cp = a.codes + static_cast<size_t>(e) * pd;
                for (int o = 0; o < pd; o += 128) prefetch_l2(cp + o);
              } else {
                const float* rp = a.rows + static_cast<size_t>(e) * pd;
                for (int o = 0; o < pd; o += 32) prefetch_l2(rp + o);
              }
            }
            const uint32_t bit = 1u << (e & 31);
            fresh = (atomicOr(&vis[e >> 5], bit) & bit) == 0u;
            al = allowed(e);  // the filter bit loads beside the visited mark
          }
        }
        if (__any_sync(0xFFFFFFFFu, bad)) {
          if (lane == 0) set_error(a.status, kDevBadIndex);
          bad = true;
          break;
        }
        const uint32_t fm = __ballot_sync(0xFFFFFFFFu, fresh);
        const int nf = __popc(fm);
        if (fresh) s.nb_id[__popc(fm & ((1u << lane) - 1u))] = e;
        // Filtered walks: the fresh neighbours' vectors start towards L2 together now, so the
        // distance passes below (8 rows each) wait on one HBM round trip, not one per pass.
        if (filtered && fresh) {
          if (kSq8) {
            const uint8_t* cp = a.codes + static_cast<size_t>(e) * pd;
            for (int o = 0; o < pd; o += 128) prefetch_l2(cp + o);
          } else {
            const float* rp = a.rows + static_cast<size_t>(e) * pd;
            for (int o = 0; o < pd; o += 32) prefetch_l2(rp + o);
          }
        }
        __syncwarp();
        // The filter bits in the compacted (list) order of the fresh neighbours.
        const int src = lane < nf ? static_cast<int>(__fns(fm, 0, lane + 1)) : 0;
        const int al_c = __shfl_sync(0xFFFFFFFFu, al ? 1 : 0, src);
        const uint32_t amask = __ballot_sync(0xFFFFFFFFu, lane < nf && al_c != 0);
        dists_of<kSq8>(a, s.q, s.nb_id, s.nb_d, nf, l2);
        dc += static_cast<uint64_t>(nf);
        // Result updates in list order decide which neighbours become candidates; the candidates
        // themselves are merged afterwards (their order of insertion does not matter).
        uint64_t mykey = ~0ull;
        bool mywant = false;
        auto consider = [&](int i) {
          const uint32_t id = s.nb_id[i];
          const float de = s.nb_d[i];
          if (nres < ef || de < lower) {
            const uint64_t key = pack_neighbor(de, id);
            if (lane == i) {
              mykey = key;
              mywant = true;
            }
            if ((amask >> i) & 1u) {
              ++c_ins;
              if (nres < ef) {
                insert_sorted(s.res, 0, nres, key);
                ++nres;
              } else if (key < s.res[ef - 1]) {
                __syncwarp();
                insert_sorted(s.res, 0, ef - 1, key);
              }
              lower = neighbor_dist(s.res[nres - 1]);
            }
          }
        };
        int i0 = 0;
        for (; i0 < nf && nres < ef; ++i0) consider(i0);
        if (i0 < nf) {
          // The result set is full: `lower` can only fall from here, so a neighbour at or beyond
          // it now is refused at its turn too. Only the others are taken in list order.
          uint32_t maybe = __ballot_sync(0xFFFFFFFFu, lane >= i0 && lane < nf && s.nb_d[lane] < lower);
          while (maybe != 0u) {
            consider(__ffs(maybe) - 1);
            maybe &= maybe - 1u;
          }
        }
        c_merge += __any_sync(0xFFFFFFFFu, mywant && mykey < pmin) ? 1 : 0;
        if (!pool_merge(mykey, mywant, s.cand, chead, ncand, pool, npool, a.pool_cap, pmin)) {
          if (lane == 0) set_error(a.status, kDevCandOverflow);
          bad = true;
          break;
        }
      }
      if (lane == 0 && a0.counters != nullptr) {
        atomicAdd(&a0.counters[0], 1ull);
        atomicAdd(&a0.counters[1], c_exp);
        atomicAdd(&a0.counters[2], c_ref);
        atomicAdd(&a0.counters[3], c_scan);
        atomicAdd(&a0.counters[4], c_merge);
        atomicAdd(&a0.counters[5], c_ins);
        atomicMax(&a0.counters[6], c_exp);
      }
    } else {
      bool full = false;
      if (lane == 0) visit(s.hash, a.hash_bits, cur, &full);
      float lower = INFINITY;
      int chead = 0, ncand = 0;
      if (allowed(cur)) {
        if (lane == 0) s.res[0] = pack_neighbor(curd, cur);
        nres = 1;
        lower = curd;
      }
      if (lane == 0) s.cand[0] = pack_neighbor(curd, cur);
      ncand = 1;
      __syncwarp();
      int steps = 0;
      while (ncand > 0 && !bad) {
        const uint64_t c = s.cand[chead];
        const float cd = neighbor_dist(c);
        if (cd > lower && (!filtered || nres >= ef)) break;
        ++chead;
        --ncand;
        if (++steps > a.step_limit) {
          if (lane == 0) set_error(a.status, kDevStepLimit);
          bad = true;
          break;
        }
        const uint32_t cid = neighbor_id(c);
        const uint32_t* ll = a.links0 + static_cast<size_t>(cid) * (1 + a.M0);
        const uint32_t cnt = ll[0];
        uint32_t e = 0;
        bool fresh = false;
        if (lane < static_cast<int>(cnt)) {
          e = ll[1 + lane];
          if (e >= n) {
            bad = true;
          } else {
            fresh = visit(s.hash, a.hash_bits, e, &full);
          }
        }
        const bool any_full = __any_sync(0xFFFFFFFFu, full);
        if (__any_sync(0xFFFFFFFFu, bad || full)) {
          if (lane == 0) set_error(a.status, any_full ? kDevOverflow : kDevBadIndex);
          bad = true;
          break;
        }
        const uint32_t fm = __ballot_sync(0xFFFFFFFFu, fresh);
        const int nf = __popc(fm);
        if (fresh) s.nb_id[__popc(fm & ((1u << lane) - 1u))] = e;
        __syncwarp();
        // The filter bits of all fresh neighbours at once (one load per lane, not one per step).
        const uint32_t amask = __ballot_sync(0xFFFFFFFFu, lane < nf && allowed(s.nb_id[lane]));
        dists_of<kSq8>(a, s.q, s.nb_id, s.nb_d, nf, l2);
        dc += static_cast<uint64_t>(nf);
        // Heap updates in list order (the fresh neighbours keep their list order).
        for (int i = 0; i < nf; ++i) {
          const uint32_t id = s.nb_id[i];
          const float de = s.nb_d[i];
          if (nres < ef || de < lower) {
            const uint64_t key = pack_neighbor(de, id);
            if (chead + ncand >= a.cand_cap) {
              // Compact to the front; if still full, drop the farthest candidate when it can never
              // be expanded again (results full and it lies beyond the current worst result).
              for (int k0 = 0; k0 < ncand; k0 += 32) {
                const int k = k0 + lane;
                uint64_t v = 0;
                if (k < ncand) v = s.cand[chead + k];
                __syncwarp();
                if (k < ncand) s.cand[k] = v;
                __syncwarp();
              }
              chead = 0;
              if (ncand >= a.cand_cap) {
                if (nres >= ef && neighbor_dist(s.cand[ncand - 1]) > lower) {
                  --ncand;
                } else {
                  if (lane == 0) set_error(a.status, kDevCandOverflow);
                  bad = true;
                  break;
                }
              }
            }
            insert_sorted(s.cand, chead, ncand, key);
            ++ncand;
            if ((amask >> i) & 1u) {
              if (nres < ef) {
                insert_sorted(s.res, 0, nres, key);
                ++nres;
              } else {
                // Push then evict the greatest: only changes anything when key is below the max.
                if (key < s.res[ef - 1]) {
                  __syncwarp();
                  insert_sorted(s.res, 0, ef - 1, key);
                }
              }
              lower = neighbor_dist(s.res[nres - 1]);
            }
          }
        }
      }
    }
  }

  // Output: the k best results; HNSW-SQ8 re-ranks the best `depth` on fp32 rows first.
  int nout = nres < a.k_graph ? nres : a.k_graph;
  if (!bad && kSq8 && a.depth > 0 && nout > 0) {
    // Rerank (src/index/index.cc:89-95): exact fp32 distances of the graph's best candidates,
    // written back in place over res[0, nout) (nout <= k_graph <= ef slots; the candidate array
    // of a pooled walk is only the sorted front, shorter than a deep re-rank), then sorted there.
    for (int i = 0; i < nout; i += 4) {
      uint32_t r[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = neighbor_id(s.res[i + c < nout ? i + c : i]);
      float d[4];
      if (a.order == kOrderAvx512 && pd <= 8 * 32 + 16) {
        warp_exact_dist4_avx512<8>(s.q, a.rows, r, nout - i, pd, l2, d);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          d[c] = warp_exact_dist(s.q, a.rows + static_cast<size_t>(r[c]) * pd, pd, l2, a.order);
      }
      __syncwarp();
      if (lane < 4 && i + lane < nout) {
        float dl = d[0];
        uint32_t rl = r[0];
#pragma unroll
        for (int c = 1; c < 4; ++c) {
          dl = lane == c ? d[c] : dl;
          rl = lane == c ? r[c] : rl;
        }
        s.res[i + lane] = pack_neighbor(dl, rl);
      }
      __syncwarp();
    }
    dc += static_cast<uint64_t>(nout);
    // Insertion sort of res[0, nout) in place: res[0, i) is sorted, res[i] is inserted into it.
    for (int i = 1; i < nout; ++i) {
      const uint64_t key = s.res[i];
      __syncwarp();
      insert_sorted(s.res, 0, i, key);
    }
  }
  const int kout = a.k;
  if (a0.segs != nullptr) {
    for (int i = lane; i < kout; i += 32)
      a0.out_keys[slot * kout + i] = (!bad && i < nout) ? s.res[i] : ~0ull;
    if (lane == 0) {
      if (a0.out_dc != nullptr) a0.out_dc[slot] = dc;
      if (a0.out_short != nullptr) a0.out_short[slot] = (!bad && static_cast<uint32_t>(nout) < need) ? 1 : 0;
    }
    return;
  }
  for (int i = lane; i < kout; i += 32) {
    const size_t o = static_cast<size_t>(q) * kout + i;
    if (!bad && i < nout) {
      a.out_dist[o] = neighbor_dist(s.res[i]);
      a.out_row[o] = neighbor_id(s.res[i]);
    } else {
      a.out_dist[o] = INFINITY;
      a.out_row[o] = UINT32_MAX;
    }
  }
  if (lane == 0 && a.out_dc != nullptr) a.out_dc[q] = dc;
}

}  // namespace

cudaError_t LaunchHnswSearch(const HnswArgs& a, cudaStream_t stream) {
  const int warps = a.warps >= 1 && a.warps <= kHnswWarps ? a.warps : kHnswWarps;
  const size_t smem = warps * HnswWarpSmemBytes(a.pd, a.hash_bits, a.ef, a.cand_cap);
  const int blocks = (a.nq + warps - 1) / warps;
  cudaError_t e;
  if (a.codes != nullptr) {
    e = cudaFuncSetAttribute(hnsw_search_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    NoteLaunch();
    hnsw_search_kernel<true><<<blocks, warps * 32, smem, stream>>>(a);
  } else {
    e = cudaFuncSetAttribute(hnsw_search_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    NoteLaunch();
    hnsw_search_kernel<false><<<blocks, warps * 32, smem, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace vdbgpu
