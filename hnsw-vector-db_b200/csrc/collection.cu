// Kernels of the multi-segment read path; the interface and the reference functions each one
// follows are listed in collection.cuh.
#include <cmath>

#include "collection.cuh"
#include "common.cuh"
#include "warp_ops.cuh"

namespace vdbgpu {
namespace {

// ------------------------------------------------------------------------------------ queries

// PrepareQuery (src/engine/collection_impl.cc:1023-1034) for one query per thread: copy into a
// zero-padded row, reject non-finite values, and for cosine NormalizeVector
// (src/util/dataset.cc:33-40): a sequential double sum of double products, inv = float(1/sqrt),
// x * inv in float. qstatus: 0 ok, 1 non-finite value, 2 zero norm.
__global__ void prepare_queries_kernel(const float* __restrict__ in, const uint32_t* __restrict__ perm,
                                       uint64_t nq, uint32_t dim, uint32_t pd, int cosine,
                                       float* __restrict__ out, int* __restrict__ qstatus) {
  const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  if (i >= nq) return;
  const uint64_t src = perm != nullptr ? perm[i] : i;
  const float* v = in + src * dim;
  float* o = out + i * pd;
  int st = 0;
  double norm = 0.0;
  for (uint32_t j = 0; j < dim; ++j) {
    const float x = v[j];
    if (!isfinite(x)) st = 1;
    o[j] = x;
    const double xd = static_cast<double>(x);
    norm = __dadd_rn(norm, __dmul_rn(xd, xd));
  }
  for (uint32_t j = dim; j < pd; ++j) o[j] = 0.f;
  if (st == 0 && cosine) {
    if (!(norm > 0.0) || !isfinite(norm)) {
      st = 2;
    } else {
      const float inv = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(norm)));
      for (uint32_t j = 0; j < dim; ++j) o[j] = __fmul_rn(o[j], inv);
    }
  }
  qstatus[i] = st;
}

// --------------------------------------------------------------------------------- leaf bitmaps

// Numeric leaves as per-row predicates: present && lo <(=) x <(=) hi, or present && x in set.
// SegmentColumns::NumericIndex::Range (columns.cc:145-168) selects the present rows whose value
// lies in the same interval by binary search over the sorted values; for finite and infinite
// values the two sets are equal. One warp builds 32 consecutive words, reading the values
// coalesced (lane = row within a word).
__global__ void leaf_range_kernel(const RangeTask* __restrict__ tasks) {
  const RangeTask t = tasks[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t w0 = (blockIdx.x * (blockDim.x >> 5) + warp) * 32u;
  if (w0 >= t.words) return;
  uint32_t mine = 0;
  for (int i = 0; i < 32; ++i) {
    const uint32_t w = w0 + i;
    if (w >= t.words) break;
    const uint32_t pw = __ldg(&t.present[w]);
    bool hit = false;
    if ((pw >> lane) & 1u) {
      const double x = __ldg(&t.values[static_cast<uint64_t>(w) * 32 + lane]);
      if (t.set != nullptr) {
        for (int s = 0; s < t.nset; ++s) hit |= x == __ldg(&t.set[s]);
      } else {
        const bool lo_ok = t.lo_incl ? x >= t.lo : x > t.lo;
        const bool hi_ok = t.hi_incl ? x <= t.hi : x < t.hi;
        hit = lo_ok && hi_ok;
      }
    }
    const uint32_t word = __ballot_sync(0xFFFFFFFFu, hit);
    if (lane == i) mine = word;
  }
  if (w0 + lane < t.words) t.out[w0 + lane] = mine;
}

__global__ void posting_scatter_kernel(const ScatterTask* __restrict__ tasks) {
  const ScatterTask t = tasks[blockIdx.x];
  for (uint32_t i = threadIdx.x; i < t.count; i += blockDim.x) {
    const uint32_t r = __ldg(&t.rows[i]);
    atomicOr(&t.out[r >> 5], 1u << (r & 31));
  }
}

// ---------------------------------------------------------------------------- filter programs

__device__ __forceinline__ uint32_t block_sum_256(uint32_t v, uint32_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xFFFFFFFFu, v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  uint32_t s = 0;
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0u;
    s = __reduce_add_sync(0xFFFFFFFFu, s);
  }
  return s;  // valid in thread 0
}

// Evaluates each (filter, segment) program over one chunk of words: a postfix program of pushes
// of leaf bitmaps and And / Or / AndNot / Not, minus deleted rows. Writes the result words, the
// chunk's match count and adds it to the segment's total.
__global__ void __launch_bounds__(256) filter_program_kernel(const ProgramTask* __restrict__ tasks,
                                                             int* status) {
  __shared__ uint32_t red[8];
  const ProgramTask t = tasks[blockIdx.y];
  const uint32_t chunk0 = blockIdx.x * kProgChunkWords;
  if (chunk0 >= t.words) return;
  uint32_t cnt = 0;
  bool bad = false;
  for (int j = 0; j < kProgChunkWords / 256; ++j) {
    const uint32_t w = chunk0 + j * 256 + threadIdx.x;
    if (w >= t.words) break;
    uint32_t stack[kProgStack];
    int sp = 0;
    for (int p = 0; p < t.nprog; ++p) {
      const int op = t.prog[p].op;
      if (op == kProgPush || op == kProgZero) {
        if (sp >= kProgStack) {
          bad = true;
          break;
        }
        stack[sp++] = op == kProgPush ? __ldg(&t.prog[p].bits[w]) : 0u;
      } else if (op == kProgNot) {
        if (sp < 1) {
          bad = true;
          break;
        }
        stack[sp - 1] = __ldg(&t.all[w]) & ~stack[sp - 1];
      } else {
        if (sp < 2) {
          bad = true;
          break;
        }
        const uint32_t b = stack[--sp];
        if (op == kProgAnd) stack[sp - 1] &= b;
        else if (op == kProgOr) stack[sp - 1] |= b;
        else stack[sp - 1] &= ~b;
      }
    }
    uint32_t r = (!bad && sp == 1) ? stack[0] : 0u;
    if (t.deletes != nullptr) r &= ~__ldg(&t.deletes[w]);
    if (t.out != nullptr) t.out[w] = r;
    cnt += __popc(r);
  }
  if (bad && status != nullptr) atomicCAS(status, 0, kDevBadIndex);
  const uint32_t total = block_sum_256(cnt, red);
  if (threadIdx.x == 0) {
    t.chunk_counts[blockIdx.x] = total;
    if (total > 0) atomicAdd(t.matches, static_cast<unsigned long long>(total));
  }
}

// Rows of a bitmap in ascending order: each thread owns 8 consecutive words of a chunk; the
// chunk's output offset is the sum of the earlier chunks' counts.
__global__ void __launch_bounds__(256) compact_rows_kernel(const CompactTask* __restrict__ tasks) {
  __shared__ uint32_t scan[256];
  __shared__ uint32_t base_s;
  const CompactTask t = tasks[blockIdx.y];
  const uint32_t chunk0 = blockIdx.x * kProgChunkWords;
  if (chunk0 >= t.words) return;
  if (threadIdx.x == 0) {
    uint32_t b = 0;
    for (uint32_t c = 0; c < blockIdx.x; ++c) b += t.chunk_counts[c];
    base_s = b;
  }
  uint32_t words[8];
  uint32_t cnt = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t w = chunk0 + threadIdx.x * 8 + j;
    words[j] = w < t.words ? __ldg(&t.bits[w]) : 0u;
    cnt += __popc(words[j]);
  }
  scan[threadIdx.x] = cnt;
  __syncthreads();
  // Inclusive Hillis-Steele scan over 256 counts.
  for (int off = 1; off < 256; off <<= 1) {
    const uint32_t v = threadIdx.x >= off ? scan[threadIdx.x - off] : 0u;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  uint32_t pos = base_s + scan[threadIdx.x] - cnt;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t m = words[j];
    const uint32_t rbase = (chunk0 + threadIdx.x * 8 + j) * 32u;
    while (m != 0) {
      const int b = __ffs(m) - 1;
      m &= m - 1;
      t.rows_out[pos++] = rbase + b;
    }
  }
}

// ---------------------------------------------------------------------------- exact top-k

constexpr int kExactWarps = 4;
constexpr int kExactQ = 4;  // queries per warp

// Per-warp top-k state for up to kExactQ queries: an unsorted buffer of packed keys per query in
// shared memory (capacity 32 * kE), the number held, and the admission threshold (the k-th
// smallest key after the last sort; keys are unique).
template <int kE>
struct TopBuf {
  uint64_t* buf;  // kExactQ x (32 * kE)
  int cnt[kExactQ];
  uint64_t thr[kExactQ];
};

// Sorts query j's buffer and keeps its k smallest keys.
template <int kE>
__device__ __forceinline__ void topbuf_sort(TopBuf<kE>& tb, int j, int k) {
  const int lane = threadIdx.x & 31;
  uint64_t* b = tb.buf + j * 32 * kE;
  uint64_t x[kE];
#pragma unroll
  for (int e = 0; e < kE; ++e) {
    const int i = e * 32 + lane;
    x[e] = i < tb.cnt[j] ? b[i] : ~0ull;
  }
  __syncwarp();
  warp_sort<kE>(x);
#pragma unroll
  for (int e = 0; e < kE; ++e) b[e * 32 + lane] = x[e];
  __syncwarp();
  if (tb.cnt[j] >= k) {
    tb.cnt[j] = k;
    tb.thr[j] = b[k - 1];
  }
}

// Offers one candidate key per lane (valid lanes only) to query j.
template <int kE>
__device__ __forceinline__ void topbuf_offer(TopBuf<kE>& tb, int j, int k, uint64_t key, bool valid) {
  const int lane = threadIdx.x & 31;
  const bool pass = valid && key < tb.thr[j];
  const uint32_t m = __ballot_sync(0xFFFFFFFFu, pass);
  if (m == 0) return;
  const int n = __popc(m);
  if (tb.cnt[j] + n > 32 * kE) topbuf_sort<kE>(tb, j, k);
  if (pass) tb.buf[j * 32 * kE + tb.cnt[j] + __popc(m & ((1u << lane) - 1u))] = key;
  tb.cnt[j] += n;
  __syncwarp();
}

template <int kE>
__device__ void topbuf_write(TopBuf<kE>& tb, int j, int k, uint64_t* out) {
  const int lane = threadIdx.x & 31;
  topbuf_sort<kE>(tb, j, k);
  const uint64_t* b = tb.buf + j * 32 * kE;
  for (int i = lane; i < k; i += 32) out[i] = i < tb.cnt[j] ? b[i] : ~0ull;
  __syncwarp();
}

// AVX-512-order distances of 16 rows at a time against up to 4 queries. Lane l accumulates the
// l-th of the 32 partial sums (element 32t + l, FMA in t order, the 16-wide tail into lanes
// < 16), exactly as the two 16-wide accumulators of src/distance/avx512.cc:19-46. The partials of
// 16 rows are then combined by a butterfly reduce-scatter whose additions pair lanes
// (l, l^16), (l, l^8), (l, l^4), (l, l^2), (l, l^1) in the order of the single-row xor tree
// (warp_exact_dist), so every sum is bit-identical to it; afterwards lanes 2r and 2r+1 hold
// row r's distance.
template <int kT, int kE>
__device__ void exact_item_avx512(const ExactArgs& a, const ExactItem& it, const bool (&act)[kExactQ],
                                  TopBuf<kE>& tb) {
  const int lane = threadIdx.x & 31;
  const int pd = a.pd, nb = pd >> 5;
  const bool tail = (pd & 31) != 0;
  const bool l2 = a.metric == 0;
  float qv[kExactQ][kT + 1];
#pragma unroll
  for (int j = 0; j < kExactQ; ++j) {
    const float* q = a.queries + static_cast<uint64_t>(it.q0 + (j < static_cast<int>(it.nq) ? j : 0)) * pd;
#pragma unroll
    for (int t = 0; t < kT; ++t) qv[j][t] = t < nb ? q[32 * t + lane] : 0.f;
    qv[j][kT] = (tail && lane < 16) ? q[32 * nb + lane] : 0.f;
  }
  for (uint32_t base = 0; base < it.count; base += 16) {
    const uint32_t nrow = min(16u, it.count - base);
    const uint32_t rid = __ldg(&it.list[base + (lane < static_cast<int>(nrow) ? lane : 0)]);
    float acc[kExactQ][16];
#pragma unroll
    for (int j = 0; j < kExactQ; ++j)
#pragma unroll
      for (int r = 0; r < 16; ++r) acc[j][r] = 0.f;
#pragma unroll
    for (int r0 = 0; r0 < 16; r0 += 4) {
      float xv[4][kT + 1];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t id = __shfl_sync(0xFFFFFFFFu, rid, r0 + c);
        const float* x = it.rows + static_cast<uint64_t>(id) * pd;
#pragma unroll
        for (int t = 0; t < kT; ++t) xv[c][t] = t < nb ? __ldg(&x[32 * t + lane]) : 0.f;
        xv[c][kT] = (tail && lane < 16) ? __ldg(&x[32 * nb + lane]) : 0.f;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int j = 0; j < kExactQ; ++j) {
          float s = 0.f;
#pragma unroll
          for (int t = 0; t < kT; ++t) {
            if (t < nb) {
              if (l2) {
                const float d = __fsub_rn(qv[j][t], xv[c][t]);
                s = __fmaf_rn(d, d, s);
              } else {
                s = __fmaf_rn(qv[j][t], xv[c][t], s);
              }
            }
          }
          if (tail && lane < 16) {
            if (l2) {
              const float d = __fsub_rn(qv[j][kT], xv[c][kT]);
              s = __fmaf_rn(d, d, s);
            } else {
              s = __fmaf_rn(qv[j][kT], xv[c][kT], s);
            }
          }
          acc[j][r0 + c] = s;
        }
      }
    }
    const uint32_t myrow = __shfl_sync(0xFFFFFFFFu, rid, lane >> 1);
    const bool valid = (lane & 1) == 0 && static_cast<uint32_t>(lane >> 1) < nrow;
#pragma unroll
    for (int j = 0; j < kExactQ; ++j) {
      float* v = acc[j];
      // 16 -> 8 -> 4 -> 2 -> 1 rows per lane; the kept half follows the lane bit.
#pragma unroll
      for (int s = 16, half = 8; s >= 2; s >>= 1, half >>= 1) {
        const bool up = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = up ? v[i] : v[half + i];
          const float keep = up ? v[half + i] : v[i];
          const float recv = __shfl_xor_sync(0xFFFFFFFFu, send, s);
          v[i] = __fadd_rn(keep, recv);
        }
      }
      const float sum = __fadd_rn(v[0], __shfl_xor_sync(0xFFFFFFFFu, v[0], 1));
      if (act[j]) topbuf_offer<kE>(tb, j, a.k, pack_neighbor(l2 ? sum : -sum, myrow), valid);
    }
  }
}

// Any kernel set, any padded dimension: one row at a time through warp_exact_dist, 16 rows per
// offer (the buffer admits at most 16 new keys per offer).
template <int kE>
__device__ void exact_item_generic(const ExactArgs& a, const ExactItem& it, const bool (&act)[kExactQ],
                                   TopBuf<kE>& tb) {
  const int lane = threadIdx.x & 31;
  const bool l2 = a.metric == 0;
  for (uint32_t base = 0; base < it.count; base += 16) {
    const uint32_t nrow = min(16u, it.count - base);
    const uint32_t rid = __ldg(&it.list[base + (lane < static_cast<int>(nrow) ? lane : 0)]);
    for (int j = 0; j < kExactQ; ++j) {
      if (!act[j]) continue;
      const float* q = a.queries + static_cast<uint64_t>(it.q0 + j) * a.pd;
      uint64_t mine = ~0ull;
      for (uint32_t r = 0; r < nrow; ++r) {
        const uint32_t id = __shfl_sync(0xFFFFFFFFu, rid, r);
        const float d = warp_exact_dist(q, it.rows + static_cast<uint64_t>(id) * a.pd, a.pd, l2, a.order);
        if (lane == static_cast<int>(r)) mine = pack_neighbor(d, id);
      }
      topbuf_offer<kE>(tb, j, a.k, mine, lane < static_cast<int>(nrow));
    }
  }
}

template <int kT, int kE>
__global__ void __launch_bounds__(kExactWarps * 32) exact_rows_kernel(const ExactArgs a) {
  __shared__ uint64_t bufs[kExactWarps][kExactQ * 32 * kE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int item = blockIdx.x * kExactWarps + warp;
  if (item >= a.nitems) return;
  const ExactItem it = a.items[item];
  bool act[kExactQ];
  bool any = false;
#pragma unroll
  for (int j = 0; j < kExactQ; ++j) {
    act[j] = j < static_cast<int>(it.nq) &&
             (it.only_if == nullptr || it.only_if[static_cast<uint64_t>(j) * a.dc_stride] != 0);
    any |= act[j];
  }
  if (!any) return;
  TopBuf<kE> tb;
  tb.buf = bufs[warp];
#pragma unroll
  for (int j = 0; j < kExactQ; ++j) {
    tb.cnt[j] = 0;
    tb.thr[j] = ~0ull;
  }
  if (a.order == kOrderAvx512 && a.pd <= 32 * kT + 16) {
    exact_item_avx512<kT, kE>(a, it, act, tb);
  } else {
    exact_item_generic<kE>(a, it, act, tb);
  }
#pragma unroll
  for (int j = 0; j < kExactQ; ++j) {
    if (!act[j]) continue;
    topbuf_write<kE>(tb, j, a.k, it.out + static_cast<uint64_t>(j) * a.out_stride);
    if (lane == 0 && it.dc != nullptr) it.dc[static_cast<uint64_t>(j) * a.dc_stride] += it.count;
  }
}

template <int kT, int kE>
cudaError_t LaunchExactT(const ExactArgs& a, cudaStream_t st) {
  const int blocks = (a.nitems + kExactWarps - 1) / kExactWarps;
  NoteLaunch();
  exact_rows_kernel<kT, kE><<<blocks, kExactWarps * 32, 0, st>>>(a);
  return cudaGetLastError();
}

template <int kT>
cudaError_t LaunchExactK(const ExactArgs& a, cudaStream_t st) {
  if (a.k <= 16) return LaunchExactT<kT, 1>(a, st);
  if (a.k <= 48) return LaunchExactT<kT, 2>(a, st);
  if (a.k <= 112) return LaunchExactT<kT, 4>(a, st);
  return LaunchExactT<kT, 8>(a, st);
}

// ------------------------------------------------------------------------------ pack / merge

__global__ void pack_hits_kernel(const PackItem* __restrict__ items, int k, uint64_t out_stride,
                                 uint64_t flag_stride) {
  const PackItem it = items[blockIdx.y];
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= it.nq) return;
  uint64_t* out = it.out + q * out_stride;
  uint32_t c = 0;
  for (uint32_t i = 0; i < it.kin && c < static_cast<uint32_t>(k); ++i) {
    const uint64_t o = static_cast<uint64_t>(q) * it.kin + i;
    const uint32_t r = it.row[o];
    if (r == UINT32_MAX) break;
    if (it.keep != nullptr && !((__ldg(&it.keep[r >> 5]) >> (r & 31)) & 1u)) continue;
    out[c++] = pack_neighbor(it.dist[o], r);
  }
  if (it.short_flag != nullptr) it.short_flag[q * flag_stride] = c < it.need ? 1 : 0;
  for (; c < static_cast<uint32_t>(k); ++c) out[c] = ~0ull;
}

constexpr int kMergeWarps = 4;

// Per-warp shared memory of the merge: kept ids (k), head keys (L), head positions (L).
__host__ __device__ inline size_t MergeWarpBytes(int L, int k) {
  return (static_cast<size_t>(k) * 8 + static_cast<size_t>(L) * 12 + 15) / 16 * 16;
}

// One warp per query: a k-way merge of sorted lists by (dist, part, row) that keeps the first hit
// of every external id and stops at k hits. Each list's head key sits in shared memory; lists
// never share a part, so (dist, part) orders the heads.
__global__ void __launch_bounds__(kMergeWarps * 32) merge_kernel(const MergeArgs a) {
  extern __shared__ __align__(16) uint8_t msm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t q = static_cast<uint64_t>(blockIdx.x) * kMergeWarps + warp;
  if (q >= a.nq) return;
  const int L = a.nlists, k = a.k;
  uint8_t* base = msm + static_cast<size_t>(warp) * MergeWarpBytes(L, k);
  uint64_t* kept = reinterpret_cast<uint64_t*>(base);  // kept external ids
  uint64_t* hk = kept + k;                             // head compare key (dist, part)
  int* head = reinterpret_cast<int*>(hk + L);          // position in each list
  auto load = [&](int l, int h, uint64_t* cmp) {
    if (h >= k) {
      *cmp = ~0ull;
      return;
    }
    const uint64_t o = (static_cast<uint64_t>(l) * a.nq + q) * k + h;
    if (a.kind == 0) {
      const uint64_t key = a.keys[o];
      *cmp = key == ~0ull ? ~0ull : ((key >> 32) << 32) | a.part_no[l];
    } else {
      const HitRecord r = a.records[o];
      *cmp = r.row == UINT32_MAX ? ~0ull : (static_cast<uint64_t>(float_key(r.dist)) << 32) | r.part;
    }
  };
  for (int l = lane; l < L; l += 32) {
    head[l] = 0;
    load(l, 0, &hk[l]);
  }
  __syncwarp();
  int nkept = 0;
  const uint64_t outq = a.perm != nullptr ? a.perm[q] : q;
  for (int guard = 0; guard < L * k && nkept < k; ++guard) {
    uint64_t best = ~0ull;
    int bl = -1;
    for (int l = lane; l < L; l += 32) {
      if (hk[l] < best) {
        best = hk[l];
        bl = l;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int ol = __shfl_xor_sync(0xFFFFFFFFu, bl, o);
      if (ob < best || (ob == best && ol < bl)) {
        best = ob;
        bl = ol;
      }
    }
    if (best == ~0ull) break;
    const int h = head[bl];
    const uint64_t o = (static_cast<uint64_t>(bl) * a.nq + q) * k + h;
    HitRecord rec;
    if (a.kind == 0) {
      const uint64_t key = a.keys[o];
      rec.dist = neighbor_dist(key);
      rec.row = neighbor_id(key);
      rec.part = a.part_no[bl];
      rec.id = a.ids[bl][rec.row];
    } else {
      rec = a.records[o];
    }
    rec.pad = 0;
    __syncwarp();
    if (lane == 0) {
      head[bl] = h + 1;
      load(bl, h + 1, &hk[bl]);
    }
    bool dup = false;
    for (int i = lane; i < nkept; i += 32) dup |= kept[i] == rec.id;
    dup = __any_sync(0xFFFFFFFFu, dup);
    if (!dup) {
      if (lane == 0) {
        kept[nkept] = rec.id;
        if (a.out_records != nullptr) a.out_records[outq * k + nkept] = rec;
        if (a.out_ids != nullptr) {
          a.out_ids[outq * k + nkept] = rec.id;
          a.out_dist[outq * k + nkept] = rec.dist;
        }
      }
      ++nkept;
    }
    __syncwarp();
  }
  for (int i = nkept + lane; i < k; i += 32) {
    if (a.out_records != nullptr) {
      HitRecord m;
      m.dist = INFINITY;
      m.part = UINT32_MAX;
      m.row = UINT32_MAX;
      m.pad = 0;
      m.id = ~0ull;
      a.out_records[outq * k + i] = m;
    }
    if (a.out_ids != nullptr) {
      a.out_ids[outq * k + i] = ~0ull;
      a.out_dist[outq * k + i] = INFINITY;
    }
  }
}

}  // namespace

cudaError_t LaunchPrepareQueries(const float* in, const uint32_t* perm, uint64_t nq, uint32_t dim,
                                 uint32_t pd, bool cosine, float* out, int* qstatus, cudaStream_t st) {
  if (nq == 0) return cudaSuccess;
  const int threads = 128;
  const unsigned blocks = static_cast<unsigned>((nq + threads - 1) / threads);
  NoteLaunch();
  prepare_queries_kernel<<<blocks, threads, 0, st>>>(in, perm, nq, dim, pd, cosine ? 1 : 0, out, qstatus);
  return cudaGetLastError();
}

cudaError_t LaunchLeafRange(const RangeTask* tasks, int ntasks, uint32_t max_words, cudaStream_t st) {
  if (ntasks == 0 || max_words == 0) return cudaSuccess;
  // 8 warps x 32 words per block.
  const dim3 grid((max_words + 255) / 256, ntasks);
  NoteLaunch();
  leaf_range_kernel<<<grid, 256, 0, st>>>(tasks);
  return cudaGetLastError();
}

cudaError_t LaunchPostingScatter(const ScatterTask* tasks, int ntasks, cudaStream_t st) {
  if (ntasks == 0) return cudaSuccess;
  NoteLaunch();
  posting_scatter_kernel<<<ntasks, 256, 0, st>>>(tasks);
  return cudaGetLastError();
}

cudaError_t LaunchFilterProgram(const ProgramTask* tasks, int ntasks, uint32_t max_words, int* status,
                                cudaStream_t st) {
  if (ntasks == 0 || max_words == 0) return cudaSuccess;
  const dim3 grid((max_words + kProgChunkWords - 1) / kProgChunkWords, ntasks);
  NoteLaunch();
  filter_program_kernel<<<grid, 256, 0, st>>>(tasks, status);
  return cudaGetLastError();
}

cudaError_t LaunchCompactRows(const CompactTask* tasks, int ntasks, uint32_t max_words, cudaStream_t st) {
  if (ntasks == 0 || max_words == 0) return cudaSuccess;
  const dim3 grid((max_words + kProgChunkWords - 1) / kProgChunkWords, ntasks);
  NoteLaunch();
  compact_rows_kernel<<<grid, 256, 0, st>>>(tasks);
  return cudaGetLastError();
}

cudaError_t LaunchExactRows(const ExactArgs& a, cudaStream_t st) {
  if (a.nitems == 0) return cudaSuccess;
  if (a.k < 1 || a.k > 240) return cudaErrorInvalidValue;
  if (a.pd <= 4 * 32 + 16) return LaunchExactK<4>(a, st);
  return LaunchExactK<8>(a, st);
}

cudaError_t LaunchPackHits(const PackItem* items, int nitems, uint32_t max_nq, int k, uint64_t out_stride,
                           uint64_t flag_stride, cudaStream_t st) {
  if (nitems == 0 || max_nq == 0) return cudaSuccess;
  const dim3 grid((max_nq + 127) / 128, nitems);
  NoteLaunch();
  pack_hits_kernel<<<grid, 128, 0, st>>>(items, k, out_stride, flag_stride);
  return cudaGetLastError();
}

cudaError_t LaunchMerge(const MergeArgs& a, cudaStream_t st) {
  if (a.nq == 0) return cudaSuccess;
  const size_t smem = kMergeWarps * MergeWarpBytes(a.nlists, a.k);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned blocks = static_cast<unsigned>((a.nq + kMergeWarps - 1) / kMergeWarps);
  NoteLaunch();
  merge_kernel<<<blocks, kMergeWarps * 32, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace vdbgpu
