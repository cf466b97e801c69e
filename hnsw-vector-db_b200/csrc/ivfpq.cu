// IVF-PQ and PQ-flat ADC scan with re-rank (sm_100a): one CTA per query.
//
// Follows IvfPqIndex::search (src/index/quant/ivf_pq.cc:169-222) and PqFlatIndex::search
// (:59-76) float operation for float:
//   * the probed lists and their coarse distances come from the GPU flat search over the coarse
//     centroids (same kernel-set summation order as the reference's dist_);
//   * tables: precomputed L2 uses table = term2[l] + 2 * (-<q_j, C_j[c]>) (:190-205), residual L2
//     uses L2SqAny(q_j - c_j, C_j[c]) (:206-208), inner product / cosine one shared
//     -DotAny(q_j, C_j[c]) table with offset -DotAny(q, c) (:191, 209-211); DotAny / L2SqAny keep
//     the reference's four accumulators (src/distance/scalar.cc:43-73);
//   * ADC: four partial sums over the m sub-quantisers (ProductQuantizer::adc, pq.h:36-47), then
//     offset + adc;
//   * TopK(R) by (dist, id) over all probed rows, then Rerank on fp32 rows (index.cc:89-95).
// The CTA's warps (eight, or four for re-rank depths above 128) share the query's tables in shared
// memory and split each list's rows (codes of 16-byte multiples in software-pipelined 16-byte
// loads); each warp
// keeps its own candidate buffer and threshold (exact: a warp's threshold is the R-th best of
// the entries it has seen, and the tighter of the warps' thresholds is shared as an inclusive
// bound), and the buffers are merged at the end.
#include <cuda_runtime.h>

#include "common.cuh"
#include "ivfpq.cuh"
#include "warp_ops.cuh"

namespace vdbgpu {
namespace {

constexpr int kIvfCap = 512;  // candidates per warp buffer (global memory)
constexpr uint64_t kNone = ~0ull;

// ProductQuantizer::adc over one code (m bytes), four partial sums.
__device__ __forceinline__ float adc(const float* table, const uint8_t* __restrict__ code, int m) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int j = 0;
  if ((m & 3) == 0) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(code);
    for (; j + 4 <= m; j += 4) {
      const uint32_t c = __ldg(&w[j >> 2]);
      s0 = __fadd_rn(s0, table[(j + 0) * 256 + (c & 0xFFu)]);
      s1 = __fadd_rn(s1, table[(j + 1) * 256 + ((c >> 8) & 0xFFu)]);
      s2 = __fadd_rn(s2, table[(j + 2) * 256 + ((c >> 16) & 0xFFu)]);
      s3 = __fadd_rn(s3, table[(j + 3) * 256 + (c >> 24)]);
    }
  } else {
    for (; j + 4 <= m; j += 4) {
      s0 = __fadd_rn(s0, table[(j + 0) * 256 + code[j + 0]]);
      s1 = __fadd_rn(s1, table[(j + 1) * 256 + code[j + 1]]);
      s2 = __fadd_rn(s2, table[(j + 2) * 256 + code[j + 2]]);
      s3 = __fadd_rn(s3, table[(j + 3) * 256 + code[j + 3]]);
    }
    for (; j < m; ++j) s0 = __fadd_rn(s0, table[j * 256 + code[j]]);
  }
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// ProductQuantizer::adc over a code held in registers (m = 16 nv bytes), the same four partial
// sums as adc.
__device__ __forceinline__ float adc_regs(const float* table, const uint4 (&v)[4], int nv) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    if (t < nv) {
      const uint32_t w[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = (t * 4 + u) * 4;
        s0 = __fadd_rn(s0, table[(j + 0) * 256 + (w[u] & 0xFFu)]);
        s1 = __fadd_rn(s1, table[(j + 1) * 256 + ((w[u] >> 8) & 0xFFu)]);
        s2 = __fadd_rn(s2, table[(j + 2) * 256 + ((w[u] >> 16) & 0xFFu)]);
        s3 = __fadd_rn(s3, table[(j + 3) * 256 + (w[u] >> 24)]);
      }
    }
  }
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// Keeps the `keep` smallest packed keys of buf[0..n) (n <= kIvfCap), sorted, at the front.
__device__ int warp_keep_best(uint64_t* buf, int n, int keep) {
  const int lane = threadIdx.x & 31;
  uint64_t x[kIvfCap / 32];
#pragma unroll
  for (int e = 0; e < kIvfCap / 32; ++e) {
    const int i = e * 32 + lane;
    x[e] = i < n ? buf[i] : kNone;
  }
  warp_sort<kIvfCap / 32>(x);
  __syncwarp();
#pragma unroll
  for (int e = 0; e < kIvfCap / 32; ++e) buf[e * 32 + lane] = x[e];
  __syncwarp();
  return n < keep ? n : keep;
}

// warp_keep_best for n <= 256 keys (an eight-per-lane sort).
__device__ int keep_best_256(uint64_t* buf, int n, int keep) {
  const int lane = threadIdx.x & 31;
  uint64_t x[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int i = e * 32 + lane;
    x[e] = i < n ? buf[i] : kNone;
  }
  warp_sort<8>(x);
  __syncwarp();
#pragma unroll
  for (int e = 0; e < 8; ++e) buf[e * 32 + lane] = x[e];
  __syncwarp();
  return n < keep ? n : keep;
}

template <int kIvfWarps>
__global__ void __launch_bounds__(kIvfWarps * 32) ivfpq_kernel(const IvfPqArgs a) {
  extern __shared__ __align__(16) uint8_t ism[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = a.qorder != nullptr ? static_cast<int>(a.qorder[blockIdx.x]) : static_cast<int>(blockIdx.x);
  const int m = a.m, ds = a.dsub, pd = a.pd, ts = m * 256;
  float* q_s = reinterpret_cast<float*>(ism);                 // pd
  float* r_s = q_s + pd;                                      // pd (residual)
  float* table = r_s + pd;                                    // ts
  float* qtab = table + ts;                                   // ts (precomputed L2 only)
  // Candidate buffers live in global memory (inserts are rare), so a CTA's shared memory is just
  // the query's tables and two CTAs of eight warps fit on an SM.
  uint64_t* bufs = a.cand + static_cast<size_t>(q) * kIvfWarps * kIvfCap;
  uint64_t* buf = bufs + warp * kIvfCap;
  __shared__ uint64_t tau_shared;
  __shared__ float offset_s;
  __shared__ int count_s[kIvfWarps];

  for (int i = threadIdx.x; i < pd; i += blockDim.x) q_s[i] = a.queries[static_cast<size_t>(q) * pd + i];
  if (threadIdx.x == 0) tau_shared = kNone;
  __syncthreads();
  const bool l2 = a.metric == 0;
  // Per-query tables.
  if (a.mode == kIvfPrecomputed) {
    for (int i = threadIdx.x; i < ts; i += blockDim.x) {
      const int j = i >> 8;
      const float d = dot_any(q_s + j * ds, a.centroids + static_cast<size_t>(i) * ds, ds);
      qtab[i] = __fmul_rn(-d, 2.f);
    }
  } else if (a.mode == kIvfShared || a.mode == kPqFlat) {
    for (int i = threadIdx.x; i < ts; i += blockDim.x) {
      const int j = i >> 8;
      const float* cen = a.centroids + static_cast<size_t>(i) * ds;
      table[i] = (l2 && a.mode == kPqFlat) ? l2_any(q_s + j * ds, cen, ds) : -dot_any(q_s + j * ds, cen, ds);
    }
  }
  __syncthreads();

  const int R = a.depth > a.k ? a.depth : a.k;  // TopK(max(depth, k))
  uint64_t tau = kNone;                          // this warp's R-th best so far (exclusive)
  int count = 0;
  uint64_t dc = 0;
  const uint32_t lt = (1u << lane) - 1u;
  const int nprobe = a.mode == kPqFlat ? 1 : a.nprobe;
  const int nv = m >> 4;
  const bool vec_codes = (m & 15) == 0 && nv >= 1 && nv <= 4 && (reinterpret_cast<uintptr_t>(a.codes) & 15u) == 0;
  for (int pi = 0; pi < nprobe; ++pi) {
    uint32_t l = 0;
    float offset = 0.f;
    if (a.mode != kPqFlat) {
      l = a.probe_ids[static_cast<size_t>(q) * a.nprobe + pi];
      if (static_cast<uint64_t>(l) >= a.nlist) {
        if (threadIdx.x == 0) set_error(a.status, kDevBadIndex);
        break;
      }
    }
    const uint64_t b0 = a.mode == kPqFlat ? 0 : a.list_off[l];
    const uint64_t e0 = a.mode == kPqFlat ? a.n : a.list_off[l + 1];
    // Row i's id and code (16 nv bytes in 16-byte loads); rows past the list end read nothing.
    auto load_row = [&](uint64_t i, uint4 (&v)[4], uint32_t& id, bool& in) {
      in = i < e0;
      id = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) v[t] = make_uint4(0u, 0u, 0u, 0u);
      if (in) {
        id = a.mode == kPqFlat ? static_cast<uint32_t>(i) : __ldg(&a.ids[i]);
        const uint4* cp = reinterpret_cast<const uint4*>(a.codes + i * m);
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (t < nv) v[t] = __ldg(&cp[t]);
      }
    };
    // The warp's first rows of the list are requested before the table is built, so their
    // latency overlaps the build.
    uint4 nxt_v[4];
    uint32_t nxt_id = 0;
    bool nxt_in = false;
    if (vec_codes) load_row(b0 + static_cast<uint64_t>(warp) * 32 + lane, nxt_v, nxt_id, nxt_in);
    if (a.mode == kIvfPrecomputed) {
      offset = a.probe_dist[static_cast<size_t>(q) * a.nprobe + pi];
      const float* t2 = a.term2 + static_cast<size_t>(l) * ts;
      // 16-byte steps: ts = 256 m floats, and term2 / table / qtab start on 16-byte boundaries.
      const float4* t24 = reinterpret_cast<const float4*>(t2);
      const float4* qt4 = reinterpret_cast<const float4*>(qtab);
      float4* tb4 = reinterpret_cast<float4*>(table);
      for (int i = threadIdx.x; i < (ts >> 2); i += blockDim.x) {
        const float4 x = __ldg(&t24[i]), y = qt4[i];
        tb4[i] = make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z), __fadd_rn(x.w, y.w));
      }
    } else if (a.mode == kIvfResidual) {
      const float* c = a.coarse + static_cast<size_t>(l) * pd;
      for (int j = threadIdx.x; j < a.dim; j += blockDim.x) r_s[j] = __fsub_rn(q_s[j], c[j]);
      __syncthreads();
      for (int i = threadIdx.x; i < ts; i += blockDim.x) {
        const int j = i >> 8;
        table[i] = l2_any(r_s + j * ds, a.centroids + static_cast<size_t>(i) * ds, ds);
      }
    } else if (a.mode == kIvfShared) {
      if (threadIdx.x == 0) offset_s = -dot_any(q_s, a.coarse + static_cast<size_t>(l) * pd, a.dim);
      __syncthreads();
      offset = offset_s;
    }
    __syncthreads();
    // The tighter shared bound (another warp's R-th best, inclusive) also prunes this warp.
    const uint64_t tb = tau_shared;
    const uint64_t bound = tb < tau ? tb : tau;
    dc += e0 - b0;
    uint64_t cur_bound = bound;
    // Appends a key below the bound to this warp's buffer; a full buffer is cut to its R best,
    // whose R-th key becomes the warp's bound (and the shared inclusive bound).
    auto file = [&](uint64_t key) {
      const bool pass = key < cur_bound;
      const uint32_t pm = __ballot_sync(0xFFFFFFFFu, pass);
      if (pm != 0u) {
        if (pass) buf[count + __popc(pm & lt)] = key;
        count += __popc(pm);
        __syncwarp();
        if (count > kIvfCap - 32) {
          count = warp_keep_best(buf, count, R);
          if (count == R) {
            tau = buf[R - 1];  // R-th best: later keys must be smaller (ids are unique)
            cur_bound = tau < cur_bound ? tau : cur_bound;
            if (lane == 0) atomicMin(reinterpret_cast<unsigned long long*>(&tau_shared), tau + 1);
          }
        }
      }
    };
    const uint64_t span = static_cast<uint64_t>(kIvfWarps) * 32;
    if (vec_codes) {
      // Software-pipelined: the warp's next 32 rows are requested before the current ones are
      // scored.
      for (uint64_t base = b0 + static_cast<uint64_t>(warp) * 32; base < e0; base += span) {
        uint4 v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = nxt_v[t];
        const uint32_t id = nxt_id;
        const bool in = nxt_in;
        load_row(base + span + lane, nxt_v, nxt_id, nxt_in);
        uint64_t key = kNone;
        if (in && (a.allow == nullptr || ((__ldg(&a.allow[id >> 5]) >> (id & 31)) & 1u)))
          key = pack_neighbor(__fadd_rn(offset, adc_regs(table, v, nv)), id);
        file(key);
      }
    } else {
      for (uint64_t base = b0 + static_cast<uint64_t>(warp) * 32; base < e0; base += span) {
        const uint64_t i = base + lane;
        uint64_t key = kNone;
        if (i < e0) {
          const uint32_t id = a.mode == kPqFlat ? static_cast<uint32_t>(i) : __ldg(&a.ids[i]);
          const bool ok = a.allow == nullptr || ((__ldg(&a.allow[id >> 5]) >> (id & 31)) & 1u);
          if (ok) {
            const float d = __fadd_rn(offset, adc(table, a.codes + i * m, m));
            key = pack_neighbor(d, id);
          }
        }
        file(key);
      }
    }
    __syncthreads();  // table is rebuilt for the next list
  }
  // Merge: every warp reduces to its R best (sorted), then the lists merge pairwise in a tree
  // into warp 0's buffer; all warps re-rank, warp 0 sorts and writes.
  count = warp_keep_best(buf, count, R);
  if (lane == 0) count_s[warp] = count;
  __syncthreads();
  for (int step = 1; step < kIvfWarps; step <<= 1) {
    if ((warp & (2 * step - 1)) == 0) {
      const int n0 = count_s[warp], n1 = count_s[warp + step];
      const uint64_t* pb = bufs + static_cast<size_t>(warp + step) * kIvfCap;
      for (int i = lane; i < n1; i += 32) buf[n0 + i] = pb[i];
      __syncwarp();
      const int kept = n0 + n1 <= 256 ? keep_best_256(buf, n0 + n1, R) : warp_keep_best(buf, n0 + n1, R);
      if (lane == 0) count_s[warp] = kept;
    }
    __syncthreads();
  }
  uint64_t* all = bufs;  // warp 0's buffer: the R best, sorted
  const int ncand = count_s[0];
  if (a.depth > 0) {
    // Rerank the R best on fp32 rows (exact, reference kernel-set order), four rows per warp step.
    for (int i = warp * 4; i < ncand; i += kIvfWarps * 4) {
      uint32_t r[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) r[c] = neighbor_id(all[i + c < ncand ? i + c : i]);
      float d[4];
      if (a.order == kOrderAvx512 && pd <= 8 * 32 + 16) {
        warp_exact_dist4_avx512<8>(q_s, a.rows, r, ncand - i, pd, l2, d);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          d[c] = warp_exact_dist(q_s, a.rows + static_cast<size_t>(r[c]) * pd, pd, l2, a.order);
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
        all[i + lane] = pack_neighbor(dl, rl);
      }
      __syncwarp();
    }
    __syncthreads();
  }
  if (warp == 0) {
    int nout;
    if (a.depth > 0) {
      {
        uint64_t x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = e * 32 + lane;
          x[e] = i < ncand ? all[i] : kNone;
        }
        warp_sort<8>(x);
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 8; ++e) all[e * 32 + lane] = x[e];
        __syncwarp();
      }
      dc += static_cast<uint64_t>(ncand);
      nout = ncand < a.k ? ncand : a.k;
    } else {
      nout = ncand < a.k ? ncand : a.k;
    }
    for (int i = lane; i < a.k; i += 32) {
      const size_t o = static_cast<size_t>(q) * a.k + i;
      if (i < nout) {
        a.out_dist[o] = neighbor_dist(all[i]);
        a.out_row[o] = neighbor_id(all[i]);
      } else {
        a.out_dist[o] = INFINITY;
        a.out_row[o] = UINT32_MAX;
      }
    }
    if (lane == 0 && a.out_dc != nullptr)
      a.out_dc[q] = (a.mode == kPqFlat ? 0 : a.nlist) + dc;
  }
}

// IvfPqIndex::precompute_tables (src/index/quant/ivf_pq.cc:152-167): term2[l][j][c] =
// DotAny(C_j[c], C_j[c]) + 2 * DotAny(coarse_l + j*dsub, C_j[c]).
__global__ void term2_kernel(const float* __restrict__ coarse, uint32_t nlist, int pd,
                             const float* __restrict__ centroids, int m, int ds, float* term2) {
  const uint64_t ts = static_cast<uint64_t>(m) * 256;
  const uint64_t total = nlist * ts;
  for (uint64_t x = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < total;
       x += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t l = x / ts, i = x % ts;
    const int j = static_cast<int>(i >> 8);
    const float* cen = centroids + i * ds;
    const float norm = dot_any(cen, cen, ds);
    term2[x] = __fadd_rn(norm, __fmul_rn(2.f, dot_any(coarse + l * pd + j * ds, cen, ds)));
  }
}

// Launch order of the list scan: the queries grouped by their nearest probed list (a counting
// sort), so CTAs that run at the same time share lists and find their codes and term2 rows in L2.
// Each query's result does not depend on when its CTA runs. Bucket nlist takes out-of-range ids
// (the scan reports them).
__global__ void probe_count_kernel(const uint32_t* probe_ids, int nq, int nprobe, uint32_t nlist,
                                   uint32_t* counts) {
  const int q = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (q >= nq) return;
  const uint32_t l = probe_ids[static_cast<size_t>(q) * nprobe];
  atomicAdd(&counts[l < nlist ? l : nlist], 1u);
}

// In-place exclusive scan of counts[0..n) by one block of 1024 threads (contiguous chunks).
__global__ void __launch_bounds__(1024) probe_scan_kernel(uint32_t* counts, uint32_t n) {
  __shared__ uint32_t part[1024];
  const uint32_t per = (n + 1023) / 1024;
  const uint32_t b = threadIdx.x * per, e = b + per < n ? b + per : n;
  uint32_t sum = 0;
  for (uint32_t i = b; i < e; ++i) sum += counts[i];
  part[threadIdx.x] = sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const uint32_t v = threadIdx.x >= static_cast<unsigned>(o) ? part[threadIdx.x - o] : 0u;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  uint32_t run = part[threadIdx.x] - sum;
  for (uint32_t i = b; i < e; ++i) {
    const uint32_t c = counts[i];
    counts[i] = run;
    run += c;
  }
}

__global__ void probe_place_kernel(const uint32_t* probe_ids, int nq, int nprobe, uint32_t nlist,
                                   uint32_t* offsets, uint32_t* order) {
  const int q = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (q >= nq) return;
  const uint32_t l = probe_ids[static_cast<size_t>(q) * nprobe];
  order[atomicAdd(&offsets[l < nlist ? l : nlist], 1u)] = static_cast<uint32_t>(q);
}

}  // namespace

size_t IvfPqSmemBytes(int pd, int m, int mode) {
  const size_t ts = static_cast<size_t>(m) * 256;
  return (2 * static_cast<size_t>(pd) + ts + (mode == kIvfPrecomputed ? ts : 0)) * 4;
}

int IvfPqWarps(int k, int depth) {
  // The final merge sorts every warp's R best at once (at most 1024 keys).
  const int r = depth > k ? depth : k;
  return 8 * r <= 1024 ? 8 : 4;
}

size_t IvfPqCandBytes(int nq, int k, int depth) {
  return static_cast<size_t>(nq) * IvfPqWarps(k, depth) * kIvfCap * sizeof(uint64_t);
}

cudaError_t LaunchProbeOrder(const uint32_t* probe_ids, int nq, int nprobe, uint32_t nlist, uint32_t* counts,
                             uint32_t* order, cudaStream_t stream) {
  if (nq <= 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(counts, 0, (static_cast<size_t>(nlist) + 1) * sizeof(uint32_t), stream);
  if (e != cudaSuccess) return e;
  const int blocks = (nq + 255) / 256;
  NoteLaunch();
  probe_count_kernel<<<blocks, 256, 0, stream>>>(probe_ids, nq, nprobe, nlist, counts);
  NoteLaunch();
  probe_scan_kernel<<<1, 1024, 0, stream>>>(counts, nlist + 1);
  NoteLaunch();
  probe_place_kernel<<<blocks, 256, 0, stream>>>(probe_ids, nq, nprobe, nlist, counts, order);
  return cudaGetLastError();
}

cudaError_t LaunchIvfPq(const IvfPqArgs& a, cudaStream_t stream) {
  const size_t smem = IvfPqSmemBytes(a.pd, a.m, a.mode);
  if (a.cand == nullptr) return cudaErrorInvalidValue;
  if (IvfPqWarps(a.k, a.depth) == 8) {
    cudaError_t e = cudaFuncSetAttribute(ivfpq_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    NoteLaunch();
    ivfpq_kernel<8><<<a.nq, 8 * 32, smem, stream>>>(a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(ivfpq_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    NoteLaunch();
    ivfpq_kernel<4><<<a.nq, 4 * 32, smem, stream>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t LaunchTerm2(const float* coarse, uint32_t nlist, int pd, const float* centroids, int m,
                        int ds, float* term2, cudaStream_t stream) {
  NoteLaunch();
  term2_kernel<<<2048, 256, 0, stream>>>(coarse, nlist, pd, centroids, m, ds, term2);
  return cudaGetLastError();
}

}  // namespace vdbgpu
