// Tensor-core pre-rank scan for flat and SQ8 search (sm_100a).
//
// Replaces the reference's per-row distance loop (FlatSearch, src/index/flat_index.cc:11-27, and
// the SQ8 distance loop over codes, src/distance/avx512.cc:48-65) with a Q x N x K contraction on
// the 5th-generation tensor cores, fused with a streaming top-C selection so the Q x N distance
// matrix never reaches HBM.
//
// One persistent CTA per SM walks "units": a 128-query tile against a contiguous slice of rows.
//   warp 0      TMA producer: loads the query tile once per unit (resident), then streams row
//               k-blocks (256 rows x 64 fp16) through an mbarrier ring of up to 6 stages.
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and one thread issues
//               tcgen05.mma (M=128, N=256, K=16) into alternating accumulators.
//   warps 2..   epilogue: each thread owns one query (one TMEM lane) and reads its 256 columns in
//               chunks of 32 (tcgen05.ld), keeping each chunk's best score (one min per value);
//               one vote per chunk finds the chunks where some query of the warp beats its
//               threshold, and only those are read again and their qualifying (key, row) pairs
//               appended to the query's candidate buffer in global memory. A full buffer is
//               compacted by the whole warp to its C best (by key, then row) and the C-th key
//               becomes the new threshold, also published to every unit of the same query.
// A seeding sample scan (chunk_best) appends only each chunk's best key instead.
// Rows inside one unit arrive in increasing order, so a strict "key < threshold" test keeps
// ties exactly as the reference's (dist, id) order does. Thresholds from other units are
// applied as "key <= their C-th key", which can never drop a member of the global top C.
#include "common.cuh"
#include "scan_mma.cuh"

#include <cuda_runtime.h>

namespace vdbgpu {
namespace {

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

constexpr uint32_t kABytesPerKB = kScanBM * 128;  // 16 KB
constexpr uint32_t kBBytesPerStage = kScanBN * 128;  // 32 KB
constexpr uint32_t kTmemCols = 512;

struct __align__(8) ScanBarriers {
  uint64_t full[kScanMaxStages];
  uint64_t empty[kScanMaxStages];
  uint64_t a_full;
  uint64_t a_empty;
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_slot;
};

// Units are ordered slice-major: the CTAs running at the same time cover one or two row slices
// for every query tile, so each slice is read from HBM about once and served from L2, and the
// later slices of a query start from the threshold its earlier slices published.
template <int kMode>
__device__ __forceinline__ void unit_rows(const ScanArgs& a, int unit, int* qtile, int* r0,
                                          int* r1) {
  if constexpr (kMode == kKeyList) {
    // List mode: unit u is query tile u against its own row range.
    const int2 u = a.unit_rows[unit];
    *qtile = unit;
    *r0 = u.x;
    *r1 = u.y;
    return;
  }
  const int qtiles = a.nunits / a.units_per_qtile;
  const int part = unit / qtiles;
  *qtile = unit - part * qtiles;
  *r0 = part * a.rows_per_unit;
  int e = *r0 + a.rows_per_unit;
  *r1 = e < a.nrows ? e : a.nrows;
}

// Warp-cooperative compaction of lane `src`'s candidate buffer (n <= 32 kT entries, in row order)
// to its `keep` best by (key, row). Returns the keep-th key (ordered) to every lane.
template <int kT>
__device__ uint32_t compact_buffer(uint2* buf, int n, int keep) {
  const int lane = threadIdx.x & 31;
  uint32_t keys[kT];
  uint2 ent[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    const int e = lane + 32 * t;
    ent[t] = e < n ? buf[e] : make_uint2(0xFFFFFFFFu, 0xFFFFFFFFu);
    keys[t] = e < n ? float_key(__uint_as_float(ent[t].x)) : 0xFFFFFFFFu;
  }
  // Largest value v with #{key < v} < keep: the keep-th smallest key.
  uint32_t ans = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = ans | (1u << bit);
    int c = 0;
#pragma unroll
    for (int t = 0; t < kT; ++t) c += keys[t] < cand ? 1 : 0;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if (c < keep) ans = cand;
  }
  int less = 0;
#pragma unroll
  for (int t = 0; t < kT; ++t) less += keys[t] < ans ? 1 : 0;
  less = __reduce_add_sync(0xFFFFFFFFu, less);
  const int need_eq = keep - less;
  const uint32_t lt_mask = (1u << lane) - 1u;
  int w = 0, eq_seen = 0;
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    const bool is_less = keys[t] < ans;
    const bool is_eq = keys[t] == ans && (lane + 32 * t) < n;
    const uint32_t eqm = __ballot_sync(0xFFFFFFFFu, is_eq);
    const int eq_before = eq_seen + __popc(eqm & lt_mask);
    const bool keep_it = is_less || (is_eq && eq_before < need_eq);
    const uint32_t km = __ballot_sync(0xFFFFFFFFu, keep_it);
    if (keep_it) buf[w + __popc(km & lt_mask)] = ent[t];
    w += __popc(km);
    eq_seen += __popc(eqm);
  }
  __syncwarp();
  return ans;
}

template <int kMode, int kWgs>
__global__ void __launch_bounds__(ScanThreads(kWgs), 1)
    scan_mma_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, const ScanArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + a.kblocks * kABytesPerKB;
  const int nstages = a.stages > 0 ? a.stages : kScanStages;
  ScanBarriers* bars =
      reinterpret_cast<ScanBarriers*>(smem_b + nstages * kBBytesPerStage);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nstages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->a_full, 1);
    mbar_init(&bars->a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      // Every epilogue thread drains its share of every tile.
      mbar_init(&bars->acc_empty[b], 128 * kWgs);
    }
    mbar_init(&bars->mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, a_phase = 0;
      uint32_t issued = 0, last_parity = 0;  // per-stage bit masks of loads in flight
      bool a_issued = false;
      uint32_t a_parity = 0;
      bool ok = true;
      bool first = true;
      for (int unit = blockIdx.x; ok && unit < a.nunits; unit += gridDim.x) {
        int qtile, r0, r1;
        unit_rows<kMode>(a, unit, &qtile, &r0, &r1);
        if (!first) {
          if (!mbar_wait(&bars->a_empty, a_phase, a.status, kDevTimeoutEmpty)) break;
          a_phase ^= 1u;
        }
        first = false;
        mbar_arrive_expect_tx(&bars->a_full, a.kblocks * kABytesPerKB);
        a_issued = true;
        a_parity = a_phase;
        for (int kb = 0; kb < a.kblocks; ++kb)
          tma_load_2d(smem_a + kb * kABytesPerKB, &tmap_a, &bars->a_full, kb * kScanBK,
                      qtile * kScanBM);
        for (int row0 = r0; ok && row0 < r1; row0 += kScanBN) {
          for (int kb = 0; kb < a.kblocks; ++kb) {
            if (!mbar_wait(&bars->empty[stage], phase ^ 1u, a.status, kDevTimeoutEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->full[stage], kBBytesPerStage);
            tma_load_2d(smem_b + stage * kBBytesPerStage, &tmap_b, &bars->full[stage],
                        kb * kScanBK, row0);
            issued |= 1u << stage;
            last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == nstages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      // Every copy this thread issued lands before the CTA may exit (bounded): the last load
      // into each stage completes the phase recorded for it.
      for (int s = 0; s < nstages; ++s)
        if ((issued >> s) & 1u)
          mbar_wait(&bars->full[s], (last_parity >> s) & 1u, nullptr, 0);
      if (a_issued) mbar_wait(&bars->a_full, a_parity, nullptr, 0);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kScanBM, kScanBN, static_cast<uint32_t>(a.ab_format));
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0, a_phase = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(smem_a), b_base = smem_u32(smem_b);
      for (int unit = blockIdx.x; ok && unit < a.nunits; unit += gridDim.x) {
        int qtile, r0, r1;
        unit_rows<kMode>(a, unit, &qtile, &r0, &r1);
        if (!mbar_wait(&bars->a_full, a_phase, a.status, kDevTimeoutFull)) break;
        a_phase ^= 1u;
        tc_fence_after();
        for (int row0 = r0; ok && row0 < r1; row0 += kScanBN) {
          if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u, a.status, kDevTimeoutAccFree)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kScanBN);
          for (int kb = 0; kb < a.kblocks; ++kb) {
            if (!mbar_wait(&bars->full[stage], phase, a.status, kDevTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_kb = a_base + kb * kABytesPerKB;
            const uint32_t b_st = b_base + stage * kBBytesPerStage;
#pragma unroll
            for (int kk = 0; kk < kScanBK / 16; ++kk) {
              umma_f16(d_tmem, umma_desc_sw128(a_kb + kk * 32), umma_desc_sw128(b_st + kk * 32),
                       idesc, (kb | kk) != 0 ? 1u : 0u);
            }
            umma_commit(&bars->empty[stage]);
            if (++stage == nstages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&bars->acc_full[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        umma_commit(&bars->a_empty);
      }
      // Every MMA this thread issued retires before TMEM is released (bounded wait).
      umma_commit(&bars->mma_done);
      mbar_wait(&bars->mma_done, 0, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // kWgs warpgroups split every tile's columns (warpgroup w takes chunks [w kChunks,
    // (w + 1) kChunks)), so an accumulator is free again after 1 / kWgs of a tile's epilogue
    // latency; each warpgroup keeps its own threshold and candidate list per query.
    const int wg = kWgs == 1 ? 0 : (warp - 2) >> 2;
    constexpr int kChunks = kScanBN / 32 / kWgs;
    const int col0 = wg * kChunks * 32;
    unsigned long long n_chunks = 0, n_trig = 0, n_ins = 0, n_comp = 0;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    uint32_t tcount = 0;  // tiles of this CTA so far
    // A list holding more than compact_at entries is compacted to `keep` (at most 32 land per chunk).
    const int compact_at = a.compact_at > 0 ? a.compact_at : kScanCap - 32;
    bool ok = true;
    for (int unit = blockIdx.x; ok && unit < a.nunits; unit += gridDim.x) {
      int qtile, r0, r1;
      unit_rows<kMode>(a, unit, &qtile, &r0, &r1);
      // q: the query's operand row (list mode: a slot of the gathered tiles, serving query qid).
      const int q = qtile * kScanBM + row_in_tile;
      uint32_t qid = static_cast<uint32_t>(q);
      float qoff = 0.f;
      if constexpr (kMode == kKeyList) {
        qid = q < a.nq ? a.slot_query[q] : 0xFFFFFFFFu;
        if (qid != 0xFFFFFFFFu) qoff = a.slot_offset[q];
      }
      const bool valid_q = kMode == kKeyList ? qid != 0xFFFFFFFFu : q < a.nq;
      // key = qs * acc (+ row term); qs is minus a power of two, so key < tau <=> acc > tau / qs
      // holds exactly and the scaled-key fast path compares raw accumulators.
      const float qs = valid_q ? a.qscale[q] : -1.f;
      const float qs_inv = 1.f / qs;
      float tau = valid_q ? INFINITY : -INFINITY;
      // A bound present before the unit starts (a seeded estimate, or the C-th key another
      // slice of this query published) applies from the first row on.
      if (valid_q) {
        const uint32_t g0 = *reinterpret_cast<volatile uint32_t*>(&a.qtau[qid]);
        if (g0 != 0xFFFFFFFFu) tau = key_float(g0);
      }
      float tau_acc = tau * qs_inv;
      int count = 0;
      const size_t slot = (static_cast<size_t>(unit) * kWgs + wg) * kScanBM + row_in_tile;
      uint2* buf = a.cand + slot * kScanCap;

      // Compacts every lane whose buffer holds more than `limit` entries to its `keep` best
      // and publishes the keep-th key for the other units of the same query.
      auto compact_lanes = [&](int limit) {
        uint32_t need = __ballot_sync(0xFFFFFFFFu, count > limit);
        while (need != 0u) {
          const int src = __ffs(need) - 1;
          need &= need - 1u;
          const int n = __shfl_sync(0xFFFFFFFFu, count, src);
          uint2* sbuf = a.cand + ((static_cast<size_t>(unit) * kWgs + wg) * kScanBM + quad * 32 + src) *
                                     kScanCap;
          ++n_comp;
          __syncwarp();
          // Short lists (the sample pass compacts at 96 + 32) take the 4-slot variant.
          const uint32_t kth = n <= 128 ? compact_buffer<4>(sbuf, n, a.keep)
                                        : compact_buffer<kScanCap / 32>(sbuf, n, a.keep);
          if (lane == src) {
            count = a.keep;
            tau = fminf(tau, key_float(kth));
            tau_acc = tau * qs_inv;
            // Other units of this query may drop keys above the keep-th key of this one.
            atomicMin(&a.qtau[qid], kth + 1u);
          }
        }
      };

      // Scores of one chunk of 32 accumulator columns starting at row c0, in place: raw
      // accumulators (larger is closer, scaled-key mode) or keys (smaller is closer, row-term
      // mode); masked columns get the worst score.
      constexpr bool kMin = kMode != kKeyScaled;
      auto better = [](float x, float y) { return kMin ? fminf(x, y) : fmaxf(x, y); };
      auto scores = [&](uint32_t (&v)[32], int c0) {
        uint32_t allow_bits = 0xFFFFFFFFu;
        if (a.allow != nullptr) allow_bits = __ldg(&a.allow[c0 >> 5]);
        const int nvalid = r1 - c0;
        const bool full = nvalid >= 32 && allow_bits == 0xFFFFFFFFu;
        const float worst = kMin ? INFINITY : -INFINITY;
        if constexpr (kMode == kKeyRowTerm) {
          const float4* rt4 = reinterpret_cast<const float4*>(a.rowterm + c0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 x = __ldg(&rt4[j]);
            v[4 * j + 0] = __float_as_uint(fmaf(qs, __uint_as_float(v[4 * j + 0]), x.x));
            v[4 * j + 1] = __float_as_uint(fmaf(qs, __uint_as_float(v[4 * j + 1]), x.y));
            v[4 * j + 2] = __float_as_uint(fmaf(qs, __uint_as_float(v[4 * j + 2]), x.z));
            v[4 * j + 3] = __float_as_uint(fmaf(qs, __uint_as_float(v[4 * j + 3]), x.w));
          }
        } else if constexpr (kMode == kKeyList) {
          // The row term plus the query's per-list offset (rows of a list start on 32-row
          // boundaries, so the row terms load in 16-byte steps).
          const float4* rt4 = reinterpret_cast<const float4*>(a.rowterm + c0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 x = __ldg(&rt4[j]);
            v[4 * j + 0] = __float_as_uint(__fadd_rn(fmaf(qs, __uint_as_float(v[4 * j + 0]), x.x), qoff));
            v[4 * j + 1] = __float_as_uint(__fadd_rn(fmaf(qs, __uint_as_float(v[4 * j + 1]), x.y), qoff));
            v[4 * j + 2] = __float_as_uint(__fadd_rn(fmaf(qs, __uint_as_float(v[4 * j + 2]), x.z), qoff));
            v[4 * j + 3] = __float_as_uint(__fadd_rn(fmaf(qs, __uint_as_float(v[4 * j + 3]), x.w), qoff));
          }
        }
        if (!full) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j >= nvalid || !((allow_bits >> j) & 1u)) v[j] = __float_as_uint(worst);
        }
      };
      // Three-input min / max (exact): 16 operations for 32 values instead of 31.
      auto better3 = [](float x, float y, float z) { return kMin ? fmin3(x, y, z) : fmax3(x, y, z); };
      auto best32 = [&](const uint32_t (&v)[32]) {
        float t[11];
#pragma unroll
        for (int i = 0; i < 10; ++i)
          t[i] = better3(__uint_as_float(v[3 * i]), __uint_as_float(v[3 * i + 1]), __uint_as_float(v[3 * i + 2]));
        t[10] = better(__uint_as_float(v[30]), __uint_as_float(v[31]));
        const float u0 = better3(t[0], t[1], t[2]), u1 = better3(t[3], t[4], t[5]);
        const float u2 = better3(t[6], t[7], t[8]), u3 = better(t[9], t[10]);
        return better(better3(u0, u1, u2), u3);
      };
      // Appends the chunk's qualifying columns in column order, descending by groups of 8
      // (hits are sparse: most groups of a chunk with a hit cost one vote).
      auto extract = [&](const uint32_t (&v)[32], int c0) {
        const float bound = kMin ? tau : tau_acc;
        auto passes = [&](float x) { return kMin ? (x < bound) : (x > bound); };
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float m = __uint_as_float(v[8 * g]);
#pragma unroll
          for (int j = 8 * g + 1; j < 8 * g + 8; ++j) m = better(m, __uint_as_float(v[j]));
          if (!__any_sync(0xFFFFFFFFu, passes(m))) continue;
#pragma unroll
          for (int j = 8 * g; j < 8 * g + 8; ++j) {
            const float sc = __uint_as_float(v[j]);
            if (passes(sc)) {
              const float key = kMin ? sc : qs * sc;
              buf[count] = make_uint2(__float_as_uint(key), static_cast<uint32_t>(c0 + j));
              ++count;
              ++n_ins;
            }
          }
        }
        compact_lanes(compact_at);
      };

      // Per tile: pass 1 reads the warp's chunks back to back and keeps each chunk's best score
      // (no branches); one vote per chunk marks the chunks where some query of the warp has a
      // hit; pass 2 reloads only those chunks from TMEM (the accumulator stays put until
      // acc_empty) and appends their hits. (Keeping a warp's 4 chunks of a two-warpgroup tile in
      // registers instead spills at the 168 registers such a CTA allows, and is slower.)
      for (int row0 = r0; row0 < r1; row0 += kScanBN, ++tcount) {
        const int accb = static_cast<int>(tcount & 1u);
        // The shared threshold is read now and applied after pass 1 (hides latency).
        uint32_t g = 0xFFFFFFFFu;
        if (valid_q) g = *reinterpret_cast<volatile uint32_t*>(&a.qtau[qid]);
        if (!mbar_wait(&bars->acc_full[accb], (tcount >> 1) & 1u, a.status, kDevTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                static_cast<uint32_t>(accb * kScanBN + col0);
        const int c_base = row0 + col0;
        auto vote = [&](const float (&cbest)[kChunks]) {
          if (g != 0xFFFFFFFFu) {
            tau = fminf(tau, key_float(g));
            tau_acc = tau * qs_inv;
          }
          const float bound = kMin ? tau : tau_acc;
          uint32_t hits = 0;
#pragma unroll
          for (int ch = 0; ch < kChunks; ++ch)
            if (__any_sync(0xFFFFFFFFu, kMin ? (cbest[ch] < bound) : (cbest[ch] > bound))) hits |= 1u << ch;
          n_chunks += kChunks;
          n_trig += __popc(hits);
          return hits;
        };
        {
          // Pass 1 reads two chunks per tcgen05.ld (64 columns): half the TMEM round trips of
          // single-chunk loads, in the same registers as two of them.
          uint32_t v2[64];
          float cbest[kChunks];
#pragma unroll
          for (int ch = 0; ch < kChunks; ch += 2) {
            __syncwarp();
            tmem_ld_32x32b_x64(t_addr + ch * 32, v2);
            tmem_ld_wait_regs(v2);
            uint32_t (&va)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v2[0]);
            uint32_t (&vb)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v2[32]);
            scores(va, c_base + ch * 32);
            cbest[ch] = best32(va);
            scores(vb, c_base + (ch + 1) * 32);
            cbest[ch + 1] = best32(vb);
          }
          uint32_t (&va)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v2[0]);
          uint32_t hits = vote(cbest);
          if (a.chunk_best) {
            // A seeding sample scan needs an estimate of the keep-th key only: each chunk's best
            // key (a real row's) stands for the chunk, filed under the chunk's first row, and
            // nothing is read again. A nearest-row scan (chunk_best 2, one warpgroup) reloads the
            // chunk to file the key under its own row (the first column holding it).
#pragma unroll
            for (int ch = 0; ch < kChunks; ++ch) {
              if ((hits >> ch) & 1u) {
                const float sc = cbest[ch];
                int col = 0;
                if (kWgs == 1 && a.chunk_best == 2) {
                  __syncwarp();
                  tmem_ld_32x32b_x32(t_addr + ch * 32, va);
                  tmem_ld_wait_regs(va);
                  scores(va, c_base + ch * 32);
#pragma unroll
                  for (int j = 31; j >= 0; --j)
                    if (__uint_as_float(va[j]) == sc) col = j;
                }
                if (kMin ? (sc < tau) : (sc > tau_acc)) {
                  const float key = kMin ? sc : qs * sc;
                  buf[count] = make_uint2(__float_as_uint(key), static_cast<uint32_t>(c_base + ch * 32 + col));
                  ++count;
                  ++n_ins;
                }
                compact_lanes(compact_at);
              }
            }
            hits = 0u;
          }
          while (hits != 0u) {
            const int ch = __ffs(hits) - 1;
            hits &= hits - 1u;
            __syncwarp();
            tmem_ld_32x32b_x32(t_addr + ch * 32, va);
            tmem_ld_wait_regs(va);
            scores(va, c_base + ch * 32);
            extract(va, c_base + ch * 32);
          }
        }
        tc_fence_before();
        mbar_arrive(&bars->acc_empty[accb]);
      }
      // Leave at most `keep` entries per query and publish this unit's keep-th key.
      if (ok) compact_lanes(a.keep);
      a.cand_count[slot] = valid_q ? count : 0;
    }
    if (a.counters != nullptr) {
      unsigned long long ins = n_ins;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ins += __shfl_xor_sync(0xFFFFFFFFu, ins, o);
      if (lane == 0) {
        atomicAdd(&a.counters[0], n_chunks);
        atomicAdd(&a.counters[1], n_trig);
        atomicAdd(&a.counters[2], ins);
        atomicAdd(&a.counters[3], n_comp);
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace

size_t ScanSmemBytes(int kblocks, int stages) {
  return 1024 + static_cast<size_t>(kblocks) * kABytesPerKB +
         static_cast<size_t>(stages > 0 ? stages : kScanStages) * kBBytesPerStage + sizeof(ScanBarriers);
}

int ScanMaxStagesFor(int kblocks) {
  int s = kScanMaxStages;
  while (s > 1 && ScanSmemBytes(kblocks, s) > 227u * 1024u) --s;
  return s;
}

template <int kMode, int kWgs>
cudaError_t LaunchScanT(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const ScanArgs& a,
                        int grid, cudaStream_t stream) {
  if (a.stages < 0 || a.stages > kScanMaxStages) return cudaErrorInvalidValue;
  const size_t smem = ScanSmemBytes(a.kblocks, a.stages);
  if (smem > 227u * 1024u) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(scan_mma_kernel<kMode, kWgs>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  NoteLaunch();
  scan_mma_kernel<kMode, kWgs><<<grid, ScanThreads(kWgs), smem, stream>>>(tmap_a, tmap_b, a);
  return cudaGetLastError();
}

cudaError_t LaunchScan(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const ScanArgs& a,
                       int grid, cudaStream_t stream) {
  if (a.mode == kKeyList) {
    if (a.unit_rows == nullptr || a.slot_query == nullptr || a.slot_offset == nullptr || a.rowterm == nullptr ||
        a.allow != nullptr || a.chunk_best != 0)
      return cudaErrorInvalidValue;
    return a.wgs == 2 ? LaunchScanT<kKeyList, 2>(tmap_a, tmap_b, a, grid, stream)
                      : LaunchScanT<kKeyList, 1>(tmap_a, tmap_b, a, grid, stream);
  }
  if (a.mode == kKeyRowTerm)
    return a.wgs == 2 ? LaunchScanT<kKeyRowTerm, 2>(tmap_a, tmap_b, a, grid, stream)
                      : LaunchScanT<kKeyRowTerm, 1>(tmap_a, tmap_b, a, grid, stream);
  return a.wgs == 2 ? LaunchScanT<kKeyScaled, 2>(tmap_a, tmap_b, a, grid, stream)
                    : LaunchScanT<kKeyScaled, 1>(tmap_a, tmap_b, a, grid, stream);
}

}  // namespace vdbgpu
