// Warp-level building blocks shared by the selection kernels: a register bitonic sort of packed
// (distance, id) keys and exact fp32 distances that sum in the same order as the reference's
// runtime-selected CPU kernels.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace vdbgpu {

// Sorts 32*E packed keys held striped across the warp (element i = e*32 + lane) ascending.
template <int E>
__device__ __forceinline__ void warp_sort(uint64_t (&x)[E]) {
  constexpr int N = 32 * E;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int je = j >> 5;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int p = e ^ je;
          if (p > e) {
            const bool up = (((e * 32) & k) == 0);
            const uint64_t a = x[e], b = x[p];
            const bool swap = up ? (a > b) : (a < b);
            x[e] = swap ? b : a;
            x[p] = swap ? a : b;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = e * 32 + lane;
          const uint64_t other = __shfl_xor_sync(0xFFFFFFFFu, x[e], j);
          const bool up = ((i & k) == 0);
          const bool lower = (lane & j) == 0;
          const bool take_min = (up == lower);
          const uint64_t mn = x[e] < other ? x[e] : other;
          const uint64_t mx = x[e] < other ? other : x[e];
          x[e] = take_min ? mn : mx;
        }
      }
    }
  }
}

// Kernel-set summation orders of the reference (src/distance/cpu_features.cc:36-60).
enum SumOrder : int { kOrderScalar = 0, kOrderAvx512 = 1, kOrderAvx2 = 2 };

// DotAny / L2SqAny (src/distance/scalar.cc:43-73): four partial sums over any length, combined as
// (s0 + s1) + (s2 + s3), without FMA.
__device__ __forceinline__ float dot_any(const float* a, const float* b, int d) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= d; i += 4) {
    s0 = __fadd_rn(s0, __fmul_rn(a[i], b[i]));
    s1 = __fadd_rn(s1, __fmul_rn(a[i + 1], b[i + 1]));
    s2 = __fadd_rn(s2, __fmul_rn(a[i + 2], b[i + 2]));
    s3 = __fadd_rn(s3, __fmul_rn(a[i + 3], b[i + 3]));
  }
  for (; i < d; ++i) s0 = __fadd_rn(s0, __fmul_rn(a[i], b[i]));
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

__device__ __forceinline__ float l2_any(const float* a, const float* b, int d) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int i = 0;
  for (; i + 4 <= d; i += 4) {
    const float t0 = __fsub_rn(a[i], b[i]), t1 = __fsub_rn(a[i + 1], b[i + 1]);
    const float t2 = __fsub_rn(a[i + 2], b[i + 2]), t3 = __fsub_rn(a[i + 3], b[i + 3]);
    s0 = __fadd_rn(s0, __fmul_rn(t0, t0));
    s1 = __fadd_rn(s1, __fmul_rn(t1, t1));
    s2 = __fadd_rn(s2, __fmul_rn(t2, t2));
    s3 = __fadd_rn(s3, __fmul_rn(t3, t3));
  }
  for (; i < d; ++i) {
    const float t = __fsub_rn(a[i], b[i]);
    s0 = __fadd_rn(s0, __fmul_rn(t, t));
  }
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}


// Exact fp32 distance between the warp's query and one row, summed in the order of the
// reference kernel set (all lanes receive the result). q_s and x point to pd floats; q_s may be
// shared memory. l2 selects squared L2, otherwise minus the dot product.
//   avx512: 16 lanes x 2 accumulators over blocks of 32, FMA, tail block of 16 into the first
//           accumulator, then _mm512_reduce_add_ps's tree (src/distance/avx512.cc:19-46)
//   avx2:   8 lanes x 2 accumulators over blocks of 16, FMA, then hadd (avx2.cc:11-46)
//   scalar: one running sum, no FMA (scalar.cc:8-23)
__device__ __forceinline__ float warp_exact_dist(const float* q_s, const float* __restrict__ x,
                                                 int pd, bool l2, int order) {
  const int lane = threadIdx.x & 31;
  float r;
  if (order == kOrderAvx512) {
    float acc = 0.f;
    const int nb = pd >> 5;
    for (int t = 0; t < nb; ++t) {
      const int e = 32 * t + lane;
      const float qv = q_s[e], xv = __ldg(&x[e]);
      if (l2) {
        const float d = __fsub_rn(qv, xv);
        acc = __fmaf_rn(d, d, acc);
      } else {
        acc = __fmaf_rn(qv, xv, acc);
      }
    }
    if ((pd & 31) != 0 && lane < 16) {
      const int e = 32 * nb + lane;
      const float qv = q_s[e], xv = __ldg(&x[e]);
      if (l2) {
        const float d = __fsub_rn(qv, xv);
        acc = __fmaf_rn(d, d, acc);
      } else {
        acc = __fmaf_rn(qv, xv, acc);
      }
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 16));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 8));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 2));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 1));
    r = acc;
  } else if (order == kOrderAvx2) {
    // lane = 8*h + j (h: 0 = acc0, 1 = acc1 within a 16-block); lanes 16..31 idle.
    float acc = 0.f;
    if (lane < 16) {
      for (int i = 0; i < pd; i += 16) {
        const int e = i + lane;
        const float qv = q_s[e], xv = __ldg(&x[e]);
        if (l2) {
          const float d = __fsub_rn(qv, xv);
          acc = __fmaf_rn(d, d, acc);
        } else {
          acc = __fmaf_rn(qv, xv, acc);
        }
      }
    }
    // v[j] = acc0[j] + acc1[j]; s[j] = v[j] + v[4+j]; (s0+s1)+(s2+s3)
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 8));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 1));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 2));
    r = acc;
  } else {
    float s = 0.f;
    if (lane == 0) {
      for (int e = 0; e < pd; ++e) {
        const float qv = q_s[e], xv = __ldg(&x[e]);
        if (l2) {
          const float d = __fsub_rn(qv, xv);
          s = __fadd_rn(s, __fmul_rn(d, d));
        } else {
          s = __fadd_rn(s, __fmul_rn(qv, xv));
        }
      }
    }
    r = s;
  }
  r = __shfl_sync(0xFFFFFFFFu, r, 0);
  return l2 ? r : -r;
}

// Exact SQ8 distance of the query against two codes at once (lanes 0..15: code0, lanes 16..31:
// code1), in the reference kernel set's order. Returns the distance of the half this lane
// belongs to. x = fma(code, scale, vmin) as in Decode16 (src/distance/avx512.cc:11-15).
__device__ __forceinline__ float halfwarp_sq8_dist(const float* q_s, const uint8_t* __restrict__ code,
                                                   const float* vmin_s, const float* scale_s,
                                                   int pd, bool l2, int order) {
  const int lane = threadIdx.x & 31;
  const int j = lane & 15;
  float r;
  if (order == kOrderAvx512) {
    float acc = 0.f;
    for (int i = 0; i < pd; i += 16) {
      const int e = i + j;
      const float xv = __fmaf_rn(static_cast<float>(code[e]), scale_s[e], vmin_s[e]);
      if (l2) {
        const float d = __fsub_rn(q_s[e], xv);
        acc = __fmaf_rn(d, d, acc);
      } else {
        acc = __fmaf_rn(q_s[e], xv, acc);
      }
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 8));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 2));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 1));
    r = acc;
  } else if (order == kOrderAvx2) {
    // lane j: j < 8 -> acc0 lane j over elements i + j; j >= 8 -> acc1 lane j-8 over i + j.
    float acc = 0.f;
    for (int i = 0; i < pd; i += 16) {
      const int e = i + j;
      const float xv = __fmaf_rn(static_cast<float>(code[e]), scale_s[e], vmin_s[e]);
      if (l2) {
        const float d = __fsub_rn(q_s[e], xv);
        acc = __fmaf_rn(d, d, acc);
      } else {
        acc = __fmaf_rn(q_s[e], xv, acc);
      }
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 8));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 1));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 2));
    r = acc;
  } else {
    float s = 0.f;
    if (j == 0) {
      for (int e = 0; e < pd; ++e) {
        const float xv = __fadd_rn(vmin_s[e], __fmul_rn(static_cast<float>(code[e]), scale_s[e]));
        if (l2) {
          const float d = __fsub_rn(q_s[e], xv);
          s = __fadd_rn(s, __fmul_rn(d, d));
        } else {
          s = __fadd_rn(s, __fmul_rn(q_s[e], xv));
        }
      }
    }
    r = s;
  }
  r = __shfl_sync(0xFFFFFFFFu, r, lane & 16);
  return l2 ? r : -r;
}

// AVX-512-order exact distances of up to 4 rows at once (ids r[0..nc)), all lanes receive them.
// Same arithmetic as warp_exact_dist with kOrderAvx512; the loads of the 4 rows are issued
// together so the gathers overlap. pd <= 32 * kMaxT + 16.
template <int kMaxT>
__device__ __forceinline__ void warp_exact_dist4_avx512(const float* q_s, const float* __restrict__ rows,
                                                        const uint32_t (&r)[4], int nc, int pd,
                                                        bool l2, float (&out)[4]) {
  const int lane = threadIdx.x & 31;
  const int nb = pd >> 5;
  const bool tail = (pd & 31) != 0 && lane < 16;
  float x[4][kMaxT + 1];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float* row = rows + static_cast<size_t>(r[c < nc ? c : 0]) * pd;
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) x[c][t] = t < nb ? __ldg(&row[32 * t + lane]) : 0.f;
    x[c][kMaxT] = tail ? __ldg(&row[32 * nb + lane]) : 0.f;
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float acc = 0.f;
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t < nb) {
        const float qv = q_s[32 * t + lane];
        if (l2) {
          const float d = __fsub_rn(qv, x[c][t]);
          acc = __fmaf_rn(d, d, acc);
        } else {
          acc = __fmaf_rn(qv, x[c][t], acc);
        }
      }
    }
    if (tail) {
      const float qv = q_s[32 * nb + lane];
      if (l2) {
        const float d = __fsub_rn(qv, x[c][kMaxT]);
        acc = __fmaf_rn(d, d, acc);
      } else {
        acc = __fmaf_rn(qv, x[c][kMaxT], acc);
      }
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 16));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 8));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 2));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 1));
    acc = __shfl_sync(0xFFFFFFFFu, acc, 0);
    out[c] = l2 ? acc : -acc;
  }
}

// Packed fp32 pairs (Blackwell's two-wide FP32 instructions): each half is one IEEE fp32 operation
// with round-to-nearest, exactly as the scalar instruction.
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }

// The AVX-512 reduction of 16 lanes (+8, +4, +2, +1) over packed pairs: lane j of a quarter-warp
// holds slots 2j and 2j + 1, so slots +8 sit four lanes away, +4 two lanes, +2 one lane and +1
// in the lane. Every lane of the quarter-warp returns the sum.
__device__ __forceinline__ float f2_reduce16(uint64_t v) {
  v = f2_add(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
  v = f2_add(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
  v = f2_add(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
  return __fadd_rn(f2_lo(v), f2_hi(v));
}

// Exact distances (L2, or minus the dot product) of n rows of 32 kT floats (pd = 96 or 128) in
// the AVX-512 kernel's order, 8 rows per pass, two per quarter-warp, every load of a pass issued
// before any arithmetic. The AVX-512 kernel keeps two 16-wide accumulators, acc0 over elements
// 32t + l and acc1 over 32t + 16 + l (t < kT), and reduces acc0 + acc1 by halves. Lane j of a
// quarter-warp holds slots 2j and 2j + 1 of both as packed pairs: its loads are 8-byte pairs and its
// arithmetic two-wide, so every distance is bit-identical to warp_exact_dist's. id_at(i) gives
// row i's id; put(i, dist) is called once per row, by one lane. q_s: 32 kT floats, 8-byte aligned.
template <int kT, class IdAt, class Put>
__device__ __forceinline__ void warp_dists_f32x2(const float* __restrict__ rows, const float* q_s, int n, bool l2,
                                                 IdAt id_at, Put put) {
  const int lane = threadIdx.x & 31, g = lane >> 3, j = lane & 7;
  const uint64_t* q2 = reinterpret_cast<const uint64_t*>(q_s);
  for (int i = 0; i < n; i += 8) {
    uint64_t x[2][2 * kT];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int my = i + 4 * h + g;
      const uint64_t* xp =
          reinterpret_cast<const uint64_t*>(rows + static_cast<size_t>(id_at(my < n ? my : i)) * (32 * kT));
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        x[h][2 * t] = __ldg(&xp[16 * t + j]);          // elements 32t + 2j, +1 (acc0)
        x[h][2 * t + 1] = __ldg(&xp[16 * t + 8 + j]);  // elements 32t + 16 + 2j, +1 (acc1)
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint64_t A0 = 0, A1 = 0;
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        const uint64_t qa = q2[16 * t + j], qb = q2[16 * t + 8 + j];
        if (l2) {
          const uint64_t da = f2_sub(qa, x[h][2 * t]), db = f2_sub(qb, x[h][2 * t + 1]);
          A0 = f2_fma(da, da, A0);
          A1 = f2_fma(db, db, A1);
        } else {
          A0 = f2_fma(qa, x[h][2 * t], A0);
          A1 = f2_fma(qb, x[h][2 * t + 1], A1);
        }
      }
      const float t3 = f2_reduce16(f2_add(A0, A1));  // s[l] = acc0[l] + acc1[l], then the tree
      const int my = i + 4 * h + g;
      if (j == 0 && my < n) put(my, l2 ? t3 : -t3);
    }
  }
  __syncwarp();
}

template <class IdAt, class Put>
__device__ __forceinline__ void warp_dists128_f32(const float* __restrict__ rows, const float* q_s, int n, bool l2,
                                                  IdAt id_at, Put put) {
  warp_dists_f32x2<4>(rows, q_s, n, l2, id_at, put);
}

// Exact SQ8 distances of n code rows of 128 bytes in the AVX-512 kernel's order: one 16-wide
// accumulator over elements 16t + l (t = 0..7) of x = fma(code, scale, vmin), reduced by halves.
// Layout as warp_dists128_f32: lane j of a quarter-warp holds slots 2j and 2j + 1 (a 2-byte load
// per t), 8 rows per pass; bit-identical to halfwarp_sq8_dist. vmin / scale / q_s: 128 floats,
// 8-byte aligned.
template <class IdAt, class Put>
__device__ __forceinline__ void warp_dists128_sq8(const uint8_t* __restrict__ codes, const float* q_s,
                                                  const float* vmin, const float* scale, int n, bool l2,
                                                  IdAt id_at, Put put) {
  const int lane = threadIdx.x & 31, g = lane >> 3, j = lane & 7;
  const uint64_t* q2 = reinterpret_cast<const uint64_t*>(q_s);
  const uint64_t* v2 = reinterpret_cast<const uint64_t*>(vmin);
  const uint64_t* s2 = reinterpret_cast<const uint64_t*>(scale);
  for (int i = 0; i < n; i += 8) {
    uint32_t c[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int my = i + 4 * h + g;
      const uint16_t* cp = reinterpret_cast<const uint16_t*>(codes + static_cast<size_t>(id_at(my < n ? my : i)) * 128);
#pragma unroll
      for (int t = 0; t < 8; ++t) c[h][t] = __ldg(&cp[8 * t + j]);  // elements 16t + 2j, +1
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint64_t A = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint64_t cv = f2_pack(static_cast<float>(c[h][t] & 255u), static_cast<float>(c[h][t] >> 8));
        const uint64_t xv = f2_fma(cv, s2[8 * t + j], v2[8 * t + j]);
        const uint64_t qv = q2[8 * t + j];
        if (l2) {
          const uint64_t dv = f2_sub(qv, xv);
          A = f2_fma(dv, dv, A);
        } else {
          A = f2_fma(qv, xv, A);
        }
      }
      const float r = f2_reduce16(A);
      const int my = i + 4 * h + g;
      if (j == 0 && my < n) put(my, l2 ? r : -r);
    }
  }
  __syncwarp();
}

}  // namespace vdbgpu
