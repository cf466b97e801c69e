// Kernels of the GPU IVF-PQ builder.
//
//   assign_kernel     AssignNearest (src/index/quant/kmeans.cc:22-53): each thread one point, the
//                     centroids streamed through shared memory in tiles, the first minimum over
//                     ascending centroid numbers. Distances follow PickL2 (kmeans.cc:16-20): the
//                     runtime kernel set's L2 in its summation order (per thread: AVX-512's 2 x 16
//                     FMA accumulators and _mm512_reduce_add_ps tree, AVX2's 2 x 8 and hadd, or the
//                     scalar running sum), or L2SqAny for rows that are not multiples of 16 floats.
//   pq_encode_kernel  ProductQuantizer::encode of each row's residual to its list's centroid
//                     (ivf_pq.cc:135-146, pq.cc:44-57): per subquantizer the first nearest of 256
//                     centroids by L2SqAny; residual elements are x - c in fp32 as the reference.
#include <cuda_runtime.h>

#include "common.cuh"
#include "ivfpq_build.cuh"
#include "warp_ops.cuh"

namespace vdbgpu {
namespace {

constexpr int kAssignThreads = 128;
constexpr int kCentTileBytes = 32 * 1024;
constexpr int kEncodeThreads = 128;
constexpr int kPqSmemBytes = 64 * 1024;

// Squared L2 of two d-float vectors in the runtime kernel set's order (d a multiple of 16 for
// the vector orders), one thread.
__device__ __forceinline__ float l2_runtime(const float* a, const float* b, int d, int order) {
  if (order == kOrderAvx512) {
    float acc0[16], acc1[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc0[j] = acc1[j] = 0.f;
    int i = 0;
    for (; i + 32 <= d; i += 32) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float t0 = __fsub_rn(a[i + j], b[i + j]);
        const float t1 = __fsub_rn(a[i + 16 + j], b[i + 16 + j]);
        acc0[j] = __fmaf_rn(t0, t0, acc0[j]);
        acc1[j] = __fmaf_rn(t1, t1, acc1[j]);
      }
    }
    if (i < d) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float t0 = __fsub_rn(a[i + j], b[i + j]);
        acc0[j] = __fmaf_rn(t0, t0, acc0[j]);
      }
    }
    float s[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) s[j] = __fadd_rn(acc0[j], acc1[j]);
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = __fadd_rn(s[8 + j], s[j]);
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = __fadd_rn(s[4 + j], s[j]);
    return __fadd_rn(__fadd_rn(s[0], s[2]), __fadd_rn(s[1], s[3]));
  }
  if (order == kOrderAvx2) {
    float acc0[8], acc1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc0[j] = acc1[j] = 0.f;
    for (int i = 0; i < d; i += 16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float t0 = __fsub_rn(a[i + j], b[i + j]);
        const float t1 = __fsub_rn(a[i + 8 + j], b[i + 8 + j]);
        acc0[j] = __fmaf_rn(t0, t0, acc0[j]);
        acc1[j] = __fmaf_rn(t1, t1, acc1[j]);
      }
    }
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(acc0[j], acc1[j]);
    float s[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = __fadd_rn(v[j], v[4 + j]);
    return __fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3]));
  }
  float s = 0.f;
  for (int i = 0; i < d; ++i) {
    const float t = __fsub_rn(a[i], b[i]);
    s = __fadd_rn(s, __fmul_rn(t, t));
  }
  return s;
}

__global__ void __launch_bounds__(kAssignThreads) assign_kernel(const AssignArgs a) {
  extern __shared__ __align__(16) float asm_s[];
  const int d = a.d, dp = d + 1;  // odd row pitch: conflict-free per-thread rows
  float* pts = asm_s;
  float* cen = asm_s + kAssignThreads * dp;
  const int tile = kCentTileBytes / (d * 4);
  const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kAssignThreads;
  const int np = static_cast<int>(a.n - base < kAssignThreads ? a.n - base : kAssignThreads);
  for (int e = threadIdx.x; e < np * d; e += kAssignThreads) {
    const int p = e / d, i = e - p * d;
    pts[p * dp + i] = a.points[(base + p) * static_cast<uint64_t>(a.stride) + i];
  }
  const float* mine = pts + threadIdx.x * dp;
  float best = INFINITY;
  uint32_t arg = 0;
  for (int c0 = 0; c0 < a.k; c0 += tile) {
    const int nc = a.k - c0 < tile ? a.k - c0 : tile;
    __syncthreads();
    for (int e = threadIdx.x; e < nc * d; e += kAssignThreads)
      cen[e] = a.centroids[static_cast<uint64_t>(c0) * d + e];
    __syncthreads();
    if (threadIdx.x < np) {
      for (int c = 0; c < nc; ++c) {
        const float* cr = cen + c * d;
        const float dd = a.kind == kAssignAny ? l2_any(mine, cr, d) : l2_runtime(mine, cr, d, a.order);
        if (dd < best) {
          best = dd;
          arg = static_cast<uint32_t>(c0 + c);
        }
      }
    }
  }
  if (threadIdx.x < np) {
    a.assign[base + threadIdx.x] = arg;
    if (a.dist != nullptr) a.dist[base + threadIdx.x] = best;
  }
}

__global__ void __launch_bounds__(kEncodeThreads) pq_encode_kernel(const PqEncodeArgs a, int group) {
  extern __shared__ __align__(16) float enc_s[];
  const int dim = a.dim, dp = dim + 1;
  float* res = enc_s;                            // kEncodeThreads x dp residuals
  float* cen = enc_s + kEncodeThreads * dp;      // `group` subquantizers x 256 x dsub
  const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kEncodeThreads;
  const int np = static_cast<int>(a.n - base < kEncodeThreads ? a.n - base : kEncodeThreads);
  for (int e = threadIdx.x; e < np * dim; e += kEncodeThreads) {
    const int p = e / dim, i = e - p * dim;
    const uint64_t row = base + p;
    float x = a.rows[row * a.pd + i];
    if (a.coarse != nullptr) x = __fsub_rn(x, a.coarse[static_cast<uint64_t>(a.assign[row]) * a.pd + i]);
    res[p * dp + i] = x;
  }
  const float* mine = res + threadIdx.x * dp;
  const int per = 256 * a.dsub;
  for (int j0 = 0; j0 < a.m; j0 += group) {
    const int ng = a.m - j0 < group ? a.m - j0 : group;
    __syncthreads();
    for (int e = threadIdx.x; e < ng * per; e += kEncodeThreads)
      cen[e] = a.pq[static_cast<uint64_t>(j0) * per + e];
    __syncthreads();
    if (threadIdx.x < np) {
      for (int jj = 0; jj < ng; ++jj) {
        const float* xs = mine + (j0 + jj) * a.dsub;
        const float* cj = cen + jj * per;
        float best = INFINITY;
        int arg = 0;
        for (int c = 0; c < 256; ++c) {
          const float dd = l2_any(xs, cj + c * a.dsub, a.dsub);
          if (dd < best) {
            best = dd;
            arg = c;
          }
        }
        a.codes[(base + threadIdx.x) * a.m + j0 + jj] = static_cast<uint8_t>(arg);
      }
    }
  }
}

}  // namespace

cudaError_t LaunchAssignNearest(const AssignArgs& a, cudaStream_t st) {
  if (a.n == 0) return cudaSuccess;
  if (a.d <= 0 || a.d > kAssignMaxDim || a.k <= 0) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(kAssignThreads) * (a.d + 1) * 4 + kCentTileBytes;
  cudaError_t e = cudaFuncSetAttribute(assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const uint64_t blocks = (a.n + kAssignThreads - 1) / kAssignThreads;
  NoteLaunch();
  assign_kernel<<<static_cast<unsigned>(blocks), kAssignThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchPqEncode(const PqEncodeArgs& a, cudaStream_t st) {
  if (a.n == 0) return cudaSuccess;
  if (a.dim <= 0 || a.dim > kAssignMaxDim || a.dsub <= 0 || a.m * a.dsub != a.dim)
    return cudaErrorInvalidValue;
  const int per_bytes = 256 * a.dsub * 4;
  int group = kPqSmemBytes / per_bytes;
  if (group < 1) return cudaErrorInvalidValue;
  if (group > a.m) group = a.m;
  const size_t smem = static_cast<size_t>(kEncodeThreads) * (a.dim + 1) * 4 + static_cast<size_t>(group) * per_bytes;
  cudaError_t e = cudaFuncSetAttribute(pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const uint64_t blocks = (a.n + kEncodeThreads - 1) / kEncodeThreads;
  NoteLaunch();
  pq_encode_kernel<<<static_cast<unsigned>(blocks), kEncodeThreads, smem, st>>>(a, group);
  return cudaGetLastError();
}

}  // namespace vdbgpu
