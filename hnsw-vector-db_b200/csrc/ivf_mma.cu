// IVF-PQ pre-rank on the tensor cores (list mode of the scan, scan_mma.cu): the operands and the
// per-batch tiles.
//
// For L2, ||q - c_l - r||^2 = ||q - c_l||^2 - 2 <q, r> + (||r||^2 + 2 <c_l, r>), where r is a row's
// decoded residual (the concatenated sub-quantizer centroids of its code). The index keeps r in
// fp16 (every list starting on a 32-row boundary) with its row term ||r||^2 + 2 <c_l, r>; a batch
// is cut into query tiles, each gathered from the queries that probe one list, and the scan keys
// every (query, row) of the tile's list as row term - 2 <q, r> + ||q - c_l||^2. These keys only
// choose candidates: the distances returned are the reference's ADC of the chosen rows
// (ivf_finalize_kernel, select.cu).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "ivfpq.cuh"

namespace vdbgpu {
namespace {

// One block per list: row i of list l goes to operand row poff[l] + (i - off[l]).
__global__ void ivf_decode_kernel(const IvfDecodeArgs a) {
  const uint32_t l = blockIdx.x;
  const uint64_t b = a.list_off[l], e = a.list_off[l + 1];
  const uint64_t pb = a.poff[l];
  const float up = ldexpf(1.f, a.scale_log2);
  const float* c = a.coarse + static_cast<size_t>(l) * a.cstride;
  const int dim = a.m * a.dsub;
  for (uint64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
    const uint8_t* code = a.codes + i * a.m;
    uint4* out = reinterpret_cast<uint4*>(a.operand + (pb + (i - b)) * a.kpad);
    float nn = 0.f, cr = 0.f;
    for (int d0 = 0; d0 < a.kpad; d0 += 8) {
      __align__(16) __half h[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int d = d0 + u;
        float r = 0.f;
        if (d < dim) {
          const int j = d / a.dsub, t = d - j * a.dsub;
          r = a.centroids[(static_cast<size_t>(j) * 256 + code[j]) * a.dsub + t];
          nn = fmaf(r, r, nn);
          cr = fmaf(c[d], r, cr);
        }
        h[u] = __float2half_rn(r * up);
      }
      out[d0 / 8] = *reinterpret_cast<const uint4*>(h);
    }
    a.rowterm[pb + (i - b)] = fmaf(2.f, cr, nn);
  }
}

// Pairs (query q, probe p < np) per list.
__global__ void ivf_pair_count_kernel(const uint32_t* probe_ids, int nq, int nprobe, int np, uint32_t nlist,
                                      uint32_t* counts) {
  const int x = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (x >= nq * np) return;
  const int q = x / np, p = x % np;
  const uint32_t l = probe_ids[static_cast<size_t>(q) * nprobe + p];
  if (l < nlist) atomicAdd(&counts[l], 1u);
}

// tiles[l] = ceil(counts[l] / 128), then an exclusive scan of tiles[0..n) (n = nlist + 1, the last
// entry 0 so that tiles[nlist] ends as the total), by one block of 1024 threads.
__global__ void __launch_bounds__(1024) ivf_tile_scan_kernel(const uint32_t* counts, uint32_t nlist,
                                                             uint32_t* tiles) {
  __shared__ uint32_t part[1024];
  const uint32_t n = nlist + 1;
  const uint32_t per = (n + 1023) / 1024;
  const uint32_t b = threadIdx.x * per, e = b + per < n ? b + per : n;
  uint32_t sum = 0;
  for (uint32_t i = b; i < e; ++i) sum += i < nlist ? (counts[i] + 127) / 128 : 0u;
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
    tiles[i] = run;
    run += i < nlist ? (counts[i] + 127) / 128 : 0u;
  }
}

// Places every pair in a slot of its list's tiles (the rank within the list from an atomic
// cursor: any order serves, a query's result does not depend on its slot).
__global__ void ivf_place_kernel(const IvfTileArgs a) {
  const int x = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (x >= a.nq * a.np) return;
  const int q = x / a.np, p = x % a.np;
  const size_t pair = static_cast<size_t>(q) * a.nprobe + p;
  const uint32_t l = a.probe_ids[pair];
  if (l >= a.nlist) return;
  const uint32_t r = atomicAdd(&a.cursor[l], 1u);
  const uint32_t tile = a.tile_start[l] + r / 128;
  const uint32_t slot = tile * 128 + r % 128;
  a.slot_query[slot] = static_cast<uint32_t>(q);
  a.slot_offset[slot] = a.probe_dist[pair];
  if (a.pair_slot != nullptr) a.pair_slot[pair] = slot;
  if (r % 128 == 0) {
    const uint64_t b = a.poff[l];
    uint64_t size = a.list_off[l + 1] - a.list_off[l];
    if (a.row_cap != 0 && size > a.row_cap) size = a.row_cap;
    a.unit_rows[tile] = make_int2(static_cast<int>(b), static_cast<int>(b + size));
  }
}

// Gathered query operand: row s = the prepared operand row of slot s's query (zero when none).
__global__ void ivf_gather_kernel(const uint4* __restrict__ operand, const float* __restrict__ qscale,
                                  const uint32_t* __restrict__ slot_query, uint32_t nslots, int row_vecs,
                                  uint4* out, float* out_scale) {
  const uint64_t x = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t s = x / row_vecs;
  const int v = static_cast<int>(x % row_vecs);
  if (s >= nslots) return;
  const uint32_t q = slot_query[s];
  out[x] = q != 0xFFFFFFFFu ? operand[static_cast<uint64_t>(q) * row_vecs + v] : make_uint4(0, 0, 0, 0);
  if (v == 0) out_scale[s] = q != 0xFFFFFFFFu ? qscale[q] : -1.f;
}

}  // namespace

cudaError_t LaunchIvfDecode(const IvfDecodeArgs& a, cudaStream_t st) {
  if (a.nlist == 0) return cudaSuccess;
  if (a.m * a.dsub > a.kpad) return cudaErrorInvalidValue;
  NoteLaunch();
  ivf_decode_kernel<<<a.nlist, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchIvfTiles(const IvfTileArgs& a, uint32_t* counts, cudaStream_t st) {
  if (a.nq <= 0 || a.np <= 0) return cudaSuccess;
  const int pairs = a.nq * a.np;
  cudaError_t e = cudaMemsetAsync(counts, 0, a.nlist * sizeof(uint32_t), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(a.cursor, 0, a.nlist * sizeof(uint32_t), st);
  if (e != cudaSuccess) return e;
  NoteLaunch();
  ivf_pair_count_kernel<<<(pairs + 255) / 256, 256, 0, st>>>(a.probe_ids, a.nq, a.nprobe, a.np, a.nlist, counts);
  NoteLaunch();
  ivf_tile_scan_kernel<<<1, 1024, 0, st>>>(counts, a.nlist, a.tile_start);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  NoteLaunch();
  ivf_place_kernel<<<(pairs + 255) / 256, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t LaunchIvfGather(const void* operand, const float* qscale, const uint32_t* slot_query, uint32_t nslots,
                            int kpad, void* out, float* out_scale, cudaStream_t st) {
  if (nslots == 0) return cudaSuccess;
  const int row_vecs = kpad * 2 / 16;
  const uint64_t total = static_cast<uint64_t>(nslots) * row_vecs;
  NoteLaunch();
  ivf_gather_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      static_cast<const uint4*>(operand), qscale, slot_query, nslots, row_vecs, static_cast<uint4*>(out), out_scale);
  return cudaGetLastError();
}

}  // namespace vdbgpu
