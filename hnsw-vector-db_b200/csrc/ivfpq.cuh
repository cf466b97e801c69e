// IVF-PQ / PQ-flat ADC scan with re-rank (one CTA per query).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vdbgpu {

enum IvfMode : int {
  kIvfPrecomputed = 0,  // L2 with precomputed term2 tables
  kIvfResidual = 1,     // L2, per-list residual tables
  kIvfShared = 2,       // inner product / cosine: one table, per-list offset -<q, c>
  kPqFlat = 3,          // PqFlatIndex: one table, every row, offset 0
};

struct IvfPqArgs {
  int nq, pd, dim, m, dsub;
  int k;
  int depth;      // re-rank depth R (0 = return ADC distances)
  int metric, order, nprobe, mode;
  uint64_t nlist, n;
  const float* queries;
  const float* rows;
  const float* coarse;     // nlist x pd
  const float* centroids;  // m x 256 x dsub
  const float* term2;      // nlist x m x 256 (precomputed mode)
  const uint64_t* list_off;
  const uint32_t* ids;
  const uint8_t* codes;    // list-major, m bytes per row
  const uint32_t* probe_ids;  // nq x nprobe
  const float* probe_dist;    // nq x nprobe (coarse distances)
  const uint32_t* allow;
  float* out_dist;
  uint32_t* out_row;
  uint64_t* out_dc;
  uint64_t* cand;             // IvfPqCandBytes(nq, k, depth) of candidate buffers
  const uint32_t* qorder;     // CTA b scans query qorder[b] (null: query b)
  int* status;
};

size_t IvfPqSmemBytes(int pd, int m, int mode);
size_t IvfPqCandBytes(int nq, int k, int depth);
// order[0..nq): the queries grouped by their first probed list; counts holds nlist + 1 words.
cudaError_t LaunchProbeOrder(const uint32_t* probe_ids, int nq, int nprobe, uint32_t nlist, uint32_t* counts,
                             uint32_t* order, cudaStream_t stream);
cudaError_t LaunchIvfPq(const IvfPqArgs& a, cudaStream_t stream);
cudaError_t LaunchTerm2(const float* coarse, uint32_t nlist, int pd, const float* centroids, int m,
                        int ds, float* term2, cudaStream_t stream);

}  // namespace vdbgpu
