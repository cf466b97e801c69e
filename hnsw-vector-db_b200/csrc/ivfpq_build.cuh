// GPU kernels of the IVF-PQ builder (ivfpq_build.cu, driven by ivfpq_build_host.cc): the
// nearest-centroid assignments of the reference's k-means and the PQ encoding, each distance summed
// in the reference's order so every argmin (first minimum over ascending centroid numbers) is the
// reference's.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vdbgpu {

// Distance kinds of AssignNearest (src/index/quant/kmeans.cc:16-20, PickL2): the runtime kernel
// set's L2 for rows whose length and stride are multiples of 16 floats, else L2SqAny.
enum AssignDist : int { kAssignRuntime = 0, kAssignAny = 1 };

struct AssignArgs {
  const float* points;     // n rows of d floats, row stride `stride` floats
  uint64_t n;
  int d, stride;
  const float* centroids;  // k x d
  int k;
  int kind;                // AssignDist
  int order;               // SumOrder of the runtime kernel set (kAssignRuntime)
  uint32_t* assign;        // n
  float* dist;             // n or null
};
// d <= kAssignMaxDim.
constexpr int kAssignMaxDim = 256;
cudaError_t LaunchAssignNearest(const AssignArgs& a, cudaStream_t st);

struct PqEncodeArgs {
  const float* rows;       // n x pd
  uint64_t n;
  int pd, dim;
  const float* coarse;     // nlist x pd, or null (PQ-flat: codes of the rows themselves)
  const uint32_t* assign;  // n (list of each row), with coarse
  const float* pq;         // m x 256 x dsub
  int m, dsub;
  uint8_t* codes;          // n x m
};
cudaError_t LaunchPqEncode(const PqEncodeArgs& a, cudaStream_t st);

}  // namespace vdbgpu
