// GPU construction of HNSW graphs in the reference's file format (hnsw_build.cc / .cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vdbgpu {

struct PruneArgs {
  const float* rows;  // layer rows, n x pd (node i of the layer at row i)
  int pd;
  int metric;         // 0 = L2, else minus the dot product
  uint64_t n;         // nodes of the layer (candidate ids are below n)
  // select: nodes [node_base, node_base + n_select) take forward links (n_select 0 = all n); their
  // candidates and output rows are indexed from node_base
  uint64_t node_base;
  uint64_t n_select;
  // select: node i's candidates cand_ids / cand_d [i * kc, (i + 1) * kc), sorted by (dist, id)
  const uint32_t* cand_ids;
  const float* cand_d;
  int kc;
  // merge: forward lists (count + ids, stride fwd_stride) and reverse adjacency (CSR)
  const uint32_t* fwd;
  int fwd_stride;
  const uint64_t* rev_off;
  const uint32_t* rev_ids;
  int maxm;           // links kept per node
  uint32_t* out;      // count + ids per node, stride out_stride
  int out_stride;
};

size_t PruneSmemBytes(int pd, int maxm);
cudaError_t LaunchSelect(const PruneArgs& a, cudaStream_t st);
cudaError_t LaunchReverse(const uint32_t* fwd, int stride, uint64_t n, uint32_t* cnt, cudaStream_t st);
// Back links of sources [0, n): the reverse entry of source u is src_base + u.
cudaError_t LaunchFillReverse(const uint32_t* fwd, int stride, uint64_t n, const uint64_t* off, uint32_t* cursor,
                              uint32_t* rev, cudaStream_t st, uint32_t src_base = 0);
cudaError_t LaunchMergeLinks(const PruneArgs& a, cudaStream_t st);
cudaError_t LaunchGatherRows(const float* rows, const uint32_t* ids, uint64_t n, int pd, float* out, cudaStream_t st);

}  // namespace vdbgpu
