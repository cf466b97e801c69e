// Host-callable launchers of the search-path kernels (all run on the caller's stream).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace vdbgpu {

// ------------------------------------------------------------------ flat / SQ8 finalize

struct FinalizeArgs {
  int nq, pd, k;
  int cpre;             // candidates recomputed exactly (<= 256)
  int depth;            // SQ8: re-rank depth on fp32 rows (0 = return SQ8 distances)
  int metric;           // 0 = L2, else minus the dot product
  int order;            // SumOrder of the reference kernel set
  int units_per_qtile;
  int wgs;              // candidate lists per unit (scan epilogue warpgroups)
  const uint2* cand;
  const int* cand_count;
  const uint32_t* qtau;
  const float* queries;  // nq x pd fp32
  const float* rows;     // n x pd fp32
  const uint8_t* codes;  // SQ8 codes (n x pd) or null for flat
  const float* vmin;
  const float* scale;
  float* out_dist;
  uint32_t* out_row;
  // Seeded scans: a query whose lists hold fewer than cpre keys below its final bound is
  // appended to fb_list (the seed was too tight; its result must come from an unseeded scan).
  uint32_t* fb_list;
  int* fb_count;
};
cudaError_t LaunchFinalize(const FinalizeArgs& a, cudaStream_t stream);

// Seed of a scan's per-query bound: the m-th smallest key (ordered) among the candidate lists
// a scan of a row sample left for the query (units_per_qtile x wgs lists of the FinalizeArgs
// layout), written to qtau_out[q], which holds that sample scan's own bound on entry;
// 0xFFFFFFFF when fewer than m keys lie below that bound.
struct SeedArgs {
  int nq;
  int m;
  int units_per_qtile;
  int wgs;
  const uint2* cand;
  const int* cand_count;
  uint32_t* qtau_out;
};
cudaError_t LaunchScanSeed(const SeedArgs& a, cudaStream_t stream);

// out_dist / out_row rows list[i] (k each) = src rows i, i < n.
cudaError_t LaunchScatterResults(const float* src_dist, const uint32_t* src_row, const uint32_t* list,
                                 uint32_t n, int k, float* out_dist, uint32_t* out_row,
                                 cudaStream_t stream);

enum PrepKind : int { kPrepFlat = 0, kPrepSq8Ip = 1, kPrepSq8L2 = 2 };

struct PrepArgs {
  int nq, nq_pad, pd, kpad;
  int kind;        // PrepKind
  int ab_format;   // 0 = fp16 (scaled by a power of two), 1 = bf16
  int key_factor;  // 2 for L2 keys (-2 * acc + row term), 1 for dot keys (-acc)
  int row_scale_log2;  // the row operand was scaled by 2^row_scale_log2
  const float* queries;
  const float* vmin;
  const float* scale;
  void* operand;   // nq_pad x kpad
  float* qscale;   // nq
};
cudaError_t LaunchPrepQueries(const PrepArgs& a, cudaStream_t stream);
// Row operand (fp16 scaled by 2^scale_log2, or bf16) and squared norms of the unscaled rows.
cudaError_t LaunchPrepRows(const float* rows, uint64_t n, int pd, int kpad, int ab_format,
                           int scale_log2, void* operand, float* norms, cudaStream_t stream);
cudaError_t LaunchAbsMax(const float* x, uint64_t count, uint32_t* out, cudaStream_t stream);

cudaError_t LaunchSq8MinMax(const float* rows, uint64_t n, int dim, int pd, uint32_t* kmin,
                            uint32_t* kmax, cudaStream_t stream);
cudaError_t LaunchSq8Encode(const float* rows, uint64_t n, int dim, int pd, int kpad,
                            const float* vmin, const float* scale, uint8_t* codes, __half* operand,
                            float* rowterm, cudaStream_t stream);
cudaError_t LaunchSq8Operand(const uint8_t* codes, uint64_t n, int pd, int kpad, const float* scale,
                             __half* operand, float* rowterm, cudaStream_t stream);

}  // namespace vdbgpu
