// IVF-PQ / PQ-flat ADC scan with re-rank (one CTA per query).
#pragma once

#include <cuda_fp16.h>
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

// ------------------------------------------------------------------ tensor-core pre-rank (ivf_mma.cu)

// The decoded residual operand of list mode: row i of list l (codes in list order) becomes operand
// row poff[l] + (i - list_off[l]) (poff: list starts rounded up to 32 rows), the concatenated
// centroids C_j[code_j] as fp16 scaled by 2^scale_log2 (zero past m * dsub), with the row term
// ||r||^2 + 2 <c_l, r> in fp32. Pad rows are left as they are (zeroed by the caller).
struct IvfDecodeArgs {
  const uint8_t* codes;
  const uint64_t* list_off;  // nlist + 1
  const uint64_t* poff;      // nlist + 1
  uint32_t nlist;
  int m, dsub, kpad, cstride;  // kpad a multiple of 8; cstride: coarse row stride (floats)
  const float* centroids;    // m x 256 x dsub
  const float* coarse;       // nlist x cstride
  int scale_log2;
  __half* operand;           // poff[nlist] rows x kpad
  float* rowterm;
};
cudaError_t LaunchIvfDecode(const IvfDecodeArgs& a, cudaStream_t st);

// One batch's query tiles: every pair (query q, probe p < np) takes a slot of one of its list's
// tiles of 128 (tile_start[l] = the list's first tile, tile_start[nlist] = the tile count);
// slot_query / slot_offset (the coarse distance) per slot, pair_slot per pair (optional), and
// each tile's row range in unit_rows. slot_query must hold 0xFFFFFFFF in every slot beforehand.
struct IvfTileArgs {
  int nq, nprobe, np;
  uint32_t nlist;
  const uint32_t* probe_ids;  // nq x nprobe
  const float* probe_dist;    // nq x nprobe
  const uint64_t* list_off;   // nlist + 1
  const uint64_t* poff;       // nlist + 1
  uint32_t* cursor;           // nlist (scratch)
  uint32_t* tile_start;       // nlist + 1
  uint32_t* slot_query;
  float* slot_offset;
  uint32_t* pair_slot;        // nq x nprobe, or null
  int2* unit_rows;
  uint32_t row_cap;           // a tile covers at most its list's first row_cap rows (0: all)
};
// counts: nlist words of scratch. Tiles number at most nq * np / 128 + nlist.
cudaError_t LaunchIvfTiles(const IvfTileArgs& a, uint32_t* counts, cudaStream_t st);
// out (nslots x kpad fp16) = the operand rows of the slots' queries, out_scale their qscale.
cudaError_t LaunchIvfGather(const void* operand, const float* qscale, const uint32_t* slot_query, uint32_t nslots,
                            int kpad, void* out, float* out_scale, cudaStream_t st);

// The exact stage after the list-mode scan, one warp per query: the entries of the query's
// nprobe x wgs candidate lists below its bound, the cpre best of them by pre-rank key, their
// reference ADC distances (precomputed or residual L2 tables, four partial sums, plus the coarse
// distance with the precomputed ones), TopK(R = max(depth, k)) by (dist, id), the re-rank on fp32
// rows when depth > 0, and the k best. Entries below the bound beyond shared memory's room are
// cut to the cpre best by a radix select over the lists.
struct IvfFinalizeArgs {
  int nq, nprobe, pd, dim, m, dsub, k, depth, cpre, order, mode, wgs;
  uint64_t nlist;
  const uint32_t* pair_slot;  // nq x nprobe
  const uint2* cand;
  const int* cand_count;
  const uint32_t* qtau;
  const uint32_t* probe_ids;
  const float* probe_dist;
  const uint64_t* list_off;
  const uint64_t* poff;
  const uint32_t* ids;
  const uint8_t* codes;
  const float* centroids;
  const float* term2;
  const float* coarse;
  const float* queries;
  const float* rows;
  float* out_dist;
  uint32_t* out_row;
  uint64_t* out_dc;
  // Optional (stage timing): [0] entries below the bounds, [1] queries cut by the radix select,
  // [2..4] warp cycles in the gather / ADC / TopK and re-rank, summed over queries.
  unsigned long long* counters;
};
cudaError_t LaunchIvfFinalize(const IvfFinalizeArgs& a, cudaStream_t st);

}  // namespace vdbgpu
