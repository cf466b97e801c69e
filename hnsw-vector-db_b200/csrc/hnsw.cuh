// Batched HNSW beam search (one warp per query) over the reference's serialized graphs.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vdbgpu {

// One segment's graph, for walks over several segments in one launch.
struct HnswSegment {
  const float* rows;
  const uint8_t* codes;
  const float* vmin;
  const float* scale;
  const uint32_t* links0;
  const uint32_t* upper;
  const uint64_t* upper_off;
  const uint8_t* level;
  uint64_t n;
  uint32_t entry;
  int max_level;
};

// One walk of a multi-segment launch: segment, query row, allowed rows, and the output slot
// (keys at slot * k, distance computations and the short flag at slot).
struct HnswItem {
  uint32_t seg;
  uint32_t query;
  const uint32_t* allow;
  uint64_t slot;
  uint32_t need;  // fewer results than this sets the short flag (the exact fallback)
  uint32_t pad;
};

struct HnswArgs {
  int nq, pd;
  int k;           // results written per query
  int k_graph;     // results the graph search keeps (HnswSq8: max(depth, k))
  int ef;          // beam width (already max(ef, k_graph))
  int depth;       // HNSW-SQ8 re-rank depth on fp32 rows (0 = none)
  int metric;      // 0 = L2, else minus the dot product
  int order;       // SumOrder of the reference kernel set
  const float* queries;
  const float* rows;       // fp32 rows (float space, re-rank)
  const uint8_t* codes;    // SQ8 codes (SQ8 space) or null
  const float* vmin;
  const float* scale;
  const uint32_t* links0;  // cap * (1 + M0)
  uint32_t M0;
  const uint32_t* upper;
  const uint64_t* upper_off;
  const uint8_t* level;
  uint32_t M;
  int max_level;
  uint32_t entry;
  uint64_t n;              // nodes (graph capacity = rows)
  const uint32_t* allow;   // allowed-row bitset (32 per word) or null
  int hash_bits;           // visited hash: 1 << hash_bits slots per warp
  int cand_cap;            // candidate array capacity per warp
  int warps;               // queries (warps) per block, 1..4
  // Pooled mode (large walks, e.g. filtered): visited bits and overflow candidates in global memory.
  int pooled;
  uint32_t* visited;       // nq x vwords bitmaps, zeroed before the launch
  uint64_t vwords;
  uint64_t* pool;          // nq x pool_cap candidate keys
  int pool_cap;
  // Multi-segment mode (segs non-null): warp i walks items[i] over segs[items[i].seg] and writes
  // packed (dist, row) keys to out_keys, its count to out_dc and the short flag to out_short.
  const HnswSegment* segs;
  const HnswItem* items;
  uint64_t* out_keys;
  int* out_short;
  // Work counters (null = off): [0] walks, [1] expansions, [2] front refills, [3] pool slots scanned
  // by refills, [4] merges into the front, [5] result inserts, [6] most expansions of one walk.
  unsigned long long* counters;
  int step_limit;          // bounded walk: expansions per query
  float* out_dist;
  uint32_t* out_row;
  uint64_t* out_dc;        // distance computations per query (device) or null
  int* status;
};

// Pooled mode: sorted candidates kept in shared memory (the rest wait in the global pool).
constexpr int kPoolFront = 96;
constexpr int kPoolRefill = 64;
constexpr int kPoolFrontSlots = 128 + 8;  // 128 sort slots + a 16-counter histogram

// Shared memory of one query's warp: query, visited hash, results, candidates, neighbour scratch.
__host__ __device__ inline size_t HnswWarpSmemBytes(int pd, int hash_bits, int ef, int cand_cap) {
  // The hash holds at least 2 slots so the 8-byte arrays after it stay 8-byte aligned.
  const size_t slots = hash_bits < 1 ? 2 : (static_cast<size_t>(1) << hash_bits);
  const size_t b = static_cast<size_t>(pd) * 4 + slots * 4 +
                   static_cast<size_t>(ef) * 8 + static_cast<size_t>(cand_cap) * 8 + 32 * 4 + 32 * 4;
  return (b + 15) / 16 * 16;
}
cudaError_t LaunchHnswSearch(const HnswArgs& a, cudaStream_t stream);

}  // namespace vdbgpu
