// Tensor-core scan with a fused streaming top-C selection: the pre-rank stage of exact flat
// search and of the exhaustive SQ8 scan.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace vdbgpu {

constexpr int kScanBM = 128;      // queries per tile: TMEM lanes, M of the MMA
constexpr int kScanBN = 256;      // rows per tile: TMEM columns of one accumulator, N of the MMA
constexpr int kScanBK = 64;       // fp16 elements per k-block (one 128-byte swizzle atom)
constexpr int kScanStages = 4;    // B k-block stages in flight unless ScanArgs::stages says otherwise
constexpr int kScanMaxStages = 6;
constexpr int kScanMaxKB = 4;     // padded dims up to 256
#ifndef VDBGPU_SCAN_CAP
#define VDBGPU_SCAN_CAP 512
#endif
constexpr int kScanCap = VDBGPU_SCAN_CAP;  // candidate slots per (unit, query)
// warp 0 TMA, warp 1 MMA + TMEM owner, then 4 epilogue warps per epilogue warpgroup (1 or 2)
constexpr int ScanThreads(int wgs) { return 64 + 128 * wgs; }

// Key transform applied to the fp32 accumulator acc = sum_i A[q,i] * B[r,i]:
//   kKeyScaled:  key = qscale[q] * acc
//   kKeyRowTerm: key = fma(qscale[q], acc, rowterm[r])
//   kKeyList:    key = fma(qscale[s], acc, rowterm[r]) + slot_offset[s], list mode: unit u is
//                query tile u (operand rows s = 128 u + i, serving query slot_query[s]) against
//                rows unit_rows[u] = [x, y), x a multiple of 32 (IVF lists, each query tile
//                gathered from the queries probing one list)
// Smaller key = closer. Keys of one query are comparable across rows and units.
enum ScanKeyMode : int { kKeyScaled = 0, kKeyRowTerm = 1, kKeyList = 2 };

struct ScanArgs {
  int nq;               // valid queries
  int nrows;            // valid rows
  int kblocks;          // ceil(padded_dim / 64)
  int mode;             // ScanKeyMode
  int ab_format;        // 0 = fp16, 1 = bf16 (both operands)
  int keep;             // candidates kept per compaction (C), < kScanCap - 32
  int compact_at;       // list length that triggers a compaction, <= kScanCap - 32 (0 = that)
  int stages;           // B k-block stages in flight, 1..kScanMaxStages (0 = kScanStages)
  int chunk_best;       // 1: each 32-row chunk contributes only its best key, filed under the chunk's
                        // first row (seeding sample scans); 2: under the key's own row (nearest rows;
                        // one epilogue warpgroup)
  int units_per_qtile;  // row slices per 128-query tile
  int rows_per_unit;    // multiple of kScanBN
  int nunits;           // qtiles * units_per_qtile
  const float* qscale;  // [nq]
  const float* rowterm; // [round_up(nrows, 256)] (kKeyRowTerm) or null
  const uint32_t* allow;// allowed-row bitset, 32 rows per word, padded to 256 rows; null = all
  int wgs;              // epilogue warpgroups (1 or 2); each keeps its own candidate lists
  uint2* cand;          // [nunits][wgs][128][kScanCap] (float key bits, row)
  int* cand_count;      // [nunits][wgs][128]
  unsigned long long* counters;  // optional: chunks, triggered chunks, inserts, compactions
  uint32_t* qtau;       // [nq] shared per-query threshold (ordered-key space), 0xFFFFFFFF = none
  int* status;          // device status word
  // List mode (kKeyList) only.
  const int2* unit_rows;       // [nunits] row range of each unit
  const uint32_t* slot_query;  // [nq] query served by each operand row (0xFFFFFFFF: none)
  const float* slot_offset;    // [nq] key offset of each operand row
};

// Launches the scan on `stream`. tmap_a: queries operand [qpad x kpad] K-major, box {64, 128};
// tmap_b: rows operand [nrows x kpad] K-major, box {64, 256}; both SWIZZLE_128B.
cudaError_t LaunchScan(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const ScanArgs& a,
                       int grid, cudaStream_t stream);

// Dynamic shared memory of a scan with `stages` B stages (0 = kScanStages).
size_t ScanSmemBytes(int kblocks, int stages = 0);
// The most B stages (<= kScanMaxStages) that fit next to the query tile in 227 KB.
int ScanMaxStagesFor(int kblocks);

}  // namespace vdbgpu
