// The allocation-free variant of the flat / SQ8-flat search (noalloc.cu).
#pragma once

#include <cuda_runtime.h>

#include "runtime.h"

namespace vdbgpu {

constexpr int kNoAllocMaxQueries = 128;
constexpr int kNoAllocMaxUnits = 16;
constexpr int kNoAllocMaxKpad = 256;
constexpr int kNoAllocMaxDevices = 64;
extern const size_t kNoAllocScratchBytes;

// Device address of the fixed scratch array on `device` (which must be current); looked up with
// cudaGetSymbolAddress on the first call per device.
Status NoAllocScratch(int device, void** out);

// The tensor-core scan + exact finalize of ScanSearch, using only the fixed scratch array.
// Everything is launched on `stream`; nothing is allocated.
Status ScanSearchNoAlloc(Context& ctx, const ScanOperands& op, int metric, uint32_t pd,
                         const SearchBatch& b, int cpre, int depth, cudaStream_t stream);

}  // namespace vdbgpu
