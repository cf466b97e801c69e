// Flat / SQ8-flat search without any device allocation, for callers that must not allocate
// device memory while they search.
//
// Some hosts cannot let a library call cudaMalloc on their search path: a serving process whose
// device memory is owned by its own allocator (a framework's caching allocator, a preallocated
// pool) would see allocations it does not account for, and cudaMalloc may synchronise the device
// or fail under memory pressure in the middle of a request. This variant of the tensor-core scan
// (scan_mma.cu + select.cu) therefore takes its scratch from a fixed array compiled into the
// library instead of the context's workspace:
//   * g_scratch below is a file-scope __device__ array of kNoAllocScratchBytes (about 8.4 MB);
//     every GPU that loads the library holds it until the process exits;
//   * its device address is looked up once per device with cudaGetSymbolAddress, on the first call
//     made on that device (with the device current);
//   * limits: at most 128 queries per call, padded dimension at most 256, at most 16 row slices,
//     k and the candidate depth as in the regular entry point; larger requests are rejected. With
//     16 slices the scan keeps at most 16 of the GPU's 148 SMs busy: the entry point is sized for
//     small latency-bound batches, not for throughput;
//   * an empty index gives misses (+inf, UINT32_MAX) in every slot, as the regular search does;
//   * every call shares the one array and keeps the previous call's contents: the per-query
//     thresholds are reset at the start of each call, everything else is fully rewritten before it
//     is read. Calls whose work overlaps on the GPU (on different streams, or from different
//     contexts on the same device) race on the array and must be serialised by the caller.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "kernels.cuh"
#include "noalloc.h"
#include "scan_mma.cuh"

namespace vdbgpu {
namespace {

constexpr size_t Align256(size_t x) { return (x + 255) / 256 * 256; }

constexpr size_t kOffOperand = 0;
constexpr size_t kOffQScale = Align256(kOffOperand + size_t(kNoAllocMaxQueries) * kNoAllocMaxKpad * 2);
constexpr size_t kOffQTau = Align256(kOffQScale + size_t(kNoAllocMaxQueries) * 4);
constexpr size_t kOffCount = Align256(kOffQTau + size_t(kNoAllocMaxQueries) * 4);
constexpr size_t kOffCand =
    Align256(kOffCount + size_t(kNoAllocMaxUnits) * kScanBM * sizeof(int));
constexpr size_t kScratchEnd =
    kOffCand + size_t(kNoAllocMaxUnits) * kScanBM * kScanCap * sizeof(uint2);

static __device__ __align__(256) unsigned char g_scratch[kScratchEnd];

std::mutex g_mu;
void* g_addr[kNoAllocMaxDevices] = {};

// Misses for every slot (+inf, UINT32_MAX), as the regular search returns them for an empty index.
__global__ void fill_misses_kernel(float* dist, uint32_t* row, uint64_t n) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
    dist[i] = __int_as_float(0x7f800000);
    row[i] = 0xFFFFFFFFu;
  }
}

}  // namespace

const size_t kNoAllocScratchBytes = kScratchEnd;

Status NoAllocScratch(int device, void** out) {
  if (device < 0 || device >= kNoAllocMaxDevices)
    return Status(Status::kInvalidArgument, "device ordinal out of range for the fixed scratch");
  std::lock_guard<std::mutex> g(g_mu);
  if (g_addr[device] == nullptr) {
    // The symbol's host-side name is only a stand-in; the device address comes from the runtime,
    // per device, with that device current (the caller made it current).
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return Status(Status::kInternal, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    }
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return Status::OK();
}

Status ScanSearchNoAlloc(Context& ctx, const ScanOperands& op, int metric, uint32_t pd,
                         const SearchBatch& b, int cpre, int depth, cudaStream_t stream) {
  if (b.nq == 0) return Status::OK();
  if (b.nq > kNoAllocMaxQueries)
    return Status(Status::kInvalidArgument, "the allocation-free search takes at most 128 queries per call");
  if (op.kpad > kNoAllocMaxKpad)
    return Status(Status::kInvalidArgument, "the allocation-free search supports padded dimensions up to 256");
  if (op.rows == 0) {
    const uint64_t n = b.nq * b.k;
    NoteLaunch();
    fill_misses_kernel<<<static_cast<unsigned>(std::min<uint64_t>((n + 255) / 256, 1024)), 256, 0, stream>>>(
        b.out_dist, b.out_row, n);
    return CudaStatus(cudaGetLastError(), "fill misses");
  }
  if (cpre > kScanCap - 64) return Status(Status::kNotSupported, "candidate depth too large");
  void* base = nullptr;
  VDBGPU_RETURN_IF_ERROR(NoAllocScratch(ctx.device(), &base));
  uint8_t* s = static_cast<uint8_t*>(base);
  void* a_op = s + kOffOperand;
  float* qscale = reinterpret_cast<float*>(s + kOffQScale);
  uint32_t* qtau = reinterpret_cast<uint32_t*>(s + kOffQTau);
  int* cnt = reinterpret_cast<int*>(s + kOffCount);
  uint2* cand = reinterpret_cast<uint2*>(s + kOffCand);

  const uint64_t nq = b.nq;
  const uint64_t nq_pad = kScanBM;  // one query tile
  // Thresholds must start "unset" on every call (the array keeps the last call's values).
  VDBGPU_CUDA(cudaMemsetAsync(qtau, 0xFF, nq * sizeof(uint32_t), stream));

  PrepArgs pa{};
  pa.nq = static_cast<int>(nq);
  pa.nq_pad = static_cast<int>(nq_pad);
  pa.pd = static_cast<int>(pd);
  pa.kpad = static_cast<int>(op.kpad);
  pa.kind = op.prep_kind;
  pa.ab_format = op.ab_format;
  pa.key_factor = op.key_factor;
  pa.row_scale_log2 = op.row_scale_log2;
  pa.queries = b.queries;
  pa.vmin = op.vmin;
  pa.scale = op.scale;
  pa.operand = a_op;
  pa.qscale = qscale;
  VDBGPU_CUDA(LaunchPrepQueries(pa, stream));

  CUtensorMap amap;
  VDBGPU_RETURN_IF_ERROR(ctx.EncodeOperandMap(&amap, a_op, nq_pad, op.kpad, kScanBM, op.ab_format));
  // Row slices: one CTA each, at most kNoAllocMaxUnits of them.
  const uint64_t ntiles = (op.rows + kScanBN - 1) / kScanBN;
  const uint64_t max_u = std::min<uint64_t>({ntiles, static_cast<uint64_t>(kNoAllocMaxUnits),
                                             static_cast<uint64_t>(ctx.sm_count())});
  const uint64_t tpu = (ntiles + max_u - 1) / max_u;
  const uint64_t upq = (ntiles + tpu - 1) / tpu;

  ScanArgs sa{};
  sa.nq = static_cast<int>(nq);
  sa.nrows = static_cast<int>(op.rows);
  sa.kblocks = static_cast<int>(op.kpad / kScanBK);
  sa.mode = op.rowterm != nullptr ? kKeyRowTerm : kKeyScaled;
  sa.ab_format = op.ab_format;
  sa.keep = cpre;
  sa.units_per_qtile = static_cast<int>(upq);
  sa.rows_per_unit = static_cast<int>(tpu * kScanBN);
  sa.nunits = static_cast<int>(upq);
  sa.qscale = qscale;
  sa.rowterm = op.rowterm;
  sa.allow = b.allow;
  sa.wgs = 1;
  sa.counters = nullptr;
  sa.cand = cand;
  sa.cand_count = cnt;
  sa.qtau = qtau;
  sa.status = ctx.status_word();
  VDBGPU_CUDA(LaunchScan(amap, op.b_map, sa, static_cast<int>(upq), stream));

  FinalizeArgs fa{};
  fa.nq = static_cast<int>(nq);
  fa.pd = static_cast<int>(pd);
  fa.k = static_cast<int>(b.k);
  fa.cpre = cpre;
  fa.depth = depth;
  fa.metric = metric;
  fa.order = ctx.order();
  fa.units_per_qtile = static_cast<int>(upq);
  fa.wgs = 1;
  fa.cand = cand;
  fa.cand_count = cnt;
  fa.qtau = qtau;
  fa.queries = b.queries;
  fa.rows = op.rows_f32;
  fa.codes = op.codes;
  fa.vmin = op.vmin;
  fa.scale = op.scale;
  fa.out_dist = b.out_dist;
  fa.out_row = b.out_row;
  VDBGPU_CUDA(LaunchFinalize(fa, stream));
  return Status::OK();
}

}  // namespace vdbgpu
