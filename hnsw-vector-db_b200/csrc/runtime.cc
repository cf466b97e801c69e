// Host runtime: device buffers, contexts, tensor-map encoding and kernel-set detection.
#include "runtime.h"

#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

namespace vdbgpu {

Status CudaStatus(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::OK();
  const Status::Code c = e == cudaErrorMemoryAllocation ? Status::kResourceExhausted
                         : (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
                             ? Status::kUnavailable
                             : Status::kInternal;
  return Status(c, std::string(what) + ": " + cudaGetErrorString(e));
}

Status DeviceBuffer::alloc(size_t bytes) {
  reset();
  if (bytes == 0) return Status::OK();
  cudaError_t e = cudaMalloc(&p_, bytes);
  if (e != cudaSuccess) {
    p_ = nullptr;
    (void)cudaGetLastError();
    return CudaStatus(e, "cudaMalloc");
  }
  n_ = bytes;
  return Status::OK();
}

void DeviceBuffer::reset() {
  if (p_ != nullptr) cudaFree(p_);
  p_ = nullptr;
  n_ = 0;
}

// The reference picks the fastest kernel set the CPU supports, or VDB_KERNELS when it names an
// available one (src/distance/cpu_features.cc:27-42): scalar < avx2 (needs avx2+fma) < avx512
// (needs avx512f too). Distances re-ranked on the GPU are summed in that set's order so they
// match the reference bit for bit on the same host.
int DetectKernelOrder() {
  bool avx2 = false, avx512 = false;
#if defined(__x86_64__)
  __builtin_cpu_init();
  avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  avx512 = avx2 && __builtin_cpu_supports("avx512f");
#endif
  if (const char* env = std::getenv("VDB_KERNELS"); env != nullptr && *env != '\0') {
    if (std::strcmp(env, "scalar") == 0) return 0;
    if (std::strcmp(env, "avx2") == 0 && avx2) return 2;
    if (std::strcmp(env, "avx512") == 0 && avx512) return 1;
  }
  return avx512 ? 1 : (avx2 ? 2 : 0);
}

const char* KernelOrderName(int order) {
  return order == 1 ? "avx512" : order == 2 ? "avx2" : "scalar";
}

namespace {
std::atomic<uint64_t> g_launches{0};
}  // namespace

void NoteLaunch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t LaunchCount() { return g_launches.load(std::memory_order_relaxed); }

MemWhere WherePointer(const void* p, int device) {
  if (p == nullptr) return MemWhere::kHost;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return MemWhere::kHost;
  }
  if (a.type == cudaMemoryTypeManaged) return MemWhere::kDevice;
  if (a.type == cudaMemoryTypeDevice) return a.device == device ? MemWhere::kDevice : MemWhere::kOtherDevice;
  return MemWhere::kHost;
}

Status RejectOtherDevice(const void* p, int device, const char* what) {
  if (WherePointer(p, device) != MemWhere::kOtherDevice) return Status::OK();
  cudaPointerAttributes a{};
  (void)cudaPointerGetAttributes(&a, p);
  return Status(Status::kInvalidArgument, std::string(what) + " is memory of device " + std::to_string(a.device) +
                                              "; this index lives on device " + std::to_string(device));
}

Status Context::Open(int device, std::unique_ptr<Context>* out) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    (void)cudaGetLastError();
    return Status(Status::kUnavailable, "no CUDA device is available");
  }
  if (device < 0 || device >= count) return Status(Status::kInvalidArgument, "bad device ordinal");
  std::unique_ptr<Context> c(new Context());
  c->device_ = device;
  VDBGPU_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  VDBGPU_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) {
    return Status(Status::kNotSupported,
                  "this library is built for sm_100a (B200); device is sm_" +
                      std::to_string(prop.major) + std::to_string(prop.minor));
  }
  c->sm_count_ = prop.multiProcessorCount;
  VDBGPU_CUDA(cudaStreamCreateWithFlags(&c->stream_, cudaStreamNonBlocking));
  VDBGPU_RETURN_IF_ERROR(c->status_.alloc(sizeof(int)));
  VDBGPU_CUDA(cudaMemset(c->status_.get(), 0, sizeof(int)));
  cudaDriverEntryPointQueryResult q;
  VDBGPU_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &c->encode_fn_, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || c->encode_fn_ == nullptr)
    return Status(Status::kUnavailable, "cuTensorMapEncodeTiled is not available");
  c->order_ = DetectKernelOrder();
  if (const char* w = std::getenv("VDB_SCAN_WARPGROUPS"); w != nullptr && *w != 0)
    c->scan_wgs_ = std::strcmp(w, "2") == 0 ? 2 : 1;
  if (const char* v = std::getenv("VDB_SCAN_STAGES"); v != nullptr && *v != 0)
    c->scan_stages_ = std::max(0, static_cast<int>(std::strtol(v, nullptr, 10)));
  *out = std::move(c);
  return Status::OK();
}

Status Context::EnableTiming(bool on) {
  if (on && marks_[0] == nullptr)
    for (int i = 0; i < kMaxMarks; ++i) VDBGPU_CUDA(cudaEventCreate(&marks_[i]));
  if (on && counters_.get() == nullptr) {
    VDBGPU_RETURN_IF_ERROR(counters_.alloc(8 * sizeof(unsigned long long)));
    VDBGPU_CUDA(cudaMemset(counters_.get(), 0, 8 * sizeof(unsigned long long)));
  }
  timing_ = on;
  return Status::OK();
}

int Context::Counters(unsigned long long* out, int cap) {
  if (!timing_ || counters_.get() == nullptr) return 0;
  unsigned long long h[8] = {};
  if (cudaMemcpy(h, counters_.get(), sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  const int n = cap < 8 ? cap : 8;
  for (int i = 0; i < n; ++i) out[i] = h[i];
  return n;
}

int Context::StageTimes(float* out, int cap) {
  if (!timing_) return 0;
  int n = 0;
  for (int i = 0; i + 1 < kMaxMarks && n < cap; ++i) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, marks_[i], marks_[i + 1]) != cudaSuccess) {
      (void)cudaGetLastError();
      ms = -1.f;
    }
    out[n++] = ms;
  }
  return n;
}

Context::~Context() {
  cudaSetDevice(device_);
  for (auto& e : marks_)
    if (e != nullptr) cudaEventDestroy(e);
  ws_.clear();
  status_.reset();
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

Status Context::workspace(int slot, size_t bytes, void** out) {
  DeviceBuffer& b = ws_[slot];
  if (b.size() < bytes) {
    // Grow geometrically so repeated calls with slightly larger batches do not reallocate.
    size_t want = bytes + bytes / 4;
    VDBGPU_CUDA(cudaStreamSynchronize(stream()));
    VDBGPU_RETURN_IF_ERROR(b.alloc(want));
  }
  *out = b.get();
  return Status::OK();
}

Status Context::EncodeOperandMap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t kpad,
                                 uint32_t box_rows, int ab_format, uint64_t row_pitch_bytes) const {
  auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(encode_fn_);
  cuuint64_t dims[2] = {kpad, rows};
  cuuint64_t strides[1] = {row_pitch_bytes != 0 ? row_pitch_bytes : kpad * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, ab_format == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return Status(Status::kInternal, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return Status::OK();
}

Status Context::CheckDeviceStatus(const char* what) {
  int code = 0;
  VDBGPU_CUDA(cudaMemcpyAsync(&code, status_.get(), sizeof(int), cudaMemcpyDeviceToHost, stream_));
  VDBGPU_CUDA(cudaStreamSynchronize(stream_));
  if (code == 0) return Status::OK();
  VDBGPU_CUDA(cudaMemsetAsync(status_.get(), 0, sizeof(int), stream_));
  VDBGPU_CUDA(cudaStreamSynchronize(stream_));
  const bool timeout = code >= 1 && code <= 5;
  return Status(timeout ? Status::kUnavailable : Status::kInternal,
                std::string(what) + ": device reported error code " + std::to_string(code));
}

Status Context::Sync(const char* what) {
  VDBGPU_CUDA(cudaStreamSynchronize(stream_));
  return CheckDeviceStatus(what);
}

}  // namespace vdbgpu
