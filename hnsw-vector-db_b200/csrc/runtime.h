// Host runtime of the B200 search path: status, device buffers, the per-device context and the
// GPU index interface that mirrors vdb::Index (src/index/index.h:36-55).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

namespace vdbgpu {

// vdb::Status (include/vdb/status.h:12-90), reduced to what crosses the C ABI.
class Status {
 public:
  enum Code : int {
    kOk = 0,
    kInvalidArgument = 1,
    kNotFound = 2,
    kAlreadyExists = 3,
    kIOError = 4,
    kCorruption = 5,
    kFailedPrecondition = 6,
    kResourceExhausted = 7,
    kUnavailable = 8,
    kNotSupported = 9,
    kInternal = 10,
  };
  Status() = default;
  Status(Code c, std::string m) : code_(c), msg_(std::move(m)) {}
  static Status OK() { return {}; }
  bool ok() const { return code_ == kOk; }
  Code code() const { return code_; }
  const std::string& message() const { return msg_; }

 private:
  Code code_ = kOk;
  std::string msg_;
};

#define VDBGPU_RETURN_IF_ERROR(expr)   \
  do {                                 \
    ::vdbgpu::Status _s = (expr);      \
    if (!_s.ok()) return _s;           \
  } while (0)

Status CudaStatus(cudaError_t e, const char* what);
#define VDBGPU_CUDA(expr) VDBGPU_RETURN_IF_ERROR(::vdbgpu::CudaStatus((expr), #expr))

// Owning device allocation.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  ~DeviceBuffer() { reset(); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr; o.n_ = 0; }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
      reset();
      p_ = o.p_;
      n_ = o.n_;
      o.p_ = nullptr;
      o.n_ = 0;
    }
    return *this;
  }
  Status alloc(size_t bytes);
  // Grows (never shrinks) to at least `bytes`; contents are not preserved.
  Status ensure(size_t bytes) { return bytes <= n_ ? Status::OK() : alloc(bytes); }
  void reset();
  template <class T>
  T* as() const { return static_cast<T*>(p_); }
  void* get() const { return p_; }
  size_t size() const { return n_; }

 private:
  void* p_ = nullptr;
  size_t n_ = 0;
};

// Summation order of the reference's runtime-selected kernel set on this host
// (src/distance/cpu_features.cc:27-72, honouring VDB_KERNELS).
int DetectKernelOrder();
const char* KernelOrderName(int order);

// Kernel launches of this library in this process (every launch site calls NoteLaunch), read by
// vdbgpu_launch_count: a caller can count the launches of a timed region.
void NoteLaunch();
uint64_t LaunchCount();

// Where a caller's buffer lives, seen from a context on `device`: host memory (staged through a
// copy), memory this device's kernels may use directly (its own allocations, managed memory), or
// another GPU's memory, which the kernels must not be given: without peer access enabled every
// access to it is an illegal address.
enum class MemWhere { kHost, kDevice, kOtherDevice };
MemWhere WherePointer(const void* p, int device);
// kInvalidArgument naming `what` when p is another GPU's memory, else OK.
Status RejectOtherDevice(const void* p, int device, const char* what);

class Context {
 public:
  static Status Open(int device, std::unique_ptr<Context>* out);
  ~Context();

  int device() const { return device_; }
  cudaStream_t stream() const { return user_stream_ != nullptr ? user_stream_ : stream_; }
  void set_user_stream(cudaStream_t s) { user_stream_ = s; }

  // Stage timing (vdbgpu_set_timing): Mark(i) records event i on the stream when enabled.
  Status EnableTiming(bool on);
  void Mark(int i) {
    if (timing_ && i < kMaxMarks) cudaEventRecord(marks_[i], stream());
  }
  int StageTimes(float* out, int cap);
  static constexpr int kMaxMarks = 4;
  bool timing() const { return timing_; }
  // Device counters of the last scan (chunks, triggered chunks, inserts, compactions), kept
  // only while timing is enabled.
  unsigned long long* counters() const { return counters_.as<unsigned long long>(); }
  int Counters(unsigned long long* out, int cap);
  // Epilogue warpgroups of the scan (VDB_SCAN_WARPGROUPS=1 or 2; 0 = per scan: 2 for seeded
  // scans, whose lists stay short, else 1).
  int scan_wgs() const { return scan_wgs_; }
  // B stages of the scan (VDB_SCAN_STAGES; 0 = as many as fit).
  int scan_stages() const { return scan_stages_; }
  int sm_count() const { return sm_count_; }
  int order() const { return order_; }
  int* status_word() const { return status_.as<int>(); }

  // Scratch buffer `slot`, grown to at least `bytes`.
  Status workspace(int slot, size_t bytes, void** out);

  // 2-D K-major fp16/bf16 tensor map with a {64, box_rows} box and 128-byte swizzle.
  // row_pitch_bytes 0 = kpad * 2 (contiguous rows); a larger pitch maps every n-th row.
  Status EncodeOperandMap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t kpad,
                          uint32_t box_rows, int ab_format, uint64_t row_pitch_bytes = 0) const;

  // Reads and clears the device status word after the stream is synchronised.
  Status CheckDeviceStatus(const char* what);
  Status Sync(const char* what);

  void set_error(const std::string& e) { last_error_ = e; }
  const std::string& last_error() const { return last_error_; }
  std::mutex& mu() { return mu_; }

 private:
  Context() = default;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  cudaStream_t user_stream_ = nullptr;
  bool timing_ = false;
  cudaEvent_t marks_[kMaxMarks] = {};
  DeviceBuffer counters_;
  int scan_wgs_ = 0;
  int scan_stages_ = 0;
  int sm_count_ = 0;
  int order_ = 1;
  DeviceBuffer status_;
  std::unordered_map<int, DeviceBuffer> ws_;
  void* encode_fn_ = nullptr;
  std::string last_error_;
  std::mutex mu_;
};

enum WorkspaceSlot : int {
  kWsQueries = 0,
  kWsOperandA,
  kWsQScale,
  kWsQTau,
  kWsCand,
  kWsCandCount,
  kWsAllow,
  kWsOutDist,
  kWsOutRow,
  kWsDistComps,
  kWsScratch0,
  kWsScratch1,
  kWsScratch2,
  kWsScratch3,
  kWsFallback,
  kWsFbQueries,
  kWsFbDist,
  kWsFbRow,
  kWsGroupIds,
  kWsGroupDist,
  kWsGroupOrder,
  kWsGroupQueries,
  kWsGroupOutDist,
  kWsGroupOutRow,
  kWsIvfA,
  kWsIvfQScale,
  kWsIvfTiles,
  kWsIvfSlotQuery,
  kWsIvfSlotOffset,
  kWsIvfPairSlot,
  kWsIvfUnits,
  kWsIvfAg,
  kWsIvfQScaleG,
};

enum IndexKind : int {
  kIndexFlat = 0,
  kIndexHnsw = 1,
  kIndexHnswSq8 = 2,
  kIndexPqFlat = 3,
  kIndexIvfPq = 4,
  kIndexSq8Flat = 16,
};

struct SearchParams {  // vdb::SearchParams (include/vdb/options.h:59-67)
  uint64_t ef = 64;
  uint64_t nprobe = 16;
  int32_t rerank = -1;
  int32_t strategy = 0;
  uint64_t prefilter_threshold = 10000;
  uint64_t post_filter_alpha = 10;
};

// Device-side arguments of one batched search: every pointer is device memory.
struct SearchBatch {
  const float* queries;      // nq x pd
  uint64_t nq;
  uint32_t k;
  SearchParams params;
  const uint32_t* allow;     // allowed-row bitset, 32 rows per word, padded; null = all rows
  float* out_dist;           // nq x k
  uint32_t* out_row;         // nq x k
  uint64_t* dist_comps;      // nq (device) or null
};

// The GPU counterpart of vdb::Index (src/index/index.h:36-55). Owns its device copies of the
// rows, codes, graph and tables for the segment's lifetime.
class GpuIndex {
 public:
  virtual ~GpuIndex() = default;
  virtual int type() const = 0;
  virtual Status Search(Context& ctx, const SearchBatch& b) = 0;
  virtual uint64_t rows() const = 0;
  virtual uint64_t device_bytes() const = 0;
  // The fp32 rows (rows() x pd) the index keeps on the device.
  virtual const float* device_rows() const = 0;
  virtual Status ExportSq8(Context&, float*, float*, uint8_t*) const {
    return Status(Status::kNotSupported, "index has no SQ8 codes");
  }
  // For indexes searched by the tensor-core scan (flat, SQ8-flat): the scan operands and the
  // candidate depths a search with these parameters uses.
  virtual Status ScanPlan(const SearchBatch&, const struct ScanOperands**, int*, int*) const {
    return Status(Status::kNotSupported, "index is not searched by the tensor-core scan");
  }

  int metric = 0;
  uint32_t dim = 0;
  uint32_t pd = 0;
};

// Factories (index_flat.cc, formats.cc).
Status CreateFlatIndex(Context& ctx, int metric, const float* rows_host, uint64_t n, uint32_t dim,
                       uint32_t pd, std::unique_ptr<GpuIndex>* out);
Status CreateSq8FlatIndex(Context& ctx, int metric, const float* rows_host, uint64_t n,
                          uint32_t dim, uint32_t pd, const float* vmin, const float* scale,
                          const uint8_t* codes, std::unique_ptr<GpuIndex>* out);
Status LoadIndexFile(Context& ctx, const void* bytes, size_t nbytes, int metric,
                     const float* rows_host, uint64_t n, uint32_t dim, uint32_t pd,
                     std::unique_ptr<GpuIndex>* out);
// HNSW, HNSW-SQ8, PQ-flat and IVF-PQ bodies (index_hnsw.cc, index_ivfpq.cc).
Status LoadGraphOrListIndex(Context& ctx, int type, std::string_view body, int metric,
                            const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                            std::unique_ptr<GpuIndex>* out);

// Filtered walks of many (segment, query) pairs over HNSW / HNSW-SQ8 segments of one collection in
// batched launches (index_graph.cc). items: host array; outputs at each item's slot (keys at
// slot * k). NotSupported when an index is not HNSW or the segments' graph parameters differ.
struct HnswItem;
struct MultiScratch {
  DeviceBuffer segs, items, visited, pool;
};
Status HnswSearchMulti(Context& ctx, const std::vector<const GpuIndex*>& indexes, const HnswItem* items,
                       size_t nitems, const float* queries, uint32_t k, const SearchParams& p, uint64_t* out_keys,
                       uint64_t* out_dc, int* out_short, MultiScratch* scratch);

// An HNSW graph over rows (host or device, n x pd) built on the GPU, as a complete index file in
// the reference's index.hnsw format (hnsw_build.cc).
// IvfPqIndex / PqFlatIndex build + save on the GPU (ivfpq_build_host.cc): type kIndexIvfPq or
// kIndexPqFlat; the reference's index file for the same rows and options.
Status BuildIvfPqFile(Context& ctx, int type, const float* rows, uint64_t n, uint32_t dim, uint32_t pd,
                      uint32_t nlist, uint32_t pq_m, uint32_t max_train_ppc, uint64_t seed, std::string* file);
Status BuildHnswFile(Context& ctx, int metric, const float* rows, uint64_t n, uint32_t dim, uint32_t pd, uint32_t M,
                     uint32_t kcand, uint64_t seed, std::string* file);
// HnswIndex::extend (src/index/hnsw/hnsw_index.cc:50-58) on the GPU: graph g (parsed from an
// index.hnsw over its first g.cap rows) with rows [g.cap, n) inserted, as a complete index file.
struct HnswGraphData;
Status ExtendHnswFile(Context& ctx, int metric, const HnswGraphData& g, uint32_t pd, const float* rows, uint64_t n,
                      uint32_t dim, std::string* file);

// Shared by flat and SQ8-flat search: a tensor-core pre-rank of every row followed by the exact
// finalize. Declared here so the HNSW/IVF indexes can reuse it for exact fallbacks.
struct ScanOperands {
  const void* b_operand = nullptr;  // rows x kpad fp16/bf16, rows padded to 256
  uint64_t rows = 0;
  uint32_t kpad = 0;
  int ab_format = 0;
  int row_scale_log2 = 0;           // operand rows were scaled by 2^row_scale_log2
  const float* rowterm = nullptr;   // per-row additive key term or null
  int prep_kind = 0;                // PrepKind
  int key_factor = 1;               // 2: key = rowterm - 2<a,b>; 1: key = -<a,b>
  const float* rows_f32 = nullptr;  // exact rows for the re-rank
  const uint8_t* codes = nullptr;   // SQ8 codes (exact SQ8 distances) or null
  const float* vmin = nullptr;
  const float* scale = nullptr;
  CUtensorMap b_map;
  // Seeding samples (index_flat.cc): level i maps every stride-th operand row through `map`, with
  // its row terms in `rowterm` when keys have one; level 1, when present, samples level 0's
  // stride 16 times more coarsely. nsamples 0 = no seeding.
  struct Sample {
    uint32_t stride = 0;
    uint64_t rows = 0;
    const float* rowterm = nullptr;
    CUtensorMap map;
  };
  Sample samples[2];
  int nsamples = 0;
  // Query grouping: a flat index over up to 1024 pivot rows chosen from a row sample. Large
  // batches are scanned in the order of each query's nearest pivot, so the 32 queries an epilogue
  // warp serves tend to share their candidate rows and fewer 32-row chunks hold a candidate for
  // any of them. Null = no grouping.
  const GpuIndex* group_index = nullptr;
};
// Attaches the seeding samples to `op` (after b_map / rowterm are set). rowterm_s[0..1] receive
// the sampled row terms. Small operands (and VDB_SCAN_SAMPLE=0) get none.
Status BuildScanSample(Context& ctx, ScanOperands* op, DeviceBuffer (&rowterm_s)[2]);
// Chooses the query-grouping pivots of `op` from about 4096 of its fp32 rows (index_flat.cc),
// builds their flat index into `pivots` (index metric) and attaches it. Small operands (and
// VDB_SCAN_GROUP=0) get none.
Status BuildQueryGrouping(Context& ctx, ScanOperands* op, int metric, uint32_t dim, uint32_t pd,
                          std::unique_ptr<GpuIndex>* pivots);
Status ScanSearch(Context& ctx, const ScanOperands& op, int metric, uint32_t pd,
                  const SearchBatch& b, int cpre, int depth);

}  // namespace vdbgpu
