// Exact flat search (FlatIndex, src/index/flat_index.h:24-44) and the exhaustive SQ8 scan with
// an fp32 re-rank on the GPU. Both run the same pipeline (ScanSearch):
//   prep_queries -> tensor-core scan with fused top-C (scan_mma.cu) -> exact finalize (select.cu)
//
// Seeded scans. On batches of at least 5e7 query-row pairs over operands of 64k rows or more, the
// pipeline first scans a strided sample of the rows (every s-th row, s = 16 by default;
// VDB_SCAN_SAMPLE sets s, 0 turns seeding off), where each 32-row chunk offers only its best key,
// keeping m candidates per query, and takes the m-th
// smallest sample key as the query's starting bound for the full scan, with m chosen so that about
// 2.25 C rows of the whole operand are expected below it. Every slice of the full scan then starts
// from that bound instead of from nothing, so few 32 x 32 chunks hold a candidate and the lists
// stay short. The sample scan can itself be seeded the same way from a 16 times coarser sample
// (VDB_SCAN_SAMPLE_LEVELS=2; a query whose coarse seed leaves fewer than m sample keys gets no
// seed). The bound is only an estimate: finalize checks that at least C keys lie below the
// query's final bound, which makes the C best exactly the C best of the whole operand (every row
// below the bound was kept), and the rare query with fewer is rescanned without a seed.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "hnsw_build.cuh"
#include "ivfpq.cuh"
#include "kernels.cuh"
#include "runtime.h"
#include "scan_mma.cuh"

namespace vdbgpu {
namespace {

uint64_t RoundUp(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

uint32_t Pow2Ceil(uint32_t x) {
  uint32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Row slices per 128-query tile: minimises waves * (tiles per slice + a fixed per-slice cost)
// for a grid of one CTA per SM.
void ChooseUnits(uint64_t qtiles, uint64_t ntiles, int sms, int* upq, int* tiles_per_unit) {
  double best = 1e300;
  *upq = 1;
  *tiles_per_unit = static_cast<int>(ntiles);
  const uint64_t max_u = std::min<uint64_t>(ntiles, 512);
  for (uint64_t u = 1; u <= max_u; ++u) {
    const uint64_t tpu = (ntiles + u - 1) / u;
    const uint64_t real_u = (ntiles + tpu - 1) / tpu;
    const uint64_t units = qtiles * real_u;
    const uint64_t waves = (units + sms - 1) / sms;
    const double t = static_cast<double>(waves) * (static_cast<double>(tpu) + 3.0);
    if (t < best) {
      best = t;
      *upq = static_cast<int>(real_u);
      *tiles_per_unit = static_cast<int>(tpu);
    }
  }
}

constexpr uint64_t kSampleMinRows = 65536;
constexpr double kSeedMinWork = 5e7;  // queries x rows below which scans are not seeded
constexpr uint64_t kSampleRatio = 16;     // stride of sample level 1 / stride of level 0
constexpr uint64_t kSample2MinRows = 1024;

uint32_t SampleStride() {
  const char* v = std::getenv("VDB_SCAN_SAMPLE");
  if (v == nullptr || *v == 0) return 16;
  const long s = std::strtol(v, nullptr, 10);
  return s < 0 ? 0u : static_cast<uint32_t>(std::min<long>(s, 1024));
}

// Sample candidates per query: the m-th smallest of every s-th row sits near rank m * s of the
// whole operand; m * s ~ 2.25 C, at least 24 keys so the estimate's spread stays within the
// margin. VDB_SCAN_SEED_KEEP sets m directly.
int SeedKeep(int cpre, uint32_t stride) {
  if (const char* v = std::getenv("VDB_SCAN_SEED_KEEP"); v != nullptr && *v != 0)
    return std::max(1, std::min(static_cast<int>(std::strtol(v, nullptr, 10)), kScanCap - 64));
  const int m = static_cast<int>(std::ceil(2.25 * cpre / stride));
  return std::max(24, m);
}

// Copies n x pd floats from host or device memory to a new device buffer.
Status UploadRows(Context& ctx, const float* rows, uint64_t n, uint32_t pd, DeviceBuffer* out) {
  VDBGPU_RETURN_IF_ERROR(out->alloc(std::max<uint64_t>(1, n * pd) * sizeof(float)));
  if (n > 0)
    VDBGPU_CUDA(cudaMemcpyAsync(out->get(), rows, n * pd * sizeof(float), cudaMemcpyDefault,
                                ctx.stream()));
  return Status::OK();
}

class FlatGpuIndex final : public GpuIndex {
 public:
  int type() const override { return kIndexFlat; }
  uint64_t rows() const override { return n_; }
  const float* device_rows() const override { return rows_.as<float>(); }
  uint64_t device_bytes() const override {
    return rows_.size() + operand_.size() + norms_.size() + sample_rowterm_[0].size() + sample_rowterm_[1].size();
  }

  Status Build(Context& ctx, const float* rows, uint64_t n) {
    n_ = n;
    const uint64_t npad = RoundUp(std::max<uint64_t>(n, 1), kScanBN);
    const uint32_t kpad = static_cast<uint32_t>(RoundUp(pd, kScanBK));
    VDBGPU_RETURN_IF_ERROR(UploadRows(ctx, rows, n, pd, &rows_));
    // fp16 when the rows fit its range (scaled by a power of two into [2^14, 2^15)), else bf16.
    DeviceBuffer amax;
    VDBGPU_RETURN_IF_ERROR(amax.alloc(sizeof(uint32_t)));
    VDBGPU_CUDA(cudaMemsetAsync(amax.get(), 0, sizeof(uint32_t), ctx.stream()));
    if (n > 0) VDBGPU_CUDA(LaunchAbsMax(rows_.as<float>(), n * pd, amax.as<uint32_t>(), ctx.stream()));
    uint32_t bits = 0;
    VDBGPU_CUDA(cudaMemcpyAsync(&bits, amax.get(), 4, cudaMemcpyDeviceToHost, ctx.stream()));
    VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    float m;
    std::memcpy(&m, &bits, 4);
    if (!std::isfinite(m)) return Status(Status::kInvalidArgument, "rows contain NaN or infinity");
    op_.ab_format = m > 60000.f ? 1 : 0;
    op_.row_scale_log2 = (op_.ab_format == 0 && m > 0.f) ? 14 - std::ilogb(m) : 0;
    VDBGPU_RETURN_IF_ERROR(operand_.alloc(npad * kpad * 2));
    VDBGPU_CUDA(cudaMemsetAsync(operand_.get(), 0, npad * kpad * 2, ctx.stream()));
    VDBGPU_RETURN_IF_ERROR(norms_.alloc(npad * sizeof(float)));
    VDBGPU_CUDA(cudaMemsetAsync(norms_.get(), 0, npad * sizeof(float), ctx.stream()));
    if (n > 0)
      VDBGPU_CUDA(LaunchPrepRows(rows_.as<float>(), n, pd, kpad, op_.ab_format, op_.row_scale_log2,
                                 operand_.get(), norms_.as<float>(), ctx.stream()));
    op_.b_operand = operand_.get();
    op_.rows = n;
    op_.kpad = kpad;
    op_.rowterm = metric == 0 ? norms_.as<float>() : nullptr;
    op_.prep_kind = kPrepFlat;
    op_.key_factor = metric == 0 ? 2 : 1;
    op_.rows_f32 = rows_.as<float>();
    VDBGPU_RETURN_IF_ERROR(
        ctx.EncodeOperandMap(&op_.b_map, operand_.get(), npad, kpad, kScanBN, op_.ab_format));
    VDBGPU_RETURN_IF_ERROR(BuildScanSample(ctx, &op_, sample_rowterm_));
    VDBGPU_RETURN_IF_ERROR(BuildQueryGrouping(ctx, &op_, metric, dim, pd, &pivots_));
    return ctx.Sync("flat index build");
  }

  Status ScanPlan(const SearchBatch& b, const ScanOperands** op, int* cpre, int* depth) const override {
    if (b.k > 256) return Status(Status::kNotSupported, "k > 256 is not supported by the GPU flat path");
    *op = &op_;
    *cpre = static_cast<int>(std::max<uint32_t>(32, Pow2Ceil(2 * b.k)));
    *depth = 0;
    return Status::OK();
  }

  // FlatIndex::search (src/index/flat_index.cc:73-77): exact top-k over allowed rows; counts
  // every row as a distance computation.
  Status Search(Context& ctx, const SearchBatch& b) override {
    if (b.k > 256) return Status(Status::kNotSupported, "k > 256 is not supported by the GPU flat path");
    const int cpre = static_cast<int>(std::max<uint32_t>(32, Pow2Ceil(2 * b.k)));
    VDBGPU_RETURN_IF_ERROR(ScanSearch(ctx, op_, metric, pd, b, cpre, 0));
    if (b.dist_comps != nullptr) {
      std::vector<uint64_t> dc(b.nq, n_);
      VDBGPU_CUDA(cudaMemcpyAsync(b.dist_comps, dc.data(), b.nq * 8, cudaMemcpyHostToDevice, ctx.stream()));
      VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    }
    return Status::OK();
  }

 private:
  uint64_t n_ = 0;
  DeviceBuffer rows_, operand_, norms_;
  DeviceBuffer sample_rowterm_[2];
  ScanOperands op_;
  std::unique_ptr<GpuIndex> pivots_;
};

class Sq8FlatGpuIndex final : public GpuIndex {
 public:
  int type() const override { return kIndexSq8Flat; }
  uint64_t rows() const override { return n_; }
  const float* device_rows() const override { return rows_.as<float>(); }
  uint64_t device_bytes() const override {
    return rows_.size() + codes_.size() + operand_.size() + rowterm_.size() + vmin_.size() +
           scale_.size() + sample_rowterm_[0].size() + sample_rowterm_[1].size();
  }

  // Sq8Quantizer::train + encode (src/index/quant/sq8.cc:9-37) on the GPU, or loads a trained
  // quantiser and its codes (vmin/scale/codes non-null, host or device memory).
  Status Build(Context& ctx, const float* rows, uint64_t n, const float* vmin, const float* scale,
               const uint8_t* codes) {
    n_ = n;
    const uint64_t npad = RoundUp(std::max<uint64_t>(n, 1), kScanBN);
    const uint32_t kpad = static_cast<uint32_t>(RoundUp(pd, kScanBK));
    VDBGPU_RETURN_IF_ERROR(UploadRows(ctx, rows, n, pd, &rows_));
    VDBGPU_RETURN_IF_ERROR(vmin_.alloc(pd * sizeof(float)));
    VDBGPU_RETURN_IF_ERROR(scale_.alloc(pd * sizeof(float)));
    VDBGPU_RETURN_IF_ERROR(codes_.alloc(std::max<uint64_t>(1, n * pd)));
    VDBGPU_RETURN_IF_ERROR(operand_.alloc(npad * kpad * 2));
    VDBGPU_CUDA(cudaMemsetAsync(operand_.get(), 0, npad * kpad * 2, ctx.stream()));
    VDBGPU_RETURN_IF_ERROR(rowterm_.alloc(npad * sizeof(float)));
    VDBGPU_CUDA(cudaMemsetAsync(rowterm_.get(), 0, npad * sizeof(float), ctx.stream()));
    if (vmin != nullptr) {
      VDBGPU_CUDA(cudaMemcpyAsync(vmin_.get(), vmin, pd * 4, cudaMemcpyDefault, ctx.stream()));
      VDBGPU_CUDA(cudaMemcpyAsync(scale_.get(), scale, pd * 4, cudaMemcpyDefault, ctx.stream()));
      if (n > 0) {
        VDBGPU_CUDA(cudaMemcpyAsync(codes_.get(), codes, n * pd, cudaMemcpyDefault, ctx.stream()));
        VDBGPU_CUDA(LaunchSq8Operand(codes_.as<uint8_t>(), n, pd, kpad, scale_.as<float>(),
                                     operand_.as<__half>(), rowterm_.as<float>(), ctx.stream()));
      }
    } else {
      // train: per-dimension min/max, then scale = (max - min) / 255 in IEEE fp32 on the host.
      std::vector<float> hmin(pd, 0.f), hscale(pd, 0.f);
      if (n > 0) {
        DeviceBuffer kmm;
        VDBGPU_RETURN_IF_ERROR(kmm.alloc(2 * dim * sizeof(uint32_t)));
        uint32_t* kmin = kmm.as<uint32_t>();
        uint32_t* kmax = kmin + dim;
        VDBGPU_CUDA(cudaMemsetAsync(kmin, 0xFF, dim * 4, ctx.stream()));
        VDBGPU_CUDA(cudaMemsetAsync(kmax, 0x00, dim * 4, ctx.stream()));
        VDBGPU_CUDA(LaunchSq8MinMax(rows_.as<float>(), n, dim, pd, kmin, kmax, ctx.stream()));
        std::vector<uint32_t> h(2 * dim);
        VDBGPU_CUDA(cudaMemcpyAsync(h.data(), kmin, 2 * dim * 4, cudaMemcpyDeviceToHost, ctx.stream()));
        VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
        for (uint32_t i = 0; i < dim; ++i) {
          const float lo = KeyToFloat(h[i]), hi = KeyToFloat(h[dim + i]);
          hmin[i] = lo;
          hscale[i] = (hi - lo) / 255.f;
        }
      }
      VDBGPU_CUDA(cudaMemcpyAsync(vmin_.get(), hmin.data(), pd * 4, cudaMemcpyHostToDevice, ctx.stream()));
      VDBGPU_CUDA(cudaMemcpyAsync(scale_.get(), hscale.data(), pd * 4, cudaMemcpyHostToDevice, ctx.stream()));
      if (n > 0)
        VDBGPU_CUDA(LaunchSq8Encode(rows_.as<float>(), n, dim, pd, kpad, vmin_.as<float>(),
                                    scale_.as<float>(), codes_.as<uint8_t>(), operand_.as<__half>(),
                                    rowterm_.as<float>(), ctx.stream()));
      VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    }
    op_.b_operand = operand_.get();
    op_.rows = n;
    op_.kpad = kpad;
    op_.ab_format = 0;
    op_.row_scale_log2 = 0;
    op_.rowterm = metric == 0 ? rowterm_.as<float>() : nullptr;
    op_.prep_kind = metric == 0 ? kPrepSq8L2 : kPrepSq8Ip;
    op_.key_factor = metric == 0 ? 2 : 1;
    op_.rows_f32 = rows_.as<float>();
    op_.codes = codes_.as<uint8_t>();
    op_.vmin = vmin_.as<float>();
    op_.scale = scale_.as<float>();
    VDBGPU_RETURN_IF_ERROR(ctx.EncodeOperandMap(&op_.b_map, operand_.get(), npad, kpad, kScanBN, 0));
    VDBGPU_RETURN_IF_ERROR(BuildScanSample(ctx, &op_, sample_rowterm_));
    VDBGPU_RETURN_IF_ERROR(BuildQueryGrouping(ctx, &op_, metric, dim, pd, &pivots_));
    return ctx.Sync("sq8 index build");
  }

  Status ScanPlan(const SearchBatch& b, const ScanOperands** op, int* cpre, int* depth) const override {
    const int32_t rr = b.params.rerank;
    const uint32_t d = rr < 0 ? std::max<uint32_t>(10 * b.k, 100) : static_cast<uint32_t>(rr);
    const uint32_t need = std::max(d, b.k);
    const uint32_t c = Pow2Ceil(need + need / 4);
    if (c > 256) return Status(Status::kNotSupported, "re-rank depth above 204 is not supported on the GPU");
    *op = &op_;
    *cpre = static_cast<int>(c);
    *depth = static_cast<int>(d);
    return Status::OK();
  }

  // Exhaustive SQ8 scan: SQ8 distances to every code pick the `depth` best, which are re-ranked
  // on fp32 rows (Rerank, src/index/index.cc:89-95). depth follows RerankDepth
  // (src/index/quant/ivf_pq.cc:16-19): rerank < 0 -> max(10k, 100), 0 -> SQ8 distances only.
  Status Search(Context& ctx, const SearchBatch& b) override {
    const int32_t rr = b.params.rerank;
    const uint32_t depth = rr < 0 ? std::max<uint32_t>(10 * b.k, 100) : static_cast<uint32_t>(rr);
    const uint32_t need = std::max(depth, b.k);
    const uint32_t cpre = Pow2Ceil(need + need / 4);
    if (cpre > 256)
      return Status(Status::kNotSupported, "re-rank depth above 204 is not supported on the GPU");
    VDBGPU_RETURN_IF_ERROR(ScanSearch(ctx, op_, metric, pd, b, static_cast<int>(cpre),
                                      static_cast<int>(depth)));
    if (b.dist_comps != nullptr) {
      std::vector<uint64_t> dc(b.nq, n_ + (depth > 0 ? std::min<uint64_t>(depth, n_) : 0));
      VDBGPU_CUDA(cudaMemcpyAsync(b.dist_comps, dc.data(), b.nq * 8, cudaMemcpyHostToDevice, ctx.stream()));
      VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    }
    return Status::OK();
  }

  Status ExportSq8(Context& ctx, float* vmin, float* scale, uint8_t* codes) const override {
    VDBGPU_CUDA(cudaMemcpyAsync(vmin, vmin_.get(), pd * 4, cudaMemcpyDefault, ctx.stream()));
    VDBGPU_CUDA(cudaMemcpyAsync(scale, scale_.get(), pd * 4, cudaMemcpyDefault, ctx.stream()));
    if (codes != nullptr && n_ > 0)
      VDBGPU_CUDA(cudaMemcpyAsync(codes, codes_.get(), n_ * pd, cudaMemcpyDefault, ctx.stream()));
    VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    return Status::OK();
  }

 private:
  static float KeyToFloat(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }

  uint64_t n_ = 0;
  DeviceBuffer rows_, codes_, operand_, rowterm_, vmin_, scale_;
  DeviceBuffer sample_rowterm_[2];
  ScanOperands op_;
  std::unique_ptr<GpuIndex> pivots_;
};

}  // namespace

Status BuildScanSample(Context& ctx, ScanOperands* op, DeviceBuffer (&rowterm_s)[2]) {
  op->nsamples = 0;
  const uint32_t s0 = SampleStride();
  if (s0 < 2 || op->rows < kSampleMinRows) return Status::OK();
  // VDB_SCAN_SAMPLE_LEVELS=2 adds the coarser level (measured on config 1: no faster than one).
  int max_levels = 1;
  if (const char* v = std::getenv("VDB_SCAN_SAMPLE_LEVELS"); v != nullptr && *v == '2') max_levels = 2;
  for (int lv = 0; lv < max_levels; ++lv) {
    const uint64_t s = lv == 0 ? s0 : static_cast<uint64_t>(s0) * kSampleRatio;
    const uint64_t ns = (op->rows + s - 1) / s;
    if (lv == 1 && ns < kSample2MinRows) break;
    ScanOperands::Sample& smp = op->samples[lv];
    smp.rowterm = nullptr;
    if (op->rowterm != nullptr) {
      const uint64_t nspad = RoundUp(ns, kScanBN);
      VDBGPU_RETURN_IF_ERROR(rowterm_s[lv].alloc(nspad * sizeof(float)));
      VDBGPU_CUDA(cudaMemsetAsync(rowterm_s[lv].get(), 0, nspad * sizeof(float), ctx.stream()));
      VDBGPU_CUDA(cudaMemcpy2DAsync(rowterm_s[lv].get(), sizeof(float), op->rowterm, s * sizeof(float),
                                    sizeof(float), ns, cudaMemcpyDeviceToDevice, ctx.stream()));
      smp.rowterm = rowterm_s[lv].as<float>();
    }
    VDBGPU_RETURN_IF_ERROR(ctx.EncodeOperandMap(&smp.map, op->b_operand, ns, op->kpad, kScanBN,
                                                op->ab_format, static_cast<uint64_t>(op->kpad) * 2 * s));
    smp.stride = static_cast<uint32_t>(s);
    smp.rows = ns;
    op->nsamples = lv + 1;
  }
  return Status::OK();
}

constexpr uint64_t kGroupPivots = 1024;      // query-grouping pivots
constexpr uint64_t kGroupSample = 4096;      // sample rows the pivots are chosen from (about)
constexpr uint64_t kGroupMinQueries = 2048;  // batches below this are scanned as given

bool GroupingEnabled() {
  const char* v = std::getenv("VDB_SCAN_GROUP");
  return v == nullptr || *v == 0 || std::strcmp(v, "0") != 0;
}

namespace {

// L2 for metric 0, else minus the dot product; four partial sums (pd is a multiple of 16).
float GroupKey(const float* a, const float* b, uint32_t pd, bool l2) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (uint32_t i = 0; i < pd; i += 4) {
    for (int j = 0; j < 4; ++j) {
      if (l2) {
        const float d = a[i + j] - b[i + j];
        s[j] += d * d;
      } else {
        s[j] += a[i + j] * b[i + j];
      }
    }
  }
  const float t = (s[0] + s[1]) + (s[2] + s[3]);
  return l2 ? t : -t;
}

// The grouping pivots, `want` rows of the n-row sample: farthest-point selection (each new pivot
// the sample row whose nearest chosen pivot is farthest, first maximum, starting at sample row 0),
// which on clustered rows takes one pivot in every cluster before a second in any, then ordered
// by a greedy nearest-neighbour chain from the first (nearest unvisited next, first minimum), so
// pivots that share a region sit next to each other in the scan order.
std::vector<float> ChooseGroupPivots(const std::vector<float>& s, uint64_t n, uint32_t pd, bool l2,
                                     uint64_t want) {
  std::vector<uint64_t> sel{0};
  std::vector<float> near(n);
  for (uint64_t i = 0; i < n; ++i) near[i] = GroupKey(&s[0], &s[i * pd], pd, l2);
  while (sel.size() < want) {
    uint64_t far = 0;
    for (uint64_t i = 1; i < n; ++i)
      if (near[i] > near[far]) far = i;
    sel.push_back(far);
    for (uint64_t i = 0; i < n; ++i) near[i] = std::min(near[i], GroupKey(&s[far * pd], &s[i * pd], pd, l2));
  }
  const uint64_t p = sel.size();
  std::vector<char> used(p, 0);
  std::vector<float> out(p * pd);
  uint64_t cur = 0;
  used[0] = 1;
  for (uint64_t o = 0; o < p; ++o) {
    std::memcpy(&out[o * pd], &s[sel[cur] * pd], pd * sizeof(float));
    uint64_t next = p;
    float best = 0.f;
    for (uint64_t j = 0; j < p; ++j) {
      if (used[j]) continue;
      const float k = GroupKey(&s[sel[cur] * pd], &s[sel[j] * pd], pd, l2);
      if (next == p || k < best) {
        best = k;
        next = j;
      }
    }
    if (next == p) break;
    used[next] = 1;
    cur = next;
  }
  return out;
}

}  // namespace

Status BuildQueryGrouping(Context& ctx, ScanOperands* op, int metric, uint32_t dim, uint32_t pd,
                          std::unique_ptr<GpuIndex>* pivots) {
  op->group_index = nullptr;
  pivots->reset();
  if (op->rows < kSampleMinRows || op->rows_f32 == nullptr || !GroupingEnabled()) return Status::OK();
  const uint64_t stride = std::max<uint64_t>(1, op->rows / kGroupSample);
  const uint64_t n = op->rows / stride;
  std::vector<float> sample(n * pd);
  VDBGPU_CUDA(cudaMemcpy2DAsync(sample.data(), pd * sizeof(float), op->rows_f32, stride * pd * sizeof(float),
                                pd * sizeof(float), n, cudaMemcpyDeviceToHost, ctx.stream()));
  VDBGPU_RETURN_IF_ERROR(ctx.Sync("grouping sample"));
  const uint64_t want = std::min<uint64_t>(kGroupPivots, n / 4);
  const std::vector<float> rows = ChooseGroupPivots(sample, n, pd, metric == 0, want);
  DeviceBuffer prow;
  VDBGPU_RETURN_IF_ERROR(prow.alloc(rows.size() * sizeof(float)));
  VDBGPU_CUDA(cudaMemcpyAsync(prow.get(), rows.data(), rows.size() * sizeof(float), cudaMemcpyHostToDevice,
                              ctx.stream()));
  VDBGPU_RETURN_IF_ERROR(CreateFlatIndex(ctx, metric, prow.as<float>(), want, dim, pd, pivots));
  op->group_index = pivots->get();
  return Status::OK();
}

namespace {

// One scan (plus its seed) and finalize over b; seeded scans rescan the queries finalize
// returns (fewer than cpre keys below their bound) without a seed. mark0 = false: the caller
// recorded stage mark 0 already.
Status ScanSearchImpl(Context& ctx, const ScanOperands& op, int metric, uint32_t pd,
                      const SearchBatch& b, int cpre, int depth, bool top, bool mark0 = true,
                      bool nearest = false) {
  if (b.nq == 0) return Status::OK();
  if (op.rows == 0) {
    // Nothing to scan: every slot is a miss.
    std::vector<float> d(b.nq * b.k, INFINITY);
    std::vector<uint32_t> r(b.nq * b.k, UINT32_MAX);
    VDBGPU_CUDA(cudaMemcpyAsync(b.out_dist, d.data(), d.size() * 4, cudaMemcpyHostToDevice, ctx.stream()));
    VDBGPU_CUDA(cudaMemcpyAsync(b.out_row, r.data(), r.size() * 4, cudaMemcpyHostToDevice, ctx.stream()));
    return ctx.Sync("empty scan");
  }
  if (cpre > kScanCap - 64) return Status(Status::kNotSupported, "candidate depth too large");
  if (op.kpad > kScanMaxKB * kScanBK)
    return Status(Status::kNotSupported, "padded dimension above 256 is not supported by the scan");
  const uint64_t nq = b.nq;
  const uint64_t nq_pad = RoundUp(nq, kScanBM);
  void *a_op, *qscale, *qtau, *cand, *cnt;
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsOperandA, nq_pad * op.kpad * 2, &a_op));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsQScale, nq * sizeof(float), &qscale));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsQTau, nq * sizeof(uint32_t), &qtau));
  VDBGPU_CUDA(cudaMemsetAsync(qtau, 0xFF, nq * sizeof(uint32_t), ctx.stream()));

  if (top && mark0) ctx.Mark(0);
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
  pa.qscale = static_cast<float*>(qscale);
  VDBGPU_CUDA(LaunchPrepQueries(pa, ctx.stream()));

  CUtensorMap amap;
  VDBGPU_RETURN_IF_ERROR(ctx.EncodeOperandMap(&amap, a_op, nq_pad, op.kpad, kScanBM, op.ab_format));
  const uint64_t qtiles = nq_pad / kScanBM;
  const uint64_t ntiles = (op.rows + kScanBN - 1) / kScanBN;
  int upq = 1, tpu = 1;
  ChooseUnits(qtiles, ntiles, ctx.sm_count(), &upq, &tpu);
  const uint64_t nunits = qtiles * static_cast<uint64_t>(upq);
  // Seed: a scan of the row sample keeping m per query, then the m-th key per query.
  // Small batches gain less than the sample pass and the count read-back cost.
  const bool seeded = top && b.allow == nullptr && op.nsamples > 0 &&
                      static_cast<double>(nq) * static_cast<double>(op.rows) >= kSeedMinWork &&
                      op.samples[0].rows >= static_cast<uint64_t>(SeedKeep(cpre, op.samples[0].stride));
  // One candidate list per (unit, epilogue warpgroup, query). Two warpgroups split each tile's
  // columns and halve the time an accumulator waits for its epilogue, but double the lists: a
  // win once seeding keeps the lists short.
  const uint64_t wgs = nearest ? 1 : static_cast<uint64_t>(ctx.scan_wgs() > 0 ? ctx.scan_wgs() : (seeded ? 2 : 1));
  // Sample levels, coarsest first: each starts from the bound the previous one seeded.
  const int levels = seeded ? (op.nsamples > 1 && op.samples[1].rows >= 4u * static_cast<uint64_t>(
                                                       SeedKeep(cpre, op.samples[0].stride)) ? 2 : 1)
                            : 0;
  int upq_s[2] = {1, 1}, tpu_s[2] = {1, 1}, m = 0;
  uint64_t nunits_s = 0;
  if (seeded) m = SeedKeep(cpre, op.samples[0].stride);
  for (int lv = 0; lv < levels; ++lv) {
    ChooseUnits(qtiles, (op.samples[lv].rows + kScanBN - 1) / kScanBN, ctx.sm_count(), &upq_s[lv], &tpu_s[lv]);
    nunits_s = std::max(nunits_s, qtiles * static_cast<uint64_t>(upq_s[lv]));
  }
  const uint64_t lists = std::max(nunits, nunits_s) * wgs * kScanBM;
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsCand, lists * kScanCap * sizeof(uint2), &cand));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsCandCount, lists * sizeof(int), &cnt));

  ScanArgs sa{};
  sa.nq = static_cast<int>(nq);
  sa.nrows = static_cast<int>(op.rows);
  sa.kblocks = static_cast<int>(op.kpad / kScanBK);
  sa.mode = op.rowterm != nullptr ? kKeyRowTerm : kKeyScaled;
  sa.ab_format = op.ab_format;
  sa.keep = cpre;
  sa.stages = ScanMaxStagesFor(sa.kblocks);
  if (ctx.scan_stages() > 0) sa.stages = std::min(sa.stages, ctx.scan_stages());
  sa.units_per_qtile = upq;
  sa.rows_per_unit = tpu * kScanBN;
  sa.nunits = static_cast<int>(nunits);
  sa.qscale = static_cast<const float*>(qscale);
  sa.rowterm = op.rowterm;
  sa.allow = b.allow;
  sa.wgs = static_cast<int>(wgs);
  sa.counters = (top && ctx.timing()) ? ctx.counters() : nullptr;
  if (sa.counters != nullptr)
    VDBGPU_CUDA(cudaMemsetAsync(sa.counters, 0, 8 * sizeof(unsigned long long), ctx.stream()));
  sa.cand = static_cast<uint2*>(cand);
  sa.cand_count = static_cast<int*>(cnt);
  sa.qtau = static_cast<uint32_t*>(qtau);
  sa.status = ctx.status_word();
  if (nearest) {
    // Only each query's nearest row is wanted: each 32-row chunk offers its best key with that
    // key's row, and lists compact to one entry.
    sa.keep = 1;
    sa.chunk_best = 2;
    sa.compact_at = 96;
  }
  for (int lv = levels - 1; lv >= 0; --lv) {
    const ScanOperands::Sample& smp = op.samples[lv];
    const uint64_t nu = qtiles * static_cast<uint64_t>(upq_s[lv]);
    ScanArgs ss = sa;
    ss.nrows = static_cast<int>(smp.rows);
    ss.keep = m;
    // The sample's lists compact early: cheap 128-slot compactions tighten its bounds sooner.
    ss.compact_at = m < 64 ? 96 : 0;
    ss.units_per_qtile = upq_s[lv];
    ss.rows_per_unit = tpu_s[lv] * kScanBN;
    ss.nunits = static_cast<int>(nu);
    ss.rowterm = smp.rowterm;
    ss.counters = nullptr;
    ss.chunk_best = 1;
    const int grid_s = static_cast<int>(std::min<uint64_t>(nu, static_cast<uint64_t>(ctx.sm_count())));
    VDBGPU_CUDA(LaunchScan(amap, smp.map, ss, grid_s, ctx.stream()));
    SeedArgs sd{};
    sd.nq = static_cast<int>(nq);
    sd.m = m;
    sd.units_per_qtile = upq_s[lv];
    sd.wgs = static_cast<int>(wgs);
    sd.cand = static_cast<const uint2*>(cand);
    sd.cand_count = static_cast<const int*>(cnt);
    sd.qtau_out = static_cast<uint32_t*>(qtau);
    VDBGPU_CUDA(LaunchScanSeed(sd, ctx.stream()));
  }
  // Stage marks: [0, 1) query preparation and the seeding sample scan, [1, 2) the scan, [2, 3)
  // finalize.
  if (top) ctx.Mark(1);
  const int grid = static_cast<int>(std::min<uint64_t>(nunits, static_cast<uint64_t>(ctx.sm_count())));
  VDBGPU_CUDA(LaunchScan(amap, op.b_map, sa, grid, ctx.stream()));
  if (top) ctx.Mark(2);

  FinalizeArgs fa{};
  fa.nq = static_cast<int>(nq);
  fa.pd = static_cast<int>(pd);
  fa.k = static_cast<int>(b.k);
  fa.cpre = cpre;
  fa.depth = depth;
  fa.metric = metric;
  fa.order = ctx.order();
  fa.units_per_qtile = upq;
  fa.wgs = static_cast<int>(wgs);
  fa.cand = static_cast<const uint2*>(cand);
  fa.cand_count = static_cast<const int*>(cnt);
  fa.qtau = static_cast<const uint32_t*>(qtau);
  fa.queries = b.queries;
  fa.rows = op.rows_f32;
  fa.codes = op.codes;
  fa.vmin = op.vmin;
  fa.scale = op.scale;
  fa.out_dist = b.out_dist;
  fa.out_row = b.out_row;
  uint32_t* fb = nullptr;  // [0] count, [1..] queries to rescan
  if (seeded) {
    void* p;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsFallback, (nq + 1) * sizeof(uint32_t), &p));
    fb = static_cast<uint32_t*>(p);
    VDBGPU_CUDA(cudaMemsetAsync(fb, 0, sizeof(uint32_t), ctx.stream()));
    fa.fb_count = reinterpret_cast<int*>(fb);
    fa.fb_list = fb + 1;
  }
  VDBGPU_CUDA(LaunchFinalize(fa, ctx.stream()));
  if (top) ctx.Mark(3);
  if (!seeded) return Status::OK();

  uint32_t nfb = 0;
  VDBGPU_CUDA(cudaMemcpyAsync(&nfb, fb, sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx.stream()));
  VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
  if (sa.counters != nullptr) {
    const unsigned long long extra[3] = {nfb, 1ull, static_cast<unsigned long long>(m)};
    VDBGPU_CUDA(cudaMemcpyAsync(sa.counters + 4, extra, sizeof(extra), cudaMemcpyHostToDevice, ctx.stream()));
    VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
  }
  if (nfb == 0) return Status::OK();
  if (nfb > nq) return Status(Status::kInternal, "seeded scan: fallback count out of range");
  void *fq, *fd, *fr;
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsFbQueries, static_cast<uint64_t>(nfb) * pd * sizeof(float), &fq));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsFbDist, static_cast<uint64_t>(nfb) * b.k * sizeof(float), &fd));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsFbRow, static_cast<uint64_t>(nfb) * b.k * sizeof(uint32_t), &fr));
  VDBGPU_CUDA(LaunchGatherRows(b.queries, fb + 1, nfb, static_cast<int>(pd), static_cast<float*>(fq),
                               ctx.stream()));
  SearchBatch sub = b;
  sub.queries = static_cast<const float*>(fq);
  sub.nq = nfb;
  sub.out_dist = static_cast<float*>(fd);
  sub.out_row = static_cast<uint32_t*>(fr);
  sub.dist_comps = nullptr;
  VDBGPU_RETURN_IF_ERROR(ScanSearchImpl(ctx, op, metric, pd, sub, cpre, depth, false));
  VDBGPU_CUDA(LaunchScatterResults(static_cast<const float*>(fd), static_cast<const uint32_t*>(fr), fb + 1,
                                   nfb, static_cast<int>(b.k), b.out_dist, b.out_row, ctx.stream()));
  return Status::OK();
}

}  // namespace

Status ScanSearch(Context& ctx, const ScanOperands& op, int metric, uint32_t pd,
                  const SearchBatch& b, int cpre, int depth) {
  if (op.group_index == nullptr || b.nq < kGroupMinQueries || b.allow != nullptr || op.rows == 0)
    return ScanSearchImpl(ctx, op, metric, pd, b, cpre, depth, true);
  // Query grouping (stage 0 includes it): each query's nearest pivot (a tensor-core scan of the
  // pivots in which each 32-row chunk offers its best row, then that row's exact distance), the queries ordered by pivot (a counting sort), the scan
  // over the reordered batch, and its results written back to the caller's query order. Every
  // query's result is its own, whatever order the batch is scanned in.
  ctx.Mark(0);
  const uint64_t nq = b.nq;
  const uint32_t cells = static_cast<uint32_t>(op.group_index->rows());
  void *pid, *pdist, *ord, *qp, *od, *orow;
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsGroupIds, nq * 4, &pid));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsGroupDist, nq * 4, &pdist));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsGroupOrder, (nq + cells + 1) * 4, &ord));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsGroupQueries, nq * pd * sizeof(float), &qp));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsGroupOutDist, nq * b.k * sizeof(float), &od));
  VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsGroupOutRow, nq * b.k * sizeof(uint32_t), &orow));
  SearchBatch pb{};
  pb.queries = b.queries;
  pb.nq = nq;
  pb.k = 1;
  pb.out_dist = static_cast<float*>(pdist);
  pb.out_row = static_cast<uint32_t*>(pid);
  const ScanOperands* pop = nullptr;
  int pcpre = 0, pdepth = 0;
  VDBGPU_RETURN_IF_ERROR(op.group_index->ScanPlan(pb, &pop, &pcpre, &pdepth));
  VDBGPU_RETURN_IF_ERROR(ScanSearchImpl(ctx, *pop, metric, pd, pb, 1, 0, false, false, true));
  uint32_t* order = static_cast<uint32_t*>(ord);
  VDBGPU_CUDA(LaunchProbeOrder(static_cast<const uint32_t*>(pid), static_cast<int>(nq), 1, cells, order + nq, order,
                               ctx.stream()));
  VDBGPU_CUDA(LaunchGatherRows(b.queries, order, nq, static_cast<int>(pd), static_cast<float*>(qp), ctx.stream()));
  SearchBatch sub = b;
  sub.queries = static_cast<const float*>(qp);
  sub.out_dist = static_cast<float*>(od);
  sub.out_row = static_cast<uint32_t*>(orow);
  sub.dist_comps = nullptr;
  VDBGPU_RETURN_IF_ERROR(ScanSearchImpl(ctx, op, metric, pd, sub, cpre, depth, true, false));
  VDBGPU_CUDA(LaunchScatterResults(static_cast<const float*>(od), static_cast<const uint32_t*>(orow), order,
                                   static_cast<uint32_t>(nq), static_cast<int>(b.k), b.out_dist, b.out_row,
                                   ctx.stream()));
  return Status::OK();
}

Status CreateFlatIndex(Context& ctx, int metric, const float* rows, uint64_t n, uint32_t dim,
                       uint32_t pd, std::unique_ptr<GpuIndex>* out) {
  auto idx = std::make_unique<FlatGpuIndex>();
  idx->metric = metric;
  idx->dim = dim;
  idx->pd = pd;
  VDBGPU_RETURN_IF_ERROR(idx->Build(ctx, rows, n));
  *out = std::move(idx);
  return Status::OK();
}

Status CreateSq8FlatIndex(Context& ctx, int metric, const float* rows, uint64_t n, uint32_t dim,
                          uint32_t pd, const float* vmin, const float* scale, const uint8_t* codes,
                          std::unique_ptr<GpuIndex>* out) {
  if (dim > 1024) return Status(Status::kNotSupported, "SQ8 training supports dim <= 1024");
  auto idx = std::make_unique<Sq8FlatGpuIndex>();
  idx->metric = metric;
  idx->dim = dim;
  idx->pd = pd;
  VDBGPU_RETURN_IF_ERROR(idx->Build(ctx, rows, n, vmin, scale, codes));
  *out = std::move(idx);
  return Status::OK();
}

}  // namespace vdbgpu
