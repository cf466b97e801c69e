// IVF-PQ (IvfPqIndex, src/index/quant/ivf_pq.h:42-81) and PQ-flat (PqFlatIndex, :12-36) on the
// GPU, loaded from the reference's own index files (IvfPqIndex::save, ivf_pq.cc:236-249;
// PqFlatIndex::save, ivf_pq.cc:78-84).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "formats.h"
#include "ivfpq.cuh"
#include "kernels.cuh"
#include "runtime.h"
#include "scan_mma.cuh"

namespace vdbgpu {
namespace {

template <class T>
Status Upload(Context& ctx, const T* p, size_t count, DeviceBuffer* out) {
  VDBGPU_RETURN_IF_ERROR(out->alloc(std::max<size_t>(1, count) * sizeof(T)));
  if (count > 0)
    VDBGPU_CUDA(cudaMemcpyAsync(out->get(), p, count * sizeof(T), cudaMemcpyDefault, ctx.stream()));
  return Status::OK();
}

uint64_t Up(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

// VDB_IVF_TENSOR=0 keeps every IVF-PQ search on the per-query kernel.
bool TensorEnabled() {
  const char* v = std::getenv("VDB_IVF_TENSOR");
  return v == nullptr || *v == 0 || std::strcmp(v, "0") != 0;
}

// The first list-mode pass covers at most the first SeedRows(cpre) rows of each query's nearest
// list (VDB_IVF_SEED_ROWS; 0 = the whole list). Its cpre-th key there bounds the query: at least
// cpre rows of a probed list lie below it, so the bound is exact, only looser than the whole
// list's.
uint32_t SeedRows(int cpre) {
  const char* v = std::getenv("VDB_IVF_SEED_ROWS");
  if (v != nullptr && *v != 0) return static_cast<uint32_t>(std::strtoul(v, nullptr, 10));
  return static_cast<uint32_t>(4 * cpre);
}

// Batches of at least this many queries (no filter, L2) take the tensor-core pre-rank.
constexpr uint64_t kIvfTensorMinQueries = 512;

// RerankDepth (src/index/quant/ivf_pq.cc:16-19).
uint32_t RerankDepth(int32_t rerank, uint32_t k) {
  return rerank < 0 ? std::max<uint32_t>(10 * k, 100) : static_cast<uint32_t>(rerank);
}

class IvfPqGpuIndex final : public GpuIndex {
 public:
  explicit IvfPqGpuIndex(bool flat) : pqflat_(flat) {}
  int type() const override { return pqflat_ ? kIndexPqFlat : kIndexIvfPq; }
  uint64_t rows() const override { return n_; }
  const float* device_rows() const override { return rows_.as<float>(); }
  uint64_t device_bytes() const override {
    return rows_.size() + coarse_.size() + cents_.size() + term2_.size() + off_.size() + ids_.size() +
           codes_.size() + poff_.size() + resid_.size() + resid_term_.size() +
           (coarse_index_ ? coarse_index_->device_bytes() : 0);
  }

  Status Load(Context& ctx, std::string_view body, const float* rows, uint64_t n) {
    n_ = n;
    PqData pq;
    std::vector<uint64_t> off;
    std::vector<uint32_t> ids;
    std::string_view codes_view;
    std::vector<uint8_t> codes;
    std::vector<float> coarse;
    if (pqflat_) {
      Reader r(body);
      uint64_t fn = 0;
      if (!r.u64(&fn) || fn != n) return Status(Status::kCorruption, "pq index does not match the segment");
      // PqFlatIndex::load (ivf_pq.cc:86-90) reports any codebook fault as a mismatch.
      if (!ParsePq(r, &pq).ok() || pq.dim != dim)
        return Status(Status::kCorruption, "pq index does not match the segment");
      if (!r.bytes(n * pq.m, &codes_view)) return Status(Status::kCorruption, "truncated pq codes");
      nlist_ = 0;
    } else {
      IvfPqData d;
      VDBGPU_RETURN_IF_ERROR(ParseIvfPq(body, n, pd, dim, &d));
      pq = std::move(d.pq);
      off = std::move(d.list_off);
      ids = std::move(d.ids);
      codes = std::move(d.codes);
      coarse = std::move(d.coarse);
      nlist_ = d.nlist;
    }
    m_ = pq.m;
    dsub_ = pq.dsub;
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, pq.centroids.data(), pq.centroids.size(), &cents_));
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, rows, n * pd, &rows_));
    if (pqflat_) {
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, reinterpret_cast<const uint8_t*>(codes_view.data()), n * m_, &codes_));
    } else {
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, codes.data(), codes.size(), &codes_));
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, off.data(), off.size(), &off_));
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, ids.data(), ids.size(), &ids_));
      VDBGPU_RETURN_IF_ERROR(Upload(ctx, coarse.data(), coarse.size(), &coarse_));
      // Precomputed tables are derived data, rebuilt on load as the reference does, under the
      // same conditions (L2, at most 1 GiB; ivf_pq.cc:155).
      const uint64_t tbytes = static_cast<uint64_t>(nlist_) * m_ * 256 * 4;
      if (metric == 0 && nlist_ > 0 && tbytes <= (uint64_t{1} << 30)) {
        VDBGPU_RETURN_IF_ERROR(term2_.alloc(tbytes));
        VDBGPU_CUDA(LaunchTerm2(coarse_.as<float>(), nlist_, pd, cents_.as<float>(), m_, dsub_,
                                term2_.as<float>(), ctx.stream()));
      }
      // The probe step is an exact flat search over the coarse centroids with the index metric
      // (the reference computes dist_(q, coarse_l) for every list, ivf_pq.cc:176-181).
      if (nlist_ > 0)
        VDBGPU_RETURN_IF_ERROR(CreateFlatIndex(ctx, metric, coarse.data(), nlist_, dim, pd, &coarse_index_));
      VDBGPU_RETURN_IF_ERROR(BuildListOperand(ctx, off));
    }
    return ctx.Sync("ivf-pq index load");
  }

  // The list-mode operand (ivf_mma.cu): decoded residuals in fp16, lists on 32-row boundaries.
  // L2 only, lists below 2^24 rows, fp16-range codebooks; otherwise none and every search takes
  // the per-query kernel.
  Status BuildListOperand(Context& ctx, const std::vector<uint64_t>& off) {
    kpad_ = static_cast<uint32_t>(Up(pd, kScanBK));
    if (metric != 0 || nlist_ == 0 || kpad_ > kScanMaxKB * kScanBK || m_ * dsub_ != dim) return Status::OK();
    std::vector<uint64_t> poff(nlist_ + 1, 0);
    for (uint32_t l = 0; l < nlist_; ++l) {
      const uint64_t size = off[l + 1] - off[l];
      if (size >= (uint64_t{1} << 24)) return Status::OK();
      poff[l + 1] = poff[l] + Up(size, 32);
    }
    if (poff[nlist_] >= (uint64_t{1} << 31) - 512) return Status::OK();
    DeviceBuffer amax;
    VDBGPU_RETURN_IF_ERROR(amax.alloc(sizeof(uint32_t)));
    VDBGPU_CUDA(cudaMemsetAsync(amax.get(), 0, sizeof(uint32_t), ctx.stream()));
    VDBGPU_CUDA(LaunchAbsMax(cents_.as<float>(), static_cast<uint64_t>(m_) * 256 * dsub_, amax.as<uint32_t>(),
                             ctx.stream()));
    uint32_t bits = 0;
    VDBGPU_CUDA(cudaMemcpyAsync(&bits, amax.get(), 4, cudaMemcpyDeviceToHost, ctx.stream()));
    VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    float mx;
    std::memcpy(&mx, &bits, 4);
    if (!std::isfinite(mx) || mx > 60000.f) return Status::OK();
    resid_scale_log2_ = mx > 0.f ? 14 - std::ilogb(mx) : 0;
    const uint64_t npad = Up(std::max<uint64_t>(poff[nlist_], 1), kScanBN);
    VDBGPU_RETURN_IF_ERROR(Upload(ctx, poff.data(), poff.size(), &poff_));
    VDBGPU_RETURN_IF_ERROR(resid_.alloc(npad * kpad_ * 2));
    VDBGPU_CUDA(cudaMemsetAsync(resid_.get(), 0, npad * kpad_ * 2, ctx.stream()));
    VDBGPU_RETURN_IF_ERROR(resid_term_.alloc((npad + kScanBN) * sizeof(float)));
    VDBGPU_CUDA(cudaMemsetAsync(resid_term_.get(), 0, (npad + kScanBN) * sizeof(float), ctx.stream()));
    IvfDecodeArgs da{};
    da.codes = codes_.as<uint8_t>();
    da.list_off = off_.as<uint64_t>();
    da.poff = poff_.as<uint64_t>();
    da.nlist = nlist_;
    da.m = static_cast<int>(m_);
    da.dsub = static_cast<int>(dsub_);
    da.kpad = static_cast<int>(kpad_);
    da.cstride = static_cast<int>(pd);
    da.centroids = cents_.as<float>();
    da.coarse = coarse_.as<float>();
    da.scale_log2 = resid_scale_log2_;
    da.operand = static_cast<__half*>(resid_.get());
    da.rowterm = resid_term_.as<float>();
    VDBGPU_CUDA(LaunchIvfDecode(da, ctx.stream()));
    VDBGPU_RETURN_IF_ERROR(ctx.EncodeOperandMap(&resid_map_, resid_.get(), npad, kpad_, kScanBN, 0));
    list_mode_ = true;
    return Status::OK();
  }

  // One list-mode scan over the pairs (query, probe < np): tiles, gathered query operand, scan.
  // Returns the tile count.
  Status ListScan(Context& ctx, const SearchBatch& b, const void* a_op, const float* qscale, const uint32_t* pid,
                  const float* pdist, int nprobe, int np, uint32_t row_cap, int cpre, uint32_t* qtau,
                  uint32_t* pair_slot, uint32_t* ntiles) {
    const uint64_t nq = b.nq;
    const uint64_t max_tiles = nq * static_cast<uint64_t>(np) / 128 + nlist_;
    void *tiles, *sq, *so, *units, *ag, *qg, *cand, *cnt;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfTiles, 3 * (static_cast<uint64_t>(nlist_) + 1) * 4, &tiles));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfSlotQuery, max_tiles * 128 * 4, &sq));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfSlotOffset, max_tiles * 128 * 4, &so));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfUnits, max_tiles * sizeof(int2), &units));
    uint32_t* counts = static_cast<uint32_t*>(tiles);
    uint32_t* cursor = counts + nlist_ + 1;
    uint32_t* tstart = cursor + nlist_ + 1;
    VDBGPU_CUDA(cudaMemsetAsync(sq, 0xFF, max_tiles * 128 * 4, ctx.stream()));
    IvfTileArgs ta{};
    ta.nq = static_cast<int>(nq);
    ta.nprobe = nprobe;
    ta.np = np;
    ta.nlist = nlist_;
    ta.probe_ids = pid;
    ta.probe_dist = pdist;
    ta.list_off = off_.as<uint64_t>();
    ta.poff = poff_.as<uint64_t>();
    ta.cursor = cursor;
    ta.tile_start = tstart;
    ta.slot_query = static_cast<uint32_t*>(sq);
    ta.slot_offset = static_cast<float*>(so);
    ta.pair_slot = pair_slot;
    ta.unit_rows = static_cast<int2*>(units);
    ta.row_cap = row_cap;
    VDBGPU_CUDA(LaunchIvfTiles(ta, counts, ctx.stream()));
    uint32_t nt = 0;
    VDBGPU_CUDA(cudaMemcpyAsync(&nt, tstart + nlist_, 4, cudaMemcpyDeviceToHost, ctx.stream()));
    VDBGPU_CUDA(cudaStreamSynchronize(ctx.stream()));
    if (nt > max_tiles) return Status(Status::kInternal, "ivf tiles: count out of range");
    *ntiles = nt;
    if (nt == 0) return Status::OK();
    const uint64_t nslots = static_cast<uint64_t>(nt) * 128;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfAg, nslots * kpad_ * 2, &ag));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfQScaleG, nslots * 4, &qg));
    VDBGPU_CUDA(LaunchIvfGather(a_op, qscale, static_cast<const uint32_t*>(sq), static_cast<uint32_t>(nslots),
                                static_cast<int>(kpad_), ag, static_cast<float*>(qg), ctx.stream()));
    CUtensorMap amap;
    VDBGPU_RETURN_IF_ERROR(ctx.EncodeOperandMap(&amap, ag, nslots, kpad_, kScanBM, 0));
    const int wgs = 2;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsCand, static_cast<uint64_t>(nt) * wgs * kScanBM * kScanCap * sizeof(uint2), &cand));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsCandCount, static_cast<uint64_t>(nt) * wgs * kScanBM * sizeof(int), &cnt));
    ScanArgs sa{};
    sa.nq = static_cast<int>(nslots);
    sa.nrows = 0;
    sa.kblocks = static_cast<int>(kpad_ / kScanBK);
    sa.mode = kKeyList;
    sa.ab_format = 0;
    sa.keep = cpre;
    sa.stages = ScanMaxStagesFor(sa.kblocks);
    if (ctx.scan_stages() > 0) sa.stages = std::min(sa.stages, ctx.scan_stages());
    sa.units_per_qtile = 1;
    sa.rows_per_unit = kScanBN;
    sa.nunits = static_cast<int>(nt);
    sa.qscale = static_cast<const float*>(qg);
    sa.rowterm = resid_term_.as<float>();
    sa.wgs = wgs;
    sa.cand = static_cast<uint2*>(cand);
    sa.cand_count = static_cast<int*>(cnt);
    sa.qtau = qtau;
    sa.status = ctx.status_word();
    sa.unit_rows = static_cast<const int2*>(units);
    sa.slot_query = static_cast<const uint32_t*>(sq);
    sa.slot_offset = static_cast<const float*>(so);
    const int grid = static_cast<int>(std::min<uint64_t>(nt, static_cast<uint64_t>(ctx.sm_count())));
    VDBGPU_CUDA(LaunchScan(amap, resid_map_, sa, grid, ctx.stream()));
    return Status::OK();
  }

  // IVF-PQ search with the tensor-core pre-rank: the probe, a first list-mode scan of every
  // query's nearest list (which publishes each query's cpre-th key there as its bound), the scan
  // of all probed lists under those bounds, and the exact stage (reference ADC of the cpre best by
  // pre-rank key, TopK, re-rank).
  Status ListSearch(Context& ctx, const SearchBatch& b, uint32_t k, uint32_t depth, int nprobe, const uint32_t* pid,
                    const float* pdist) {
    const uint64_t nq = b.nq;
    const uint32_t R = std::max(depth, k);
    // cpre: R + R / 4 rounded up to a power of two, as the SQ8 scan's pre-rank (128 for R = 100).
    uint32_t c = 32;
    while (c < R + R / 4 && c < 256) c <<= 1;
    const int cpre = static_cast<int>(c);
    const uint64_t nq_pad = Up(nq, kScanBM);
    void *a_op, *qscale, *qtau, *ps;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfA, nq_pad * kpad_ * 2, &a_op));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfQScale, nq * 4, &qscale));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsQTau, nq * 4, &qtau));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsIvfPairSlot, nq * nprobe * 4, &ps));
    PrepArgs pa{};
    pa.nq = static_cast<int>(nq);
    pa.nq_pad = static_cast<int>(nq_pad);
    pa.pd = static_cast<int>(pd);
    pa.kpad = static_cast<int>(kpad_);
    pa.kind = kPrepFlat;
    pa.ab_format = 0;
    pa.key_factor = 2;
    pa.row_scale_log2 = resid_scale_log2_;
    pa.queries = b.queries;
    pa.operand = a_op;
    pa.qscale = static_cast<float*>(qscale);
    VDBGPU_CUDA(LaunchPrepQueries(pa, ctx.stream()));
    VDBGPU_CUDA(cudaMemsetAsync(qtau, 0xFF, nq * 4, ctx.stream()));
    uint32_t nt = 0;
    VDBGPU_RETURN_IF_ERROR(ListScan(ctx, b, a_op, static_cast<const float*>(qscale), pid, pdist, nprobe, 1,
                                    SeedRows(cpre), cpre, static_cast<uint32_t*>(qtau), nullptr, &nt));
    ctx.Mark(1);
    VDBGPU_RETURN_IF_ERROR(ListScan(ctx, b, a_op, static_cast<const float*>(qscale), pid, pdist, nprobe, nprobe, 0,
                                    cpre, static_cast<uint32_t*>(qtau), static_cast<uint32_t*>(ps), &nt));
    ctx.Mark(2);
    void *cand, *cnt;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsCand, 0, &cand));
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsCandCount, 0, &cnt));
    IvfFinalizeArgs fa{};
    fa.nq = static_cast<int>(nq);
    fa.nprobe = nprobe;
    fa.pd = static_cast<int>(pd);
    fa.dim = static_cast<int>(dim);
    fa.m = static_cast<int>(m_);
    fa.dsub = static_cast<int>(dsub_);
    fa.k = static_cast<int>(k);
    fa.depth = static_cast<int>(depth);
    fa.cpre = cpre;
    fa.order = ctx.order();
    fa.mode = term2_.get() != nullptr ? kIvfPrecomputed : kIvfResidual;
    fa.wgs = 2;
    fa.nlist = nlist_;
    fa.pair_slot = static_cast<const uint32_t*>(ps);
    fa.cand = static_cast<const uint2*>(cand);
    fa.cand_count = static_cast<const int*>(cnt);
    fa.qtau = static_cast<const uint32_t*>(qtau);
    fa.probe_ids = pid;
    fa.probe_dist = pdist;
    fa.list_off = off_.as<uint64_t>();
    fa.poff = poff_.as<uint64_t>();
    fa.ids = ids_.as<uint32_t>();
    fa.codes = codes_.as<uint8_t>();
    fa.centroids = cents_.as<float>();
    fa.term2 = term2_.as<float>();
    fa.coarse = coarse_.as<float>();
    fa.queries = b.queries;
    fa.rows = rows_.as<float>();
    fa.out_dist = b.out_dist;
    fa.out_row = b.out_row;
    fa.out_dc = b.dist_comps;
    fa.counters = ctx.timing() ? ctx.counters() : nullptr;
    if (fa.counters != nullptr)
      VDBGPU_CUDA(cudaMemsetAsync(fa.counters, 0, 8 * sizeof(unsigned long long), ctx.stream()));
    VDBGPU_CUDA(LaunchIvfFinalize(fa, ctx.stream()));
    ctx.Mark(3);
    return Status::OK();
  }

  // The fields of the per-query kernel's arguments that do not depend on the probe.
  IvfPqArgs BaseArgs(const SearchBatch& b, uint32_t k, uint32_t depth) const {
    IvfPqArgs a{};
    a.nq = static_cast<int>(b.nq);
    a.pd = static_cast<int>(pd);
    a.dim = static_cast<int>(dim);
    a.m = static_cast<int>(m_);
    a.dsub = static_cast<int>(dsub_);
    a.k = static_cast<int>(k);
    a.depth = static_cast<int>(depth);
    a.metric = metric;
    a.nlist = nlist_;
    a.n = n_;
    a.queries = b.queries;
    a.rows = rows_.as<float>();
    a.coarse = coarse_.as<float>();
    a.centroids = cents_.as<float>();
    a.term2 = term2_.as<float>();
    a.list_off = off_.as<uint64_t>();
    a.ids = ids_.as<uint32_t>();
    a.codes = codes_.as<uint8_t>();
    a.allow = b.allow;
    a.out_dist = b.out_dist;
    a.out_row = b.out_row;
    a.out_dc = b.dist_comps;
    return a;
  }

  Status Search(Context& ctx, const SearchBatch& b) override {
    const uint32_t k = b.k;
    const uint32_t depth = RerankDepth(b.params.rerank, k);
    if (std::max(depth, k) > 256)
      return Status(Status::kNotSupported, "re-rank depth or k above 256 is not supported on the GPU");
    if (!pqflat_ && nlist_ == 0) {
      std::vector<float> d(b.nq * k, INFINITY);
      std::vector<uint32_t> r(b.nq * k, UINT32_MAX);
      VDBGPU_CUDA(cudaMemcpyAsync(b.out_dist, d.data(), d.size() * 4, cudaMemcpyHostToDevice, ctx.stream()));
      VDBGPU_CUDA(cudaMemcpyAsync(b.out_row, r.data(), r.size() * 4, cudaMemcpyHostToDevice, ctx.stream()));
      return ctx.Sync("empty ivf search");
    }
    IvfPqArgs a = BaseArgs(b, k, depth);
    a.order = ctx.order();
    a.status = ctx.status_word();
    if (pqflat_) {
      a.mode = kPqFlat;
      a.nprobe = 1;
    } else {
      const uint64_t nprobe = std::clamp<uint64_t>(b.params.nprobe, 1, nlist_);
      if (nprobe > 128) return Status(Status::kNotSupported, "nprobe above 128 is not supported on the GPU");
      a.nprobe = static_cast<int>(nprobe);
      a.mode = metric != 0 ? kIvfShared : (term2_.get() != nullptr ? kIvfPrecomputed : kIvfResidual);
      void *pid, *pdist;
      VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsScratch0, b.nq * nprobe * 4, &pid));
      VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsScratch1, b.nq * nprobe * 4, &pdist));
      SearchBatch cb = b;
      cb.k = static_cast<uint32_t>(nprobe);
      cb.allow = nullptr;
      cb.out_dist = static_cast<float*>(pdist);
      cb.out_row = static_cast<uint32_t*>(pid);
      cb.dist_comps = nullptr;
      VDBGPU_RETURN_IF_ERROR(coarse_index_->Search(ctx, cb));
      a.probe_ids = static_cast<const uint32_t*>(pid);
      a.probe_dist = static_cast<const float*>(pdist);
      // The exact stage takes at most 256 pre-rank keys, at least 1.25 times TopK's depth.
      if (list_mode_ && TensorEnabled() && b.allow == nullptr && b.nq >= kIvfTensorMinQueries &&
          b.nq * a.nprobe <= (uint64_t{1} << 30) && std::max(depth, k) <= 204 &&
          (a.mode == kIvfPrecomputed || a.mode == kIvfResidual)) {
        ctx.Mark(0);
        return ListSearch(ctx, b, k, depth, a.nprobe, a.probe_ids, a.probe_dist);
      }
      void* ord;
      VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsScratch3, (b.nq + nlist_ + 1) * sizeof(uint32_t), &ord));
      uint32_t* counts = static_cast<uint32_t*>(ord) + b.nq;
      VDBGPU_CUDA(LaunchProbeOrder(a.probe_ids, a.nq, a.nprobe, static_cast<uint32_t>(nlist_), counts,
                                   static_cast<uint32_t*>(ord), ctx.stream()));
      a.qorder = static_cast<const uint32_t*>(ord);
    }
    if (IvfPqSmemBytes(a.pd, a.m, a.mode) > 227 * 1024)
      return Status(Status::kNotSupported, "PQ tables do not fit in shared memory");
    void* cand;
    VDBGPU_RETURN_IF_ERROR(ctx.workspace(kWsScratch2, IvfPqCandBytes(a.nq, a.k, a.depth), &cand));
    a.cand = static_cast<uint64_t*>(cand);
    ctx.Mark(2);
    VDBGPU_CUDA(LaunchIvfPq(a, ctx.stream()));
    ctx.Mark(3);
    return Status::OK();
  }

 private:
  bool pqflat_;
  uint64_t n_ = 0;
  uint32_t nlist_ = 0, m_ = 0, dsub_ = 0;
  DeviceBuffer rows_, coarse_, cents_, term2_, off_, ids_, codes_;
  std::unique_ptr<GpuIndex> coarse_index_;
  // List mode (tensor-core pre-rank).
  bool list_mode_ = false;
  uint32_t kpad_ = 0;
  int resid_scale_log2_ = 0;
  DeviceBuffer poff_, resid_, resid_term_;
  CUtensorMap resid_map_;
};

}  // namespace

Status LoadIvfPqIndex(Context& ctx, int type, std::string_view body, int metric, const float* rows,
                      uint64_t n, uint32_t dim, uint32_t pd, std::unique_ptr<GpuIndex>* out) {
  if (type != kIndexIvfPq && type != kIndexPqFlat) return Status(Status::kCorruption, "unknown index type");
  auto idx = std::make_unique<IvfPqGpuIndex>(type == kIndexPqFlat);
  idx->metric = metric;
  idx->dim = dim;
  idx->pd = pd;
  VDBGPU_RETURN_IF_ERROR(idx->Load(ctx, body, rows, n));
  *out = std::move(idx);
  return Status::OK();
}

}  // namespace vdbgpu
