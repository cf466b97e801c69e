// IVF-PQ (IvfPqIndex, src/index/quant/ivf_pq.h:42-81) and PQ-flat (PqFlatIndex, :12-36) on the
// GPU, loaded from the reference's own index files (IvfPqIndex::save, ivf_pq.cc:236-249;
// PqFlatIndex::save, ivf_pq.cc:78-84).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "formats.h"
#include "ivfpq.cuh"
#include "runtime.h"

namespace vdbgpu {
namespace {

template <class T>
Status Upload(Context& ctx, const T* p, size_t count, DeviceBuffer* out) {
  VDBGPU_RETURN_IF_ERROR(out->alloc(std::max<size_t>(1, count) * sizeof(T)));
  if (count > 0)
    VDBGPU_CUDA(cudaMemcpyAsync(out->get(), p, count * sizeof(T), cudaMemcpyDefault, ctx.stream()));
  return Status::OK();
}

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
           codes_.size() + (coarse_index_ ? coarse_index_->device_bytes() : 0);
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
    }
    return ctx.Sync("ivf-pq index load");
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
    IvfPqArgs a{};
    a.nq = static_cast<int>(b.nq);
    a.pd = static_cast<int>(pd);
    a.dim = static_cast<int>(dim);
    a.m = static_cast<int>(m_);
    a.dsub = static_cast<int>(dsub_);
    a.k = static_cast<int>(k);
    a.depth = static_cast<int>(depth);
    a.metric = metric;
    a.order = ctx.order();
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
