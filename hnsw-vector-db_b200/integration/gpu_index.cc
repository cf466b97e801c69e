// vdb::GpuIndex (gpu_index.h): forwards the reference's Index calls to the C ABI of vdbgpu.h.
#include "gpu_index.h"

#include <algorithm>
#include <cstdint>

namespace vdb {

Status GpuIndex::Error(int rc) const {
  char msg[512] = {};
  vdbgpu_last_error(ctx_, msg, sizeof(msg));
  // vdbgpu_status values are vdb::Status::Code values (include/vdb/status.h:14-26).
  switch (rc) {
    case VDBGPU_INVALID_ARGUMENT: return Status::InvalidArgument(msg);
    case VDBGPU_NOT_FOUND: return Status::NotFound(msg);
    case VDBGPU_CORRUPTION: return Status::Corruption(msg);
    case VDBGPU_RESOURCE_EXHAUSTED: return Status::ResourceExhausted(msg);
    case VDBGPU_UNAVAILABLE: return Status::Unavailable(msg);
    case VDBGPU_NOT_SUPPORTED: return Status::NotSupported(msg);
    default: return Status::Internal(msg);
  }
}

StatusOr<std::unique_ptr<Index>> GpuIndex::Load(vdbgpu_ctx* ctx, std::string_view file, Metric metric,
                                                const VectorView& view) {
  int type = -1;
  int rc = vdbgpu_index_file_inspect(file.data(), file.size(), &type);
  if (rc != VDBGPU_OK || type < 0 || type > 4) return Status::Corruption("not a vdb index file");
  vdbgpu_index* h = nullptr;
  rc = vdbgpu_index_load(ctx, file.data(), file.size(), static_cast<int>(metric), view.data, view.rows,
                         static_cast<uint32_t>(view.dim), static_cast<uint32_t>(view.padded_dim), &h);
  if (rc != VDBGPU_OK) {
    char msg[512] = {};
    vdbgpu_last_error(ctx, msg, sizeof(msg));
    return rc == VDBGPU_CORRUPTION ? Status::Corruption(msg) : Status::Internal(msg);
  }
  return std::unique_ptr<Index>(new GpuIndex(ctx, h, view, static_cast<IndexType>(type), metric, std::string(file)));
}

GpuIndex::~GpuIndex() { vdbgpu_index_free(h_); }

Status GpuIndex::build(ThreadPool*) {
  return Status::NotSupported("a GpuIndex is loaded from an index file the CPU index wrote");
}

size_t GpuIndex::memory_bytes() const {
  vdbgpu_index_info info{};
  return vdbgpu_index_get_info(h_, &info) == VDBGPU_OK ? static_cast<size_t>(info.device_bytes) : 0;
}

Status GpuIndex::save(WritableFile& f) const {
  std::string_view magic, body;
  VDB_RETURN_IF_ERROR(CheckIndexFile(file_, &magic, &body));
  return WriteIndexFile(f, magic, std::string(body));
}

StatusOr<std::unique_ptr<Index>> GpuIndex::extend(const VectorView& vectors, ThreadPool*) const {
  if (vectors.rows < view_.rows || vectors.padded_dim != view_.padded_dim)
    return Status::InvalidArgument("extend needs a superset of the indexed rows");
  if (type_ == IndexType::Flat) return Load(ctx_, file_, metric_, vectors);  // a flat index has no state
  if (type_ != IndexType::Hnsw)
    return Status::NotSupported(std::string("extend is not supported by ") + IndexTypeName(type_));
  void* out = nullptr;
  size_t nbytes = 0;
  const int rc = vdbgpu_hnsw_extend(ctx_, static_cast<int>(metric_), file_.data(), file_.size(), vectors.data,
                                    vectors.rows, static_cast<uint32_t>(vectors.dim),
                                    static_cast<uint32_t>(vectors.padded_dim), &out, &nbytes);
  if (rc != VDBGPU_OK) return Error(rc);
  std::string file(static_cast<const char*>(out), nbytes);
  vdbgpu_buffer_free(out);
  return Load(ctx_, file, metric_, vectors);
}

Status GpuIndex::search_batch(const float* q, size_t nq, size_t k, const SearchParams& p, const RowFilter* filter,
                              std::vector<std::vector<Neighbor>>* out, IndexSearchStats* stats) const {
  out->assign(nq, {});
  if (nq == 0 || k == 0) return Status::OK();
  std::vector<uint64_t> bits;
  if (filter != nullptr) {  // the RowFilter as a dense bitset of allowed rows (bit r of word r/64)
    bits.assign((view_.rows + 63) / 64, 0);
    for (size_t r = 0; r < view_.rows; ++r)
      if (filter->allowed(static_cast<InternalId>(r))) bits[r >> 6] |= uint64_t{1} << (r & 63);
  }
  vdbgpu_search_params gp;
  vdbgpu_search_params_default(&gp);
  gp.ef = p.ef;
  gp.nprobe = p.nprobe;
  gp.rerank = p.rerank;
  std::vector<float> dist(nq * k);
  std::vector<uint32_t> rows(nq * k);
  std::vector<uint64_t> dc(nq);
  const int rc = vdbgpu_index_search(h_, q, nq, static_cast<uint32_t>(k), &gp, filter != nullptr ? bits.data() : nullptr,
                                     dist.data(), rows.data(), dc.data());
  if (rc != VDBGPU_OK) return Error(rc);
  for (size_t i = 0; i < nq; ++i) {
    auto& o = (*out)[i];
    for (size_t j = 0; j < k && rows[i * k + j] != UINT32_MAX; ++j) o.push_back({dist[i * k + j], rows[i * k + j]});
  }
  if (stats != nullptr) {
    for (uint64_t d : dc) stats->distance_computations += d;
    // IndexSearchStats::ef as HnswIndex / HnswSq8Index report it (src/index/hnsw/hnsw_index.cc:32, 100).
    if (type_ == IndexType::Hnsw) {
      stats->ef = std::max(p.ef, k);
    } else if (type_ == IndexType::HnswSq8) {
      const size_t depth = p.rerank < 0 ? std::max(p.ef, k) : static_cast<size_t>(p.rerank);
      stats->ef = std::max({p.ef, k, depth});
    }
  }
  return Status::OK();
}

void GpuIndex::search(const float* q, size_t k, const SearchParams& p, const RowFilter* filter,
                      std::vector<Neighbor>& out, IndexSearchStats* stats) const {
  // Index::search cannot fail (src/index/index.h:44-45): a device error returns no neighbours.
  std::vector<std::vector<Neighbor>> all;
  out.clear();
  if (search_batch(q, 1, k, p, filter, &all, stats).ok()) out = std::move(all[0]);
}

}  // namespace vdb
