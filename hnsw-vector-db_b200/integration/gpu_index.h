// vdb::GpuIndex: the reference's Index interface (src/index/index.h:36-55) answered by the B200
// search library (include/vdbgpu.h, lib/libvdbgpu.so).
//
// A maintainer adds this header and gpu_index.cc to src/index/ of the reference tree, links
// libvdbgpu.so, and hands GpuIndex::Load's result to Segment::Open as the segment's prebuilt index
// (src/storage/segment_reader.cc:20-27 takes one). Everything above the index stays as it is:
// SearchDiskSegment (src/engine/planner.cc:42-129) calls search() with its DeleteFilter /
// BitmapFilter, ExactOverBitmap reads the segment's rows, and CollectionImpl::Search merges.
// search_batch() is the batched form a GPU-aware SearchBatch uses: one call per (segment, batch).
#pragma once

#include <memory>
#include <string>
#include <string_view>
#include <vector>

#include "index/index.h"
#include "vdbgpu.h"

namespace vdb {

class GpuIndex final : public Index {
 public:
  // LoadIndex (src/index/index.h:61-62) on the GPU: an index file the reference wrote (any of the
  // five types) over the segment's rows, copied to the context's device. The rows stay owned by
  // the segment (the view must outlive this index, as for every Index).
  static StatusOr<std::unique_ptr<Index>> Load(vdbgpu_ctx* ctx, std::string_view file, Metric metric,
                                               const VectorView& view);
  ~GpuIndex() override;

  IndexType type() const override { return type_; }
  // The GPU index is loaded from a file the CPU index wrote; building stays on the CPU.
  Status build(ThreadPool* pool) override;
  void search(const float* q, size_t k, const SearchParams& p, const RowFilter* filter,
              std::vector<Neighbor>& out, IndexSearchStats* stats) const override;
  // nq queries in one call (nq x padded_dim, prepared as PrepareQuery does); out[i] as search()'s.
  Status search_batch(const float* q, size_t nq, size_t k, const SearchParams& p, const RowFilter* filter,
                      std::vector<std::vector<Neighbor>>* out, IndexSearchStats* stats) const;
  size_t size() const override { return view_.rows; }
  size_t memory_bytes() const override;
  // Writes back the file it was loaded from (magic, body, CRC32C footer).
  Status save(WritableFile& f) const override;
  // Index::extend (src/index/index.h:53-54): Flat is rebuilt over `vectors`; an HNSW graph gets
  // the new rows inserted on the GPU (vdbgpu_hnsw_extend); other types are not extendable, as in
  // the reference. The new index lives on the same device.
  StatusOr<std::unique_ptr<Index>> extend(const VectorView& vectors, ThreadPool* pool) const override;

 private:
  GpuIndex(vdbgpu_ctx* ctx, vdbgpu_index* h, const VectorView& view, IndexType type, Metric metric, std::string file)
      : ctx_(ctx), h_(h), view_(view), type_(type), metric_(metric), file_(std::move(file)) {}
  Status Error(int rc) const;
  vdbgpu_ctx* ctx_;
  vdbgpu_index* h_;
  VectorView view_;
  IndexType type_;
  Metric metric_;
  std::string file_;
};

}  // namespace vdb
