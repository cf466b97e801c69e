// The C ABI of include/vdbgpu.h over the C++ runtime. No exception or C++ type crosses it;
// every failure becomes a vdbgpu_status code plus a message readable with vdbgpu_last_error.
#include "../../include/vdbgpu.h"

#include <algorithm>
#include <initializer_list>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "collection.h"
#include "filter.h"
#include "formats.h"
#include "noalloc.h"
#include "runtime.h"
#include "shard.h"

struct vdbgpu_ctx {
  std::unique_ptr<vdbgpu::Context> c;
  std::string open_error;
};

struct vdbgpu_index {
  vdbgpu_ctx* ctx;
  std::unique_ptr<vdbgpu::GpuIndex> idx;
};

struct vdbgpu_collection {
  vdbgpu_ctx* ctx;
  std::unique_ptr<vdbgpu::GpuCollection> c;
};

struct vdbgpu_shard_group {
  vdbgpu_ctx* ctx;
  std::unique_ptr<vdbgpu::ShardGroup> g;
};

static_assert(sizeof(vdbgpu_hit) == sizeof(vdbgpu::HitRecord), "vdbgpu_hit layout");

namespace {

using vdbgpu::Status;

int Fail(vdbgpu_ctx* ctx, const Status& s) {
  if (ctx != nullptr && ctx->c) ctx->c->set_error(s.message());
  return static_cast<int>(s.code());
}

// True for memory the context's device may use directly. Callers first reject other GPUs'
// memory (RejectForeign), so false means host memory to be staged through a copy.
bool IsDevicePtr(const void* p, int device) {
  return p != nullptr && vdbgpu::WherePointer(p, device) == vdbgpu::MemWhere::kDevice;
}

// kInvalidArgument when any of the caller's buffers is another GPU's memory.
Status RejectForeign(int device, std::initializer_list<std::pair<const void*, const char*>> bufs) {
  for (const auto& b : bufs) VDBGPU_RETURN_IF_ERROR(vdbgpu::RejectOtherDevice(b.first, device, b.second));
  return Status::OK();
}

uint64_t RoundUp(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

}  // namespace

extern "C" {

int vdbgpu_abi_version(void) { return VDBGPU_ABI_VERSION; }

int vdbgpu_launch_count(uint64_t* out) {
  if (out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = vdbgpu::LaunchCount();
  return VDBGPU_OK;
}

int vdbgpu_device_count(int* out) {
  if (out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  *out = n;
  return VDBGPU_OK;
}

int vdbgpu_open(int device, vdbgpu_ctx** out) {
  if (out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = nullptr;
  auto* h = new (std::nothrow) vdbgpu_ctx;
  if (h == nullptr) return VDBGPU_RESOURCE_EXHAUSTED;
  Status s = vdbgpu::Context::Open(device, &h->c);
  if (!s.ok()) {
    delete h;
    return static_cast<int>(s.code());
  }
  *out = h;
  return VDBGPU_OK;
}

void vdbgpu_close(vdbgpu_ctx* ctx) { delete ctx; }

size_t vdbgpu_last_error(const vdbgpu_ctx* ctx, char* buf, size_t cap) {
  const std::string empty;
  const std::string& e = (ctx != nullptr && ctx->c) ? ctx->c->last_error() : empty;
  if (buf != nullptr && cap > 0) {
    const size_t n = std::min(cap - 1, e.size());
    std::memcpy(buf, e.data(), n);
    buf[n] = '\0';
  }
  return e.size();
}

int vdbgpu_set_stream(vdbgpu_ctx* ctx, void* stream) {
  if (ctx == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  ctx->c->set_user_stream(static_cast<cudaStream_t>(stream));
  return VDBGPU_OK;
}

int vdbgpu_set_timing(vdbgpu_ctx* ctx, int enable) {
  if (ctx == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  Status s = ctx->c->EnableTiming(enable != 0);
  return s.ok() ? VDBGPU_OK : Fail(ctx, s);
}

int vdbgpu_stage_times(vdbgpu_ctx* ctx, float* out, int cap) {
  if (ctx == nullptr || out == nullptr) return 0;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  return ctx->c->StageTimes(out, cap);
}

int vdbgpu_stage_counters(vdbgpu_ctx* ctx, uint64_t* out, int cap) {
  if (ctx == nullptr || out == nullptr) return 0;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  unsigned long long tmp[8];
  const int n = ctx->c->Counters(tmp, cap < 8 ? cap : 8);
  for (int i = 0; i < n; ++i) out[i] = tmp[i];
  return n;
}

int vdbgpu_synchronize(vdbgpu_ctx* ctx) {
  if (ctx == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  Status s = ctx->c->Sync("synchronize");
  return s.ok() ? VDBGPU_OK : Fail(ctx, s);
}

void vdbgpu_search_params_default(vdbgpu_search_params* p) {
  if (p == nullptr) return;
  p->ef = 64;
  p->nprobe = 16;
  p->rerank = -1;
  p->strategy = 0;
  p->prefilter_threshold = 10000;
  p->post_filter_alpha = 10;
}

int vdbgpu_index_load(vdbgpu_ctx* ctx, const void* file_bytes, size_t nbytes, int metric,
                      const float* rows, uint64_t nrows, uint32_t dim, uint32_t padded_dim,
                      vdbgpu_index** out) {
  if (ctx == nullptr || out == nullptr || file_bytes == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = nullptr;
  if (metric < 0 || metric > 2 || dim == 0 || dim > padded_dim || padded_dim % 16 != 0 ||
      (nrows > 0 && rows == nullptr))
    return Fail(ctx, Status(Status::kInvalidArgument, "bad index geometry or metric"));
  if (nrows > 0xFFFFFFFFull)
    return Fail(ctx, Status(Status::kInvalidArgument, "a segment holds at most 2^32 - 1 rows"));
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  std::unique_ptr<vdbgpu::GpuIndex> idx;
  Status s = vdbgpu::LoadIndexFile(*ctx->c, file_bytes, nbytes, metric, rows, nrows, dim,
                                   padded_dim, &idx);
  if (!s.ok()) return Fail(ctx, s);
  *out = new vdbgpu_index{ctx, std::move(idx)};
  return VDBGPU_OK;
}

int vdbgpu_index_create(vdbgpu_ctx* ctx, int type, int metric, const float* rows, uint64_t nrows,
                        uint32_t dim, uint32_t padded_dim, vdbgpu_index** out) {
  if (ctx == nullptr || out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = nullptr;
  if (metric < 0 || metric > 2 || dim == 0 || dim > padded_dim || padded_dim % 16 != 0 ||
      (nrows > 0 && rows == nullptr))
    return Fail(ctx, Status(Status::kInvalidArgument, "bad index geometry or metric"));
  if (nrows > 0xFFFFFFFFull)
    return Fail(ctx, Status(Status::kInvalidArgument, "a segment holds at most 2^32 - 1 rows"));
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  std::unique_ptr<vdbgpu::GpuIndex> idx;
  Status s;
  if (type == VDBGPU_INDEX_FLAT) {
    s = vdbgpu::CreateFlatIndex(*ctx->c, metric, rows, nrows, dim, padded_dim, &idx);
  } else if (type == VDBGPU_INDEX_SQ8_FLAT) {
    s = vdbgpu::CreateSq8FlatIndex(*ctx->c, metric, rows, nrows, dim, padded_dim, nullptr, nullptr,
                                   nullptr, &idx);
  } else {
    s = Status(Status::kNotSupported,
               "only FLAT and SQ8_FLAT are built on the GPU; load other types from index files");
  }
  if (!s.ok()) return Fail(ctx, s);
  *out = new vdbgpu_index{ctx, std::move(idx)};
  return VDBGPU_OK;
}

void vdbgpu_index_free(vdbgpu_index* index) {
  if (index == nullptr) return;
  if (index->ctx != nullptr && index->ctx->c) {
    std::lock_guard<std::mutex> g(index->ctx->c->mu());
    cudaSetDevice(index->ctx->c->device());
    cudaStreamSynchronize(index->ctx->c->stream());
    index->idx.reset();
  }
  delete index;
}

int vdbgpu_index_get_info(const vdbgpu_index* index, vdbgpu_index_info* out) {
  if (index == nullptr || out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  out->type = index->idx->type();
  out->metric = index->idx->metric;
  out->rows = index->idx->rows();
  out->dim = index->idx->dim;
  out->padded_dim = index->idx->pd;
  out->device_bytes = index->idx->device_bytes();
  return VDBGPU_OK;
}

int vdbgpu_index_search(vdbgpu_index* index, const float* queries, uint64_t nq, uint32_t k,
                        const vdbgpu_search_params* params, const uint64_t* allow_bits,
                        float* out_dist, uint32_t* out_row, uint64_t* out_dist_comps) {
  if (index == nullptr) return VDBGPU_INVALID_ARGUMENT;
  vdbgpu_ctx* ctx = index->ctx;
  if (nq == 0 || k == 0) return VDBGPU_OK;
  if (queries == nullptr || out_dist == nullptr || out_row == nullptr)
    return Fail(ctx, Status(Status::kInvalidArgument, "null query or output buffer"));
  if (k > 10000) return Fail(ctx, Status(Status::kInvalidArgument, "k must be in 1..10000"));
  vdbgpu::Context& c = *ctx->c;
  std::lock_guard<std::mutex> g(c.mu());
  cudaSetDevice(c.device());
  vdbgpu::GpuIndex& idx = *index->idx;
  const uint32_t pd = idx.pd;
  const cudaStream_t st = c.stream();

  vdbgpu::SearchBatch b{};
  b.nq = nq;
  b.k = k;
  if (params != nullptr) {
    b.params.ef = params->ef;
    b.params.nprobe = params->nprobe;
    b.params.rerank = params->rerank;
    b.params.strategy = params->strategy;
    b.params.prefilter_threshold = params->prefilter_threshold;
    b.params.post_filter_alpha = params->post_filter_alpha;
  }
  Status s;
  auto check = [&](const Status& x) { s = x; return x.ok(); };
  auto cuda = [&](cudaError_t e, const char* what) { return check(vdbgpu::CudaStatus(e, what)); };

  if (!check(RejectForeign(c.device(), {{queries, "the query buffer"}, {allow_bits, "the filter bitset"},
                                         {out_dist, "the distance output"}, {out_row, "the row output"},
                                         {out_dist_comps, "the distance-count output"}})))
    return Fail(ctx, s);
  // Queries.
  void* p = nullptr;
  if (IsDevicePtr(queries, c.device())) {
    b.queries = queries;
  } else {
    if (!check(c.workspace(vdbgpu::kWsQueries, nq * pd * sizeof(float), &p))) return Fail(ctx, s);
    if (!cuda(cudaMemcpyAsync(p, queries, nq * pd * sizeof(float), cudaMemcpyHostToDevice, st), "copy queries"))
      return Fail(ctx, s);
    b.queries = static_cast<const float*>(p);
  }
  // Filter bitset: 64-bit words (little-endian) seen as 32-bit words, padded to 256 rows.
  if (allow_bits != nullptr) {
    const uint64_t n = idx.rows();
    const uint64_t words64 = (n + 63) / 64;
    const uint64_t bytes = RoundUp(std::max<uint64_t>(n, 1), 256) / 8 + 64;
    if (!check(c.workspace(vdbgpu::kWsAllow, bytes, &p))) return Fail(ctx, s);
    if (!cuda(cudaMemsetAsync(p, 0, bytes, st), "clear filter")) return Fail(ctx, s);
    if (words64 > 0 &&
        !cuda(cudaMemcpyAsync(p, allow_bits, words64 * 8, cudaMemcpyDefault, st), "copy filter"))
      return Fail(ctx, s);
    b.allow = static_cast<const uint32_t*>(p);
  }
  // Outputs.
  const bool dev_out = IsDevicePtr(out_dist, c.device()) && IsDevicePtr(out_row, c.device());
  if (dev_out) {
    b.out_dist = out_dist;
    b.out_row = out_row;
  } else {
    void* od = nullptr;
    void* orow = nullptr;
    if (!check(c.workspace(vdbgpu::kWsOutDist, nq * k * sizeof(float), &od)) ||
        !check(c.workspace(vdbgpu::kWsOutRow, nq * k * sizeof(uint32_t), &orow)))
      return Fail(ctx, s);
    b.out_dist = static_cast<float*>(od);
    b.out_row = static_cast<uint32_t*>(orow);
  }
  const bool dev_dc = out_dist_comps != nullptr && IsDevicePtr(out_dist_comps, c.device());
  if (out_dist_comps != nullptr) {
    if (dev_dc) {
      b.dist_comps = out_dist_comps;
    } else {
      if (!check(c.workspace(vdbgpu::kWsDistComps, nq * sizeof(uint64_t), &p))) return Fail(ctx, s);
      b.dist_comps = static_cast<uint64_t*>(p);
    }
  }
  if (!check(idx.Search(c, b))) return Fail(ctx, s);
  if (!dev_out) {
    if (!cuda(cudaMemcpyAsync(out_dist, b.out_dist, nq * k * sizeof(float), cudaMemcpyDeviceToHost, st), "copy distances") ||
        !cuda(cudaMemcpyAsync(out_row, b.out_row, nq * k * sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "copy rows"))
      return Fail(ctx, s);
  }
  if (out_dist_comps != nullptr && !dev_dc) {
    if (!cuda(cudaMemcpyAsync(out_dist_comps, b.dist_comps, nq * sizeof(uint64_t), cudaMemcpyDeviceToHost, st), "copy stats"))
      return Fail(ctx, s);
  }
  if (!check(c.Sync("search"))) return Fail(ctx, s);
  return VDBGPU_OK;
}

int vdbgpu_index_sq8_export(const vdbgpu_index* index, float* vmin, float* scale, uint8_t* codes) {
  if (index == nullptr || vmin == nullptr || scale == nullptr) return VDBGPU_INVALID_ARGUMENT;
  vdbgpu_ctx* ctx = index->ctx;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  Status s = index->idx->ExportSq8(*ctx->c, vmin, scale, codes);
  return s.ok() ? VDBGPU_OK : Fail(ctx, s);
}

int vdbgpu_index_search_noalloc(vdbgpu_index* index, const float* queries, uint64_t nq, uint32_t k,
                                const vdbgpu_search_params* params, float* out_dist,
                                uint32_t* out_row, void* stream) {
  if (index == nullptr) return VDBGPU_INVALID_ARGUMENT;
  vdbgpu_ctx* ctx = index->ctx;
  if (nq == 0 || k == 0) return VDBGPU_OK;
  if (queries == nullptr || out_dist == nullptr || out_row == nullptr)
    return Fail(ctx, Status(Status::kInvalidArgument, "null query or output buffer"));
  vdbgpu::Context& c = *ctx->c;
  std::lock_guard<std::mutex> g(c.mu());
  cudaSetDevice(c.device());
  // Host buffers would need staging copies in allocated memory: only device pointers are taken.
  if (Status f = RejectForeign(c.device(), {{queries, "the query buffer"}, {out_dist, "the distance output"},
                                            {out_row, "the row output"}});
      !f.ok())
    return Fail(ctx, f);
  if (!IsDevicePtr(queries, c.device()) || !IsDevicePtr(out_dist, c.device()) || !IsDevicePtr(out_row, c.device()))
    return Fail(ctx, Status(Status::kInvalidArgument,
                            "the allocation-free search takes device pointers for queries and outputs"));
  vdbgpu::SearchBatch b{};
  b.queries = queries;
  b.nq = nq;
  b.k = k;
  if (params != nullptr) {
    b.params.ef = params->ef;
    b.params.nprobe = params->nprobe;
    b.params.rerank = params->rerank;
    b.params.strategy = params->strategy;
  }
  b.out_dist = out_dist;
  b.out_row = out_row;
  const vdbgpu::ScanOperands* op = nullptr;
  int cpre = 0, depth = 0;
  Status s = index->idx->ScanPlan(b, &op, &cpre, &depth);
  if (!s.ok()) return Fail(ctx, s);
  const cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : c.stream();
  s = vdbgpu::ScanSearchNoAlloc(c, *op, index->idx->metric, index->idx->pd, b, cpre, depth, st);
  if (!s.ok()) return Fail(ctx, s);
  if (cudaStreamSynchronize(st) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    return Fail(ctx, vdbgpu::CudaStatus(e == cudaSuccess ? cudaErrorUnknown : e, "allocation-free search"));
  }
  s = c.CheckDeviceStatus("allocation-free search");
  return s.ok() ? VDBGPU_OK : Fail(ctx, s);
}

int vdbgpu_index_file_inspect(const void* file_bytes, size_t nbytes, int* type) {
  if (file_bytes == nullptr || type == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::string_view magic, body;
  Status s = vdbgpu::CheckIndexFile(std::string_view(static_cast<const char*>(file_bytes), nbytes),
                                    &magic, &body);
  if (!s.ok()) return static_cast<int>(s.code());
  *type = vdbgpu::IndexTypeForMagic(magic);
  return *type < 0 ? VDBGPU_CORRUPTION : VDBGPU_OK;
}


// ------------------------------------------------------------------------------ collections

namespace {

vdbgpu::SearchParams ToParams(const vdbgpu_search_params* params) {
  vdbgpu::SearchParams p;
  if (params != nullptr) {
    p.ef = params->ef;
    p.nprobe = params->nprobe;
    p.rerank = params->rerank;
    p.strategy = params->strategy;
    p.prefilter_threshold = params->prefilter_threshold;
    p.post_filter_alpha = params->post_filter_alpha;
  }
  return p;
}

bool BadStrategy(const vdbgpu_search_params* params) {
  return params != nullptr && (params->strategy < 0 || params->strategy > 3);
}

}  // namespace

int vdbgpu_collection_open(vdbgpu_ctx* ctx, const char* path, uint32_t shard, uint32_t nshards,
                           vdbgpu_collection** out) {
  if (ctx == nullptr || path == nullptr || out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = nullptr;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  std::unique_ptr<vdbgpu::GpuCollection> c;
  Status s = vdbgpu::GpuCollection::Open(*ctx->c, path, shard, nshards, &c);
  if (!s.ok()) return Fail(ctx, s);
  *out = new vdbgpu_collection{ctx, std::move(c)};
  return VDBGPU_OK;
}

int vdbgpu_collection_create(vdbgpu_ctx* ctx, const char* options_json, vdbgpu_collection** out) {
  if (ctx == nullptr || options_json == nullptr || out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = nullptr;
  std::unique_ptr<vdbgpu::GpuCollection> c;
  Status s = vdbgpu::GpuCollection::Create(options_json, &c);
  if (!s.ok()) return Fail(ctx, s);
  *out = new vdbgpu_collection{ctx, std::move(c)};
  return VDBGPU_OK;
}

int vdbgpu_collection_add_segment(vdbgpu_collection* c, uint32_t segment_id, uint32_t ordinal,
                                  const float* rows, uint64_t n, const uint64_t* ids, const void* meta,
                                  size_t meta_bytes, const void* index_file, size_t index_bytes) {
  if (c == nullptr || index_file == nullptr || (n > 0 && (rows == nullptr || ids == nullptr)))
    return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(c->ctx->c->mu());
  cudaSetDevice(c->ctx->c->device());
  Status s = c->c->AddSegment(*c->ctx->c, segment_id, ordinal, rows, n, ids,
                              meta != nullptr ? std::string_view(static_cast<const char*>(meta), meta_bytes)
                                              : std::string_view(),
                              std::string_view(static_cast<const char*>(index_file), index_bytes));
  return s.ok() ? VDBGPU_OK : Fail(c->ctx, s);
}

int vdbgpu_collection_set_deleted(vdbgpu_collection* c, uint32_t segment_id, const uint32_t* bits) {
  if (c == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(c->ctx->c->mu());
  cudaSetDevice(c->ctx->c->device());
  Status s = c->c->SetDeleted(*c->ctx->c, segment_id, bits);
  return s.ok() ? VDBGPU_OK : Fail(c->ctx, s);
}

void vdbgpu_collection_free(vdbgpu_collection* c) {
  if (c == nullptr) return;
  if (c->ctx != nullptr && c->ctx->c) {
    std::lock_guard<std::mutex> g(c->ctx->c->mu());
    cudaSetDevice(c->ctx->c->device());
    cudaStreamSynchronize(c->ctx->c->stream());
    c->c.reset();
  }
  delete c;
}

int vdbgpu_collection_get_info(const vdbgpu_collection* c, vdbgpu_collection_info* out) {
  if (c == nullptr || out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  const auto& o = c->c->options();
  out->dim = o.dim;
  out->padded_dim = o.pd;
  out->metric = o.metric;
  out->index_type = o.index_type;
  out->segments_total = c->c->segments_total();
  out->segments_local = static_cast<uint32_t>(c->c->segments_local());
  out->rows_local = c->c->rows_local();
  out->device_bytes = c->c->device_bytes();
  return VDBGPU_OK;
}

int vdbgpu_collection_search_grouped(vdbgpu_collection* c, const float* queries, uint64_t nq, uint32_t k,
                                     const vdbgpu_search_params* params, const char* const* filters,
                                     uint32_t nfilters, const int32_t* query_filter, uint64_t* out_ids,
                                     float* out_dist, vdbgpu_hit* out_hits) {
  if (c == nullptr || (nq > 0 && queries == nullptr) || (nfilters > 0 && filters == nullptr) ||
      ((out_ids == nullptr) != (out_dist == nullptr)))
    return VDBGPU_INVALID_ARGUMENT;
  if (BadStrategy(params)) return Fail(c->ctx, Status(Status::kInvalidArgument, "bad strategy"));
  vdbgpu::GpuCollection::Request r;
  r.queries = queries;
  r.nq = nq;
  r.k = k;
  r.params = ToParams(params);
  for (uint32_t i = 0; i < nfilters; ++i) {
    if (filters[i] == nullptr) return Fail(c->ctx, Status(Status::kInvalidArgument, "null filter"));
    r.filters.emplace_back(filters[i]);
  }
  r.query_filter = query_filter;
  r.out_ids = out_ids;
  r.out_dist = out_dist;
  r.out_records = reinterpret_cast<vdbgpu::HitRecord*>(out_hits);
  std::lock_guard<std::mutex> g(c->ctx->c->mu());
  cudaSetDevice(c->ctx->c->device());
  Status s = c->c->Search(*c->ctx->c, r);
  return s.ok() ? VDBGPU_OK : Fail(c->ctx, s);
}

int vdbgpu_collection_search(vdbgpu_collection* c, const float* queries, uint64_t nq, uint32_t k,
                             const vdbgpu_search_params* params, const char* filter_json, uint64_t* out_ids,
                             float* out_dist) {
  if (out_ids == nullptr || out_dist == nullptr) return VDBGPU_INVALID_ARGUMENT;
  const char* f[1] = {filter_json};
  return vdbgpu_collection_search_grouped(c, queries, nq, k, params, f, filter_json != nullptr ? 1 : 0,
                                          nullptr, out_ids, out_dist, nullptr);
}

int vdbgpu_collection_stats(vdbgpu_collection* c, int enable, uint64_t* out, int cap) {
  if (c == nullptr) return 0;
  if (enable >= 0) c->c->set_stats(enable != 0);
  const int n = std::min(cap, vdbgpu::GpuCollection::kStats);
  for (int i = 0; out != nullptr && i < n; ++i) out[i] = c->c->stats()[i];
  return out != nullptr ? n : 0;
}

int vdbgpu_collection_explain(vdbgpu_collection* c, const float* query, uint32_t k,
                              const vdbgpu_search_params* params, const char* filter_json, char* out_json,
                              size_t cap) {
  if (c == nullptr || query == nullptr || out_json == nullptr) return VDBGPU_INVALID_ARGUMENT;
  if (BadStrategy(params)) return Fail(c->ctx, Status(Status::kInvalidArgument, "bad strategy"));
  vdbgpu::GpuCollection::Request r;
  r.queries = query;
  r.nq = 1;
  r.k = k;
  r.params = ToParams(params);
  if (filter_json != nullptr) r.filters.emplace_back(filter_json);
  std::vector<std::vector<vdbgpu::PartExplain>> ex;
  r.explain = &ex;
  std::lock_guard<std::mutex> g(c->ctx->c->mu());
  cudaSetDevice(c->ctx->c->device());
  Status s = c->c->Search(*c->ctx->c, r);
  if (!s.ok()) return Fail(c->ctx, s);
  std::string j = "[";
  for (size_t i = 0; i < ex[0].size(); ++i) {
    const auto& e = ex[0][i];
    if (i > 0) j += ",";
    j += "{\"id\":" + std::to_string(e.segment_id) + ",\"kind\":\"" + (e.is_mutable ? "mutable" : "disk") +
         "\",\"strategy\":\"" + e.strategy +
         "\",\"matches\":" + std::to_string(e.matches) + ",\"live_rows\":" + std::to_string(e.live_rows) +
         ",\"distance_computations\":" + std::to_string(e.dc) + ",\"results\":" + std::to_string(e.results) +
         "}";
  }
  j += "]";
  if (j.size() + 1 > cap) return Fail(c->ctx, Status(Status::kResourceExhausted, "explain buffer too small"));
  std::memcpy(out_json, j.c_str(), j.size() + 1);
  return VDBGPU_OK;
}

int vdbgpu_collection_filter_bitmap(vdbgpu_collection* c, const char* filter_json, uint32_t segment_id,
                                    uint32_t* out_words, uint64_t* matches) {
  if (c == nullptr || filter_json == nullptr || out_words == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(c->ctx->c->mu());
  cudaSetDevice(c->ctx->c->device());
  Status s = c->c->FilterBitmap(*c->ctx->c, filter_json, segment_id, out_words, matches);
  return s.ok() ? VDBGPU_OK : Fail(c->ctx, s);
}

int vdbgpu_merge_hits(vdbgpu_ctx* ctx, const vdbgpu_hit* lists, uint32_t nlists, uint64_t nq, uint32_t k,
                      uint64_t* out_ids, float* out_dist, vdbgpu_hit* out_hits) {
  if (ctx == nullptr || (nlists > 0 && nq > 0 && lists == nullptr) ||
      ((out_ids == nullptr) != (out_dist == nullptr)))
    return VDBGPU_INVALID_ARGUMENT;
  if (k == 0 || k > 240) return Fail(ctx, Status(Status::kInvalidArgument, "k must be in 1..240"));
  if (nq == 0) return VDBGPU_OK;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  vdbgpu::Context& cx = *ctx->c;
  cudaStream_t st = cx.stream();
  const size_t nrec = static_cast<size_t>(nlists) * nq * k;
  const vdbgpu_hit* in = lists;
  void* buf;
  Status s;
  s = RejectForeign(cx.device(), {{lists, "the hit lists"}, {out_ids, "the id output"}, {out_dist, "the distance output"},
                                  {out_hits, "the hit output"}});
  if (!s.ok()) return Fail(ctx, s);
  if (nrec > 0 && !IsDevicePtr(lists, cx.device())) {
    s = cx.workspace(vdbgpu::kWsScratch0, nrec * sizeof(vdbgpu_hit), &buf);
    if (!s.ok()) return Fail(ctx, s);
    if (cudaMemcpyAsync(buf, lists, nrec * sizeof(vdbgpu_hit), cudaMemcpyHostToDevice, st) != cudaSuccess)
      return Fail(ctx, Status(Status::kInternal, "copy hit lists"));
    in = static_cast<const vdbgpu_hit*>(buf);
  }
  vdbgpu::MergeArgs ma{};
  ma.kind = 1;
  ma.nlists = static_cast<int>(nlists);
  ma.k = static_cast<int>(k);
  ma.nq = nq;
  ma.records = reinterpret_cast<const vdbgpu::HitRecord*>(in);
  const bool ids_dev = IsDevicePtr(out_ids, cx.device()) && IsDevicePtr(out_dist, cx.device());
  const bool hits_dev = IsDevicePtr(out_hits, cx.device());
  void *ib = nullptr, *db = nullptr, *hb = nullptr;
  if (out_ids != nullptr) {
    if (ids_dev) {
      ma.out_ids = out_ids;
      ma.out_dist = out_dist;
    } else {
      if (!(s = cx.workspace(vdbgpu::kWsScratch1, nq * k * 8, &ib)).ok()) return Fail(ctx, s);
      if (!(s = cx.workspace(vdbgpu::kWsScratch2, nq * k * 4, &db)).ok()) return Fail(ctx, s);
      ma.out_ids = static_cast<uint64_t*>(ib);
      ma.out_dist = static_cast<float*>(db);
    }
  }
  if (out_hits != nullptr) {
    if (hits_dev) {
      ma.out_records = reinterpret_cast<vdbgpu::HitRecord*>(out_hits);
    } else {
      if (!(s = cx.workspace(vdbgpu::kWsScratch3, nq * k * sizeof(vdbgpu_hit), &hb)).ok()) return Fail(ctx, s);
      ma.out_records = static_cast<vdbgpu::HitRecord*>(hb);
    }
  }
  if (vdbgpu::LaunchMerge(ma, st) != cudaSuccess) return Fail(ctx, Status(Status::kInternal, "merge launch"));
  if (ib != nullptr) {
    cudaMemcpyAsync(out_ids, ib, nq * k * 8, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(out_dist, db, nq * k * 4, cudaMemcpyDeviceToHost, st);
  }
  if (hb != nullptr) cudaMemcpyAsync(out_hits, hb, nq * k * sizeof(vdbgpu_hit), cudaMemcpyDeviceToHost, st);
  s = cx.Sync("merge hits");
  return s.ok() ? VDBGPU_OK : Fail(ctx, s);
}

int vdbgpu_shard_id(void* out_id) {
  if (out_id == nullptr) return VDBGPU_INVALID_ARGUMENT;
  return static_cast<int>(vdbgpu::ShardUniqueId(out_id).code());
}

int vdbgpu_shard_group_open(vdbgpu_ctx* ctx, const void* id, int rank, int nranks, int timeout_ms,
                            vdbgpu_shard_group** out) {
  if (ctx == nullptr || id == nullptr || out == nullptr) return VDBGPU_INVALID_ARGUMENT;
  *out = nullptr;
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  std::unique_ptr<vdbgpu::ShardGroup> sg;
  Status s = vdbgpu::ShardGroup::Open(*ctx->c, id, rank, nranks, timeout_ms, &sg);
  if (!s.ok()) return Fail(ctx, s);
  *out = new (std::nothrow) vdbgpu_shard_group{ctx, std::move(sg)};
  return *out != nullptr ? VDBGPU_OK : VDBGPU_RESOURCE_EXHAUSTED;
}

void vdbgpu_shard_group_close(vdbgpu_shard_group* g) {
  if (g == nullptr) return;
  {
    std::lock_guard<std::mutex> l(g->ctx->c->mu());
    cudaSetDevice(g->ctx->c->device());
    g->g.reset();
  }
  delete g;
}

int vdbgpu_shard_merge(vdbgpu_shard_group* g, const vdbgpu_hit* local, uint64_t nq, uint32_t k, int root,
                       uint64_t* out_ids, float* out_dist, vdbgpu_hit* out_hits) {
  if (g == nullptr || (nq > 0 && local == nullptr) || ((out_ids == nullptr) != (out_dist == nullptr)))
    return VDBGPU_INVALID_ARGUMENT;
  vdbgpu_ctx* ctx = g->ctx;
  if (k == 0 || k > 240) return Fail(ctx, Status(Status::kInvalidArgument, "k must be in 1..240"));
  std::lock_guard<std::mutex> l(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  Status s = RejectForeign(ctx->c->device(), {{local, "the local hit records"}, {out_ids, "the id output"},
                                              {out_dist, "the distance output"}, {out_hits, "the hit output"}});
  if (s.ok())
    s = g->g->Merge(reinterpret_cast<const vdbgpu::HitRecord*>(local), nq, k, root, out_ids, out_dist,
                    reinterpret_cast<vdbgpu::HitRecord*>(out_hits));
  return s.ok() ? VDBGPU_OK : Fail(ctx, s);
}

int vdbgpu_hnsw_build(vdbgpu_ctx* ctx, int metric, const float* rows, uint64_t nrows, uint32_t dim,
                      uint32_t padded_dim, uint32_t M, uint32_t candidates, uint64_t seed, void** out_file,
                      size_t* out_bytes) {
  if (ctx == nullptr || out_file == nullptr || out_bytes == nullptr || (nrows > 0 && rows == nullptr))
    return VDBGPU_INVALID_ARGUMENT;
  *out_file = nullptr;
  *out_bytes = 0;
  if (metric < 0 || metric > 2 || dim == 0 || dim > padded_dim || padded_dim % 16 != 0)
    return Fail(ctx, Status(Status::kInvalidArgument, "bad geometry or metric"));
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  std::string file;
  Status s = vdbgpu::BuildHnswFile(*ctx->c, metric, rows, nrows, dim, padded_dim, M, candidates, seed, &file);
  if (!s.ok()) return Fail(ctx, s);
  void* p = std::malloc(file.size());
  if (p == nullptr) return Fail(ctx, Status(Status::kResourceExhausted, "host allocation"));
  std::memcpy(p, file.data(), file.size());
  *out_file = p;
  *out_bytes = file.size();
  return VDBGPU_OK;
}

int vdbgpu_hnsw_extend(vdbgpu_ctx* ctx, int metric, const void* file_bytes, size_t nbytes, const float* rows,
                       uint64_t nrows, uint32_t dim, uint32_t padded_dim, void** out_file, size_t* out_bytes) {
  if (ctx == nullptr || file_bytes == nullptr || out_file == nullptr || out_bytes == nullptr ||
      (nrows > 0 && rows == nullptr))
    return VDBGPU_INVALID_ARGUMENT;
  *out_file = nullptr;
  *out_bytes = 0;
  if (metric < 0 || metric > 2 || dim == 0 || dim > padded_dim || padded_dim % 16 != 0)
    return Fail(ctx, Status(Status::kInvalidArgument, "bad geometry or metric"));
  std::string_view magic, body;
  Status s = vdbgpu::CheckIndexFile(std::string_view(static_cast<const char*>(file_bytes), nbytes), &magic, &body);
  if (!s.ok()) return Fail(ctx, s);
  if (magic != "VDBHNSW1") {
    const int t = vdbgpu::IndexTypeForMagic(magic);
    static const char* kNames[] = {"flat", "hnsw", "hnsw_sq8", "pq", "ivf_pq"};
    return Fail(ctx, Status(Status::kNotSupported, std::string("extend is not supported by ") +
                                                       (t >= 0 && t <= 4 ? kNames[t] : "this index file")));
  }
  // index.hnsw: padded dim, then the graph, whose capacity is its row count.
  vdbgpu::Reader peek(body);
  uint32_t fpd = 0;
  uint64_t cap = 0;
  if (!peek.u32(&fpd) || !peek.u64(&cap)) return Fail(ctx, Status(Status::kCorruption, "truncated hnsw header"));
  if (fpd != padded_dim) return Fail(ctx, Status(Status::kCorruption, "hnsw dim mismatch"));
  if (nrows < cap) return Fail(ctx, Status(Status::kInvalidArgument, "extend needs a superset of the indexed rows"));
  vdbgpu::Reader r(body);
  r.u32(&fpd);
  vdbgpu::HnswGraphData g;
  s = vdbgpu::ParseHnswGraph(r, cap, &g);
  if (!s.ok()) return Fail(ctx, s);
  if (g.size != g.cap) return Fail(ctx, Status(Status::kNotSupported, "extend needs a complete graph"));
  std::lock_guard<std::mutex> lk(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  s = RejectForeign(ctx->c->device(), {{rows, "the rows"}});
  std::string file;
  if (s.ok()) s = vdbgpu::ExtendHnswFile(*ctx->c, metric, g, padded_dim, rows, nrows, dim, &file);
  if (!s.ok()) return Fail(ctx, s);
  void* p = std::malloc(file.size());
  if (p == nullptr) return Fail(ctx, Status(Status::kResourceExhausted, "host allocation"));
  std::memcpy(p, file.data(), file.size());
  *out_file = p;
  *out_bytes = file.size();
  return VDBGPU_OK;
}

int vdbgpu_ivfpq_build(vdbgpu_ctx* ctx, int type, const float* rows, uint64_t nrows, uint32_t dim,
                       uint32_t padded_dim, uint32_t nlist, uint32_t pq_m, uint32_t max_train_ppc,
                       uint64_t seed, void** out_file, size_t* out_bytes) {
  if (ctx == nullptr || out_file == nullptr || out_bytes == nullptr || (nrows > 0 && rows == nullptr))
    return VDBGPU_INVALID_ARGUMENT;
  *out_file = nullptr;
  *out_bytes = 0;
  if (dim == 0 || dim > padded_dim || padded_dim % 16 != 0 || nrows > 0xFFFFFFFFull)
    return Fail(ctx, Status(Status::kInvalidArgument, "bad geometry"));
  std::lock_guard<std::mutex> g(ctx->c->mu());
  cudaSetDevice(ctx->c->device());
  std::string file;
  Status s = vdbgpu::BuildIvfPqFile(*ctx->c, type, rows, nrows, dim, padded_dim, nlist, pq_m, max_train_ppc,
                                    seed, &file);
  if (!s.ok()) return Fail(ctx, s);
  void* p = std::malloc(file.size());
  if (p == nullptr) return Fail(ctx, Status(Status::kResourceExhausted, "host allocation"));
  std::memcpy(p, file.data(), file.size());
  *out_file = p;
  *out_bytes = file.size();
  return VDBGPU_OK;
}

void vdbgpu_buffer_free(void* p) { std::free(p); }

int vdbgpu_collection_apply_log(vdbgpu_collection* c, const void* records, size_t bytes, uint64_t* applied) {
  if (c == nullptr || (records == nullptr && bytes > 0)) return VDBGPU_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(c->ctx->c->mu());
  cudaSetDevice(c->ctx->c->device());
  Status s = c->c->ApplyLog(*c->ctx->c, std::string_view(static_cast<const char*>(records), bytes), applied);
  if (!s.ok()) return Fail(c->ctx, s);
  return VDBGPU_OK;
}

int vdbgpu_collection_inspect(const char* path, char* out_json, size_t cap) {
  if (path == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::string text;
  Status s = vdbgpu::GpuCollection::Inspect(path, &text);
  int rc = VDBGPU_OK;
  if (!s.ok()) {
    rc = static_cast<int>(s.code());
    text = s.message();
  } else if (out_json != nullptr && text.size() + 1 > cap) {
    rc = VDBGPU_RESOURCE_EXHAUSTED;
  }
  if (out_json != nullptr && cap > 0) {
    const size_t n = std::min(cap - 1, text.size());
    std::memcpy(out_json, text.data(), n);
    out_json[n] = '\0';
  }
  return rc;
}

int vdbgpu_filter_describe(const char* schema_json, const char* filter_json, char* out, size_t cap) {
  if (schema_json == nullptr || filter_json == nullptr) return VDBGPU_INVALID_ARGUMENT;
  std::string text;
  int rc = VDBGPU_OK;
  vdbgpu::JsonValue sj;
  vdbgpu::Schema schema;
  Status s = vdbgpu::ParseJson(schema_json, &sj) ? vdbgpu::SchemaFromJson(sj, &schema)
                                                 : Status(Status::kInvalidArgument, "schema must be JSON");
  if (s.ok()) {
    std::unique_ptr<vdbgpu::FilterExpr> f;
    s = vdbgpu::FilterExpr::Parse(filter_json, schema, &f);
    if (s.ok()) text = f->ToString();
  }
  if (!s.ok()) {
    rc = static_cast<int>(s.code());
    text = s.message();
  }
  if (out != nullptr && cap > 0) {
    const size_t n = std::min(cap - 1, text.size());
    std::memcpy(out, text.data(), n);
    out[n] = '\0';
  }
  return rc;
}

}  // extern "C"
