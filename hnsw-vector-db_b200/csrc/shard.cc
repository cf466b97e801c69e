// The exchange step of a collection sharded over the GPUs of one node (vdbgpu_shard_*).
//
// The reference searches every segment of a collection and merges the per-segment top-k lists
// (CollectionImpl::Search, src/engine/collection_impl.cc:1056-1108). With the disk segments spread
// over GPUs, each rank merges its own segments (GpuCollection::Search) into k hit records per
// query; this file moves those records between ranks with NCCL over NVLink / NVSwitch and runs the
// same merge over the ranks' lists on the receiving GPU:
//   * root < 0: ncclAllGather, every rank merges (all ranks hold the result);
//   * root >= 0: a gather (grouped ncclSend to the root, ncclRecv from every rank on the root),
//     only the root merges.
// The merged result equals the unsharded one: a hit among a query's first k distinct ids overall
// is among the first k distinct ids of the rank holding its segment.
//
// NCCL is opened with dlopen on first use (libnccl.so.2: the copy the process already holds, else
// the file VDBGPU_NCCL_LIB names, else the loader's), so the library has no link-time dependency
// on it and callers that never shard need no NCCL. The communicator is non-blocking: every wait (the
// rendezvous, each exchange) polls ncclCommGetAsyncError and the stream against a deadline, and a
// wait that runs out aborts the communicator and returns VDBGPU_UNAVAILABLE, so a rank that died
// or never joined ends the others' calls with an error instead of a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "collection.cuh"
#include "shard.h"

namespace vdbgpu {
namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char* (*GetErrorString)(ncclResult_t);
};

std::mutex g_nccl_mu;
NcclApi g_nccl;
bool g_nccl_loaded = false;
std::string g_nccl_error;

template <class F>
bool Sym(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

Status LoadNccl(const NcclApi** out) {
  std::lock_guard<std::mutex> g(g_nccl_mu);
  if (!g_nccl_loaded && g_nccl_error.empty()) {
    // One NCCL per process: a libnccl.so.2 the process already holds is reused (RTLD_NOLOAD);
    // else VDBGPU_NCCL_LIB names the file to load (the copy a framework loaded later in the same
    // process will also use: the first library loaded under a soname serves every later request
    // for it); else the loader's search path.
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (const char* path = std::getenv("VDBGPU_NCCL_LIB"); h == nullptr && path != nullptr && *path != '\0')
      h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) {
      const char* e = dlerror();
      g_nccl_error = std::string("NCCL (libnccl.so.2) could not be loaded: ") + (e != nullptr ? e : "");
    } else {
      NcclApi a{};
      const bool ok = Sym(h, "ncclGetUniqueId", &a.GetUniqueId) &&
                      Sym(h, "ncclCommInitRankConfig", &a.CommInitRankConfig) &&
                      Sym(h, "ncclCommGetAsyncError", &a.CommGetAsyncError) && Sym(h, "ncclCommAbort", &a.CommAbort) &&
                      Sym(h, "ncclCommFinalize", &a.CommFinalize) && Sym(h, "ncclCommDestroy", &a.CommDestroy) &&
                      Sym(h, "ncclAllGather", &a.AllGather) && Sym(h, "ncclSend", &a.Send) &&
                      Sym(h, "ncclRecv", &a.Recv) && Sym(h, "ncclGroupStart", &a.GroupStart) &&
                      Sym(h, "ncclGroupEnd", &a.GroupEnd) && Sym(h, "ncclGetErrorString", &a.GetErrorString);
      if (!ok) {
        g_nccl_error = "libnccl.so.2 lacks a symbol this library needs (NCCL 2.14 or later is required)";
      } else {
        g_nccl = a;
        g_nccl_loaded = true;
      }
    }
  }
  if (!g_nccl_loaded) return Status(Status::kUnavailable, g_nccl_error);
  *out = &g_nccl;
  return Status::OK();
}

using Clock = std::chrono::steady_clock;

}  // namespace

Status ShardUniqueId(void* out) {
  const NcclApi* nc = nullptr;
  VDBGPU_RETURN_IF_ERROR(LoadNccl(&nc));
  ncclUniqueId id;
  const ncclResult_t r = nc->GetUniqueId(&id);
  if (r != ncclSuccess) return Status(Status::kUnavailable, std::string("ncclGetUniqueId: ") + nc->GetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == kShardIdBytes, "ncclUniqueId size");
  std::memcpy(out, &id, sizeof(id));
  return Status::OK();
}

ShardGroup::~ShardGroup() {
  if (comm_ == nullptr) return;
  const NcclApi* nc = nullptr;
  if (!LoadNccl(&nc).ok()) return;
  auto comm = static_cast<ncclComm_t>(comm_);
  if (broken_) {
    nc->CommAbort(comm);
    return;
  }
  // Finalize flushes outstanding work; in non-blocking mode it may report progress, polled with a
  // bound like every other wait here.
  ncclResult_t r = nc->CommFinalize(comm);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms_);
  while (r == ncclInProgress && Clock::now() < deadline) {
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    nc->CommGetAsyncError(comm, &r);
  }
  if (r == ncclSuccess)
    nc->CommDestroy(comm);
  else
    nc->CommAbort(comm);
}

Status ShardGroup::Wait(const char* what, cudaStream_t st) {
  const NcclApi* nc = nullptr;
  VDBGPU_RETURN_IF_ERROR(LoadNccl(&nc));
  auto comm = static_cast<ncclComm_t>(comm_);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms_);
  for (;;) {
    ncclResult_t r = ncclSuccess;
    nc->CommGetAsyncError(comm, &r);
    if (r != ncclSuccess && r != ncclInProgress) {
      broken_ = true;
      nc->CommAbort(comm);
      comm_ = nullptr;
      return Status(Status::kUnavailable, std::string(what) + ": " + nc->GetErrorString(r));
    }
    bool done = r == ncclSuccess;
    if (done && st != nullptr) {
      const cudaError_t e = cudaStreamQuery(st);
      if (e != cudaSuccess && e != cudaErrorNotReady) return CudaStatus(e, what);
      done = e == cudaSuccess;
    }
    if (done) return Status::OK();
    if (Clock::now() >= deadline) {
      broken_ = true;
      nc->CommAbort(comm);
      comm_ = nullptr;
      return Status(Status::kUnavailable,
                    std::string(what) + ": no progress within " + std::to_string(timeout_ms_) +
                        " ms (a rank died, never joined or called with other arguments); the group was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

Status ShardGroup::Open(Context& ctx, const void* id, int rank, int nranks, int timeout_ms,
                        std::unique_ptr<ShardGroup>* out) {
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return Status(Status::kInvalidArgument, "rank must be in 0..nranks-1");
  const NcclApi* nc = nullptr;
  VDBGPU_RETURN_IF_ERROR(LoadNccl(&nc));
  std::unique_ptr<ShardGroup> g(new ShardGroup());
  g->ctx_ = &ctx;
  g->rank_ = rank;
  g->nranks_ = nranks;
  g->timeout_ms_ = timeout_ms > 0 ? timeout_ms : 60000;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  const ncclResult_t r = nc->CommInitRankConfig(&comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress)
    return Status(Status::kUnavailable, std::string("ncclCommInitRankConfig: ") + nc->GetErrorString(r));
  g->comm_ = comm;
  VDBGPU_RETURN_IF_ERROR(g->Wait("NCCL rendezvous", nullptr));
  *out = std::move(g);
  return Status::OK();
}

Status ShardGroup::Merge(const HitRecord* local, uint64_t nq, uint32_t k, int root, uint64_t* out_ids,
                         float* out_dist, HitRecord* out_records) {
  if (broken_ || comm_ == nullptr)
    return Status(Status::kFailedPrecondition, "the shard group was aborted by an earlier failure; open a new one");
  if (root >= nranks_) return Status(Status::kInvalidArgument, "root must be below nranks (or negative)");
  const NcclApi* nc = nullptr;
  VDBGPU_RETURN_IF_ERROR(LoadNccl(&nc));
  Context& ctx = *ctx_;
  const cudaStream_t st = ctx.stream();
  auto comm = static_cast<ncclComm_t>(comm_);
  const size_t bytes = nq * k * sizeof(HitRecord);
  const bool receives = root < 0 || root == rank_;
  VDBGPU_RETURN_IF_ERROR(send_.ensure(std::max<size_t>(bytes, 16)));
  VDBGPU_RETURN_IF_ERROR(all_.ensure(std::max<size_t>(bytes * nranks_, 16)));
  // The local records go into the send buffer in stream order (host or device source).
  VDBGPU_CUDA(cudaMemcpyAsync(send_.get(), local, bytes, cudaMemcpyDefault, st));
  uint8_t* all = all_.as<uint8_t>();
  ncclResult_t r;
  if (root < 0) {
    r = nc->AllGather(send_.get(), all, bytes, ncclUint8, comm, st);
  } else {
    r = nc->GroupStart();
    if (r == ncclSuccess) {
      if (rank_ == root) {
        for (int p = 0; p < nranks_ && r == ncclSuccess; ++p)
          if (p != rank_) r = nc->Recv(all + p * bytes, bytes, ncclUint8, p, comm, st);
      } else {
        r = nc->Send(send_.get(), bytes, ncclUint8, root, comm, st);
      }
      const ncclResult_t e = nc->GroupEnd();
      if (r == ncclSuccess) r = e;
    }
    if (r == ncclSuccess && rank_ == root)
      VDBGPU_CUDA(cudaMemcpyAsync(all + rank_ * bytes, send_.get(), bytes, cudaMemcpyDeviceToDevice, st));
  }
  if (r != ncclSuccess && r != ncclInProgress) {
    broken_ = true;
    nc->CommAbort(comm);
    comm_ = nullptr;
    return Status(Status::kUnavailable, std::string("hit exchange: ") + nc->GetErrorString(r));
  }
  VDBGPU_RETURN_IF_ERROR(Wait("hit exchange", st));
  if (!receives) return Status::OK();

  MergeArgs ma{};
  ma.kind = 1;
  ma.nlists = nranks_;
  ma.k = static_cast<int>(k);
  ma.nq = nq;
  ma.records = reinterpret_cast<const HitRecord*>(all);
  const bool ids_dev = out_ids != nullptr && WherePointer(out_ids, ctx.device()) == MemWhere::kDevice &&
                       WherePointer(out_dist, ctx.device()) == MemWhere::kDevice;
  const bool rec_dev = out_records != nullptr && WherePointer(out_records, ctx.device()) == MemWhere::kDevice;
  if (out_ids != nullptr) {
    if (ids_dev) {
      ma.out_ids = out_ids;
      ma.out_dist = out_dist;
    } else {
      VDBGPU_RETURN_IF_ERROR(ids_.ensure(nq * k * 8));
      VDBGPU_RETURN_IF_ERROR(dist_.ensure(nq * k * 4));
      ma.out_ids = ids_.as<uint64_t>();
      ma.out_dist = dist_.as<float>();
    }
  }
  if (out_records != nullptr) {
    if (rec_dev) {
      ma.out_records = out_records;
    } else {
      VDBGPU_RETURN_IF_ERROR(recs_.ensure(nq * k * sizeof(HitRecord)));
      ma.out_records = recs_.as<HitRecord>();
    }
  }
  VDBGPU_CUDA(LaunchMerge(ma, st));
  if (out_ids != nullptr && !ids_dev) {
    VDBGPU_CUDA(cudaMemcpyAsync(out_ids, ma.out_ids, nq * k * 8, cudaMemcpyDeviceToHost, st));
    VDBGPU_CUDA(cudaMemcpyAsync(out_dist, ma.out_dist, nq * k * 4, cudaMemcpyDeviceToHost, st));
  }
  if (out_records != nullptr && !rec_dev)
    VDBGPU_CUDA(cudaMemcpyAsync(out_records, ma.out_records, nq * k * sizeof(HitRecord), cudaMemcpyDeviceToHost, st));
  return ctx.Sync("shard merge");
}

}  // namespace vdbgpu
