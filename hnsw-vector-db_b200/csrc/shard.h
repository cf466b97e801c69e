// The exchange step of a collection sharded over the GPUs of one node (shard.cc).
#pragma once

#include <memory>

#include "collection.cuh"
#include "runtime.h"

namespace vdbgpu {

constexpr size_t kShardIdBytes = 128;  // sizeof(ncclUniqueId)

// A new rendezvous token (ncclGetUniqueId), made on one rank and handed to every rank.
Status ShardUniqueId(void* out);

// One rank's membership in an NCCL communicator over `nranks` GPUs, bound to a context (its device
// and stream). Not thread-safe: callers serialise use through the context's mutex.
class ShardGroup {
 public:
  static Status Open(Context& ctx, const void* id, int rank, int nranks, int timeout_ms,
                     std::unique_ptr<ShardGroup>* out);
  ~ShardGroup();

  // Every rank's nq x k merged hit records (local: host or device) are exchanged; root < 0: all
  // ranks receive and merge; else only `root` does. Outputs (host or device, nullable) as
  // vdbgpu_merge_hits. Every rank must call with the same nq, k and root.
  Status Merge(const HitRecord* local, uint64_t nq, uint32_t k, int root, uint64_t* out_ids, float* out_dist,
               HitRecord* out_records);

  int rank() const { return rank_; }
  int nranks() const { return nranks_; }
  Context& context() const { return *ctx_; }

 private:
  ShardGroup() = default;
  Status Wait(const char* what, cudaStream_t st);
  Context* ctx_ = nullptr;
  void* comm_ = nullptr;  // ncclComm_t
  int rank_ = 0, nranks_ = 1, timeout_ms_ = 60000;
  bool broken_ = false;
  DeviceBuffer send_, all_, ids_, dist_, recs_;
};

}  // namespace vdbgpu
