"""One collection's disk segments sharded over the GPUs of a node, one process per GPU.

The reference searches every segment of a collection and merges the per-segment top-k lists
(CollectionImpl::Search, src/engine/collection_impl.cc:1056-1108). Segments are independent, so
rank r holds the segments whose manifest position i has i % world == r (rank 0 also holds the
mutable segment rebuilt from the log), searches them with its own GPU and merges them locally
(ordered by (dist, part, row), one hit per external id). The only exchange is the library's
vdbgpu_shard_merge: every rank's k merged hit records per query (24 bytes each) cross NVLink in one
NCCL collective, and the receiving GPU(s) run the same merge over the world lists. The result
equals the unsharded merge: a hit among a query's global first k distinct ids is among the first k
distinct ids of its own rank.

torch.distributed serves only to hand the NCCL rendezvous token from rank 0 to the other ranks
(any backend, gloo included); the exchange itself is the C ABI's.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import vdb_b200

HIT_BYTES = vdb_b200.HIT_DTYPE.itemsize


def owner(ordinal: int, world: int) -> int:
    """The rank that holds the segment at manifest position `ordinal`."""
    return ordinal % world


def share_token(group=None, make: Optional[Callable[[], bytes]] = None) -> bytes:
    """The shard group's rendezvous token, made on rank 0 (vdb_b200.shard_id, or `make`) and
    broadcast to every rank of the torch.distributed group."""
    import torch.distributed as dist
    rank = dist.get_rank(group)
    box = [(make or vdb_b200.shard_id)() if rank == 0 else None]
    src = 0 if group is None else dist.get_global_rank(group, 0)
    dist.broadcast_object_list(box, src=src, group=group)
    token = box[0]
    if not isinstance(token, (bytes, bytearray)) or len(token) != vdb_b200.SHARD_ID_BYTES:
        raise RuntimeError("bad shard token received from rank 0")
    return bytes(token)


class ShardedCollection:
    """This rank's shard of a collection directory written by the reference, searched on this
    rank's GPU, with results merged across ranks over NCCL."""

    def __init__(self, path: str, rank: int, world: int, device: Optional[int] = None, group=None,
                 ctx: Optional[vdb_b200.Context] = None, local: Optional[vdb_b200.Collection] = None,
                 timeout_ms: int = 60000):
        import torch
        self.rank, self.world = rank, world
        self.device = torch.cuda.current_device() if device is None else device
        self.ctx = ctx if ctx is not None else vdb_b200.Context(self.device)
        self.local = local if local is not None else vdb_b200.Collection.open(self.ctx, path, shard=rank,
                                                                               nshards=world)
        self.shards = vdb_b200.ShardGroup(self.ctx, share_token(group), rank, world, timeout_ms)

    def search(self, queries, filters: Sequence = (), query_filter=None, k: int = 10, on_all_ranks: bool = False,
               **params):
        """Collection::SearchBatch over all ranks' segments: (ids uint64[nq,k], dists
        float32[nq,k]) as CUDA tensors on rank 0 (every rank when on_all_ranks), None elsewhere.
        `queries` (nq, dim) float32, host or CUDA; filters / query_filter as
        Collection.search_grouped. Every rank must call it with the same queries and filters."""
        import torch
        nq = int(queries.shape[0])
        dev = torch.device("cuda", self.device)
        hits = torch.empty(nq * k * HIT_BYTES, dtype=torch.uint8, device=dev)
        self.local.search_grouped(queries, list(filters), query_filter, k=k, out=False, hits=hits, **params)
        root = -1 if on_all_ranks else 0
        receives = on_all_ranks or self.rank == 0
        ids = torch.empty((nq, k), dtype=torch.int64, device=dev) if receives else None
        dists = torch.empty((nq, k), dtype=torch.float32, device=dev) if receives else None
        self.shards.merge(hits, nq, k, root=root, out=(ids, dists) if receives else None)
        if not receives:
            return None
        return ids.view(torch.uint64) if hasattr(torch, "uint64") else ids, dists

    def apply_log(self, records: bytes) -> int:
        """Applies write-ahead log records on this rank (Collection.apply_log): every rank keeps the
        id map, deletes rows of its own segments, and rank 0 rebuilds the mutable segment. Every
        rank must be given the same records, between searches."""
        return self.local.apply_log(records)

    def close(self):
        self.shards.close()
