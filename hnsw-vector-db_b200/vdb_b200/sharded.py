"""One collection's disk segments sharded over the GPUs of a node, one process per GPU.

The reference searches every segment of a collection and merges the per-segment top-k lists
(CollectionImpl::Search, src/engine/collection_impl.cc:1056-1108). Segments are independent, so
rank r holds the segments whose manifest position i has i % world == r (rank 0 also holds the
mutable segment rebuilt from the log), searches them with its own GPU and merges them locally (ordered by (dist, part, row), one hit per external id). The
only exchange is one all-gather of every rank's k merged hit records per query (24 bytes each)
over NCCL, after which each rank (or rank 0 alone) runs the same merge over the world lists on
its GPU. The result equals the unsharded merge: a hit among a query's global first k distinct
ids is among the first k distinct ids of its own rank.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

import vdb_b200

HIT_BYTES = vdb_b200.HIT_DTYPE.itemsize


def owner(ordinal: int, world: int) -> int:
    """The rank that holds the segment at manifest position `ordinal`."""
    return ordinal % world


def gather_hits(local, group=None):
    """All-gathers each rank's merged hit records (a flat uint8 tensor of nq * k * 24 bytes) into
    a (world, nq * k * 24) tensor on the same device (NCCL for CUDA tensors, gloo on the CPU)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = local.contiguous().view(-1)
    out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    if out.is_cuda:
        # The collective is ordered on torch's stream only; the library launches on its own
        # stream, so the gathered records must be complete before this returns.
        torch.cuda.current_stream(out.device).synchronize()
    return out.view(world, flat.numel())


class ShardedCollection:
    """This rank's shard of a collection directory written by the reference, searched on this
    rank's GPU, with results merged across ranks."""

    def __init__(self, path: str, rank: int, world: int, device: Optional[int] = None, group=None,
                 ctx: Optional[vdb_b200.Context] = None, local: Optional[vdb_b200.Collection] = None):
        import torch
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.cuda.current_device() if device is None else device
        self.ctx = ctx if ctx is not None else vdb_b200.Context(self.device)
        self.local = local if local is not None else vdb_b200.Collection.open(self.ctx, path, shard=rank,
                                                                               nshards=world)

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
        gathered = gather_hits(hits, self.group)
        if not on_all_ranks and self.rank != 0:
            return None
        ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
        dists = torch.empty((nq, k), dtype=torch.float32, device=dev)
        vdb_b200.merge_hits(self.ctx, gathered.view(self.world, nq, k * HIT_BYTES), k, out=(ids, dists))
        return ids.view(torch.uint64) if hasattr(torch, "uint64") else ids, dists

    def apply_log(self, records: bytes) -> int:
        """Applies write-ahead log records on this rank (Collection.apply_log): every rank keeps the
        id map, deletes rows of its own segments, and rank 0 rebuilds the mutable segment. Every
        rank must be given the same records, between searches."""
        return self.local.apply_log(records)
