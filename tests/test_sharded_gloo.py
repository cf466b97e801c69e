"""The host side of the sharded collection on the CPU, with two gloo ranks:
* the NCCL rendezvous token is made on rank 0 and reaches every rank (vdb_b200.sharded.share_token);
* each rank's merged records, laid out rank-major as vdbgpu_shard_merge exchanges them, merge into
  the merge of all segments at once (CollectionImpl::Search's order and dedupe, restated in
  oracle.merge_hits_py), whatever segments each rank owns (sharded.owner)."""
import datetime
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _candidates(nq, nparts, per_part, seed):
    """Per query and part: sorted (dist, part, row, id) lists; ids collide across parts and
    distances tie, so order and dedupe both matter."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(nq):
        parts = []
        for p in range(nparts):
            rows = rng.choice(1000, size=per_part, replace=False)
            d = np.round(rng.random(per_part) * 4) / 4  # many exact ties
            ids = rng.integers(0, 40, size=per_part)
            lst = sorted(zip(d.astype(np.float32).tolist(), [p] * per_part, rows.tolist(), ids.tolist()),
                         key=lambda t: (t[0], t[2]))
            parts.append(lst)
        out.append(parts)
    return out


def _records(hits, k, dtype):
    a = np.zeros(k, dtype=dtype)
    a["dist"], a["part"], a["row"], a["id"] = np.inf, 0xFFFFFFFF, 0xFFFFFFFF, np.iinfo(np.uint64).max
    for i, (d, p, r, idv) in enumerate(hits):
        a[i] = (d, p, r, 0, idv)
    return a


def _worker(rank, world, port, nq, k, result_q):
    import torch
    import torch.distributed as dist
    import oracle
    import vdb_b200
    from vdb_b200 import sharded
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
      try:
        cands = _candidates(nq, 5, 8, seed=9)
        local = np.stack([
            _records(oracle.merge_hits_py([c for p, lst in enumerate(parts) if sharded.owner(p, world) == rank
                                           for c in lst], k), k, vdb_b200.HIT_DTYPE)
            for parts in cands])
        token = sharded.share_token(make=lambda: bytes(range(128)))
        assert token == bytes(range(128))
        # The rank-major exchange of vdbgpu_shard_merge (an all-gather), done here with gloo.
        t = torch.from_numpy(local.view(np.uint8).reshape(-1).copy())
        g = torch.empty(world * t.numel(), dtype=torch.uint8)
        dist.all_gather_into_tensor(g, t)
        result_q.put((rank, g.numpy().tobytes()))
      except Exception as e:  # report instead of leaving the parent waiting
        result_q.put((rank, "error: %r" % (e,)))
        raise
    finally:
        dist.destroy_process_group()


def test_gather_and_merge_two_ranks():
    import torch.multiprocessing as mp
    import oracle
    import vdb_b200
    world, nq, k = 2, 6, 7
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, nq, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for r, v in results.items():
        assert not isinstance(v, str), v
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # Every rank received the same (world, nq, k) records.
    assert results[0] == results[1]
    gathered = np.frombuffer(results[0], dtype=vdb_b200.HIT_DTYPE).reshape(world, nq, k)
    cands = _candidates(nq, 5, 8, seed=9)
    for qi in range(nq):
        want = oracle.merge_hits_py([c for lst in cands[qi] for c in lst], k)
        lists = [[tuple(x) for x in gathered[r, qi] if x["row"] != 0xFFFFFFFF] for r in range(world)]
        got = oracle.merge_hits_py([(d, p, r, i) for lst in lists for (d, p, r, _, i) in lst], k)
        assert [(float(a[0]), a[1], a[2], a[3]) for a in got] == [(float(a[0]), a[1], a[2], a[3]) for a in want]
