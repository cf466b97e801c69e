"""The exchange step of a sharded collection through the C ABI (vdbgpu_shard_*): NCCL moves every
rank's merged hit records and the receiving GPU merges them; the result is the unsharded
collection's, which equals the reference's own search of the collection it wrote (fixture
coll_hnsw, made by tests/golden/make_collection_golden.py).

* one GPU: a one-rank group (the all-gather and the gather are copies) over each shard in turn;
* two GPUs (when the box has them): two processes, one shard each, merged over NVLink;
* a rank that never joins: the rendezvous runs out its bound and returns Unavailable. Nothing is
  launched on a GPU before the rendezvous completes, so this failure stays on the host."""
import datetime
import json
import os
import socket

import numpy as np
import pytest

from helpers import extract_collection, golden

pytestmark = pytest.mark.gpu


def _case(g, ci):
    strategy, thr, ef, nprobe, k, alpha = json.loads(str(g["cases"][ci]))
    return dict(strategy=strategy, prefilter_threshold=thr, ef=ef, nprobe=nprobe, k=k, post_filter_alpha=alpha)


def test_one_rank_group_merges_like_merge_hits(tmp_path):
    import vdb_b200
    g = golden("coll_hnsw")
    path = extract_collection(g, tmp_path)
    ctx = vdb_b200.Context(0)
    group = vdb_b200.ShardGroup(ctx, vdb_b200.shard_id(), 0, 1, timeout_ms=20000)
    coll = vdb_b200.Collection.open(ctx, path)
    q = g["queries"]
    nf = len(g["filters"])
    for ci in (0, 3):
        kw = _case(g, ci)
        k = kw["k"]
        for fi in list(range(min(nf, 4))) + [nf]:
            f = str(g["filters"][fi]) if fi < nf else None
            hits = np.empty((q.shape[0], k), dtype=vdb_b200.HIT_DTYPE)
            coll.search_grouped(q, [f] if f is not None else [], None, hits=hits, **kw)
            for root in (-1, 0):
                ids, d = group.merge(hits, q.shape[0], k, root=root)
                np.testing.assert_array_equal(ids, g[f"ids_{ci}_{fi}"])
                np.testing.assert_array_equal(d, g[f"dist_{ci}_{fi}"])
    group.close()
    coll.free()
    ctx.close()


def test_rank_that_never_joins_times_out():
    """Rank 0 of a two-rank group whose rank 1 never calls: the rendezvous gives up after the
    group's bound with Unavailable (no kernel or collective is ever launched)."""
    import time
    import vdb_b200
    ctx = vdb_b200.Context(0)
    t0 = time.time()
    with pytest.raises(vdb_b200.VdbError) as e:
        vdb_b200.ShardGroup(ctx, vdb_b200.shard_id(), 0, 2, timeout_ms=3000)
    assert e.value.code == vdb_b200.UNAVAILABLE
    assert time.time() - t0 < 60
    ctx.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_gpu_worker(rank, world, port, path, out_q):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from vdb_b200 import sharded
        g = golden("coll_hnsw")
        sc = sharded.ShardedCollection(path, rank, world, device=rank, timeout_ms=30000)
        q = g["queries"]
        res = []
        for ci in (0, 1, 3):
            kw = _case(g, ci)
            for f in [str(x) for x in g["filters"]] + [None]:
                r = sc.search(q, [f] if f is not None else [], None, on_all_ranks=True, **kw)
                res.append((r[0].cpu().numpy().view(np.uint64).tobytes(), r[1].cpu().numpy().tobytes()))
        sc.close()
        out_q.put((rank, res))
    except Exception as e:  # report instead of leaving the parent waiting
        out_q.put((rank, "error: %r" % (e,)))
    finally:
        dist.destroy_process_group()


def test_two_gpus_merge_to_the_reference(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    g = golden("coll_hnsw")
    path = extract_collection(g, tmp_path)
    port = _free_port()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_two_gpu_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r, v in results.items():
        assert not isinstance(v, str), v
    nf = len(g["filters"])
    i = 0
    for ci in (0, 1, 3):
        for fi in range(nf + 1):
            for r in range(2):
                ids = np.frombuffer(results[r][i][0], np.uint64).reshape(g[f"ids_{ci}_{fi}"].shape)
                d = np.frombuffer(results[r][i][1], np.float32).reshape(ids.shape)
                np.testing.assert_array_equal(ids, g[f"ids_{ci}_{fi}"])
                np.testing.assert_array_equal(d, g[f"dist_{ci}_{fi}"])
            i += 1
