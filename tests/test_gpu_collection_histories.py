"""Random write histories run by the reference's own Collection (bulk loads, upserts of new and
existing ids with metadata, removals, flushes; flat and HNSW; L2 and cosine), closed, then
searched after recovery: by the reference's Collection::Open + SearchBatch and by
vdb_b200.Collection.open on the GPU. Ids and distances must be identical, unfiltered and with a
metadata filter, for every strategy. Covers the corners a fixed fixture does not: one-row and
mostly deleted segments, a mutable segment alone or next to many small segments, upserts of ids
whose old rows sit in any segment. Needs the reference engine (oracle/_ref)."""
import os
import shutil

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FILTERS = [None, {"field": "year", "gte": 2010}, {"field": "year", "exists": False}]
STRATEGIES = ["auto", "prefilter", "graph", "postfilter"]


def _history(rng, path, dim):
    import oracle
    c = oracle.RefCollection(path, dim, metric=str(rng.choice(["l2", "cosine"])),
                             index={"type": str(rng.choice(["flat", "hnsw"])), "M": 8, "ef_construction": 32},
                             schema=[{"name": "year", "type": "int64"}], threads=1)
    live, next_id = [], 1
    for _ in range(int(rng.integers(3, 12))):
        op = rng.random()
        if op < 0.25:
            m = int(rng.integers(1, 300))
            ids = np.arange(next_id, next_id + m, dtype=np.uint64)
            next_id += m
            years = [{"year": int(rng.integers(1990, 2030))} if rng.random() < 0.7 else None for _ in range(m)]
            c.bulk_load(ids, rng.standard_normal((m, dim)).astype(np.float32), metadata=years)
            live += ids.tolist()
        elif op < 0.6:
            m = int(rng.integers(1, 60))
            if live and rng.random() < 0.5:
                ids = np.array([live[int(i)] for i in rng.integers(0, len(live), m)], np.uint64)
            else:
                ids = np.arange(next_id, next_id + m, dtype=np.uint64)
                next_id += m
            meta = [None if rng.random() < 0.3 else {"year": int(rng.integers(1990, 2030))} for _ in range(m)]
            c.upsert(ids, rng.standard_normal((m, dim)).astype(np.float32), meta)
            live = sorted(set(live) | set(ids.tolist()))
        elif op < 0.85:
            m = int(rng.integers(1, 40))
            ids = np.array([live[int(i)] for i in rng.integers(0, len(live), m)] if live else [1], np.uint64)
            c.remove(ids)
            live = sorted(set(live) - set(ids.tolist()))
        else:
            c.flush()
    c.close()


def test_random_histories_match_reference(tmp_path):
    import oracle
    import vdb_b200
    if not os.path.exists(oracle.REF_ENGINE_LIB):
        pytest.skip("the reference engine is not built here")
    ctx = vdb_b200.Context(0)
    bad = []
    for sc in range(16):
        rng = np.random.default_rng(7000 + sc)
        dim = 8
        path, copy = str(tmp_path / f"c{sc}"), str(tmp_path / f"r{sc}")
        _history(rng, path, dim)
        shutil.copytree(path, copy)  # the reference's recovery writes into the directory
        q = rng.standard_normal((12, dim)).astype(np.float32)
        ref = oracle.RefCollection.open(copy, threads=1)
        gpu = vdb_b200.Collection.open(ctx, path)
        for f in FILTERS:
            for strategy in STRATEGIES:
                wi, wd = ref.search(q, k=10, ef=32, strategy=strategy, filter=f)
                gi, gd = gpu.search(q, k=10, ef=32, strategy=strategy, filter=f)
                if not (np.array_equal(gi, wi) and np.array_equal(gd, wd)):
                    bad.append((sc, strategy, f))
        ref.close()
    assert not bad, bad[:6]
