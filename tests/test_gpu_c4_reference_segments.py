"""Config 4 parity on full-size segments the reference wrote itself: two segments of 1,562,500
cosine rows with year / tags metadata, bulk-loaded by the reference's own Collection (BulkLoad
builds each segment's HNSW graph, M=16, ef_construction=200; src/engine/collection_impl.cc:926-1016).
The GPU opens that directory (the reference's vectors.f32, meta.bin and index.hnsw) and searches it
with config 4's filters (year >= 2020 AND tags contains a Zipf-drawn tag) under the auto planner:
for a sample of queries over many filters, ids and distances equal the reference's SearchBatch on
the same directory, and per-segment explains (strategy, matches, distance computations, results)
equal its Search with explain (planner.cc:42-129)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

SEG_ROWS, SEGMENTS, EF, K = 1_562_500, 2, 64, 10
OPTIONS_INDEX = {"type": "hnsw", "M": 16, "ef_construction": 200}
SCHEMA = [{"name": "year", "type": "int64"}, {"name": "tags", "type": "keyword_list"}]


@pytest.fixture(scope="module")
def reference_dir(tmp_path_factory):
    import os
    from vdb_b200 import synth
    path = str(tmp_path_factory.mktemp("c4ref") / "c")
    rc = oracle.RefCollection(path, 128, metric="cosine", index=OPTIONS_INDEX, schema=SCHEMA,
                              threads=os.cpu_count())
    for s in range(SEGMENTS):
        rows, ids, years, tags = synth.c4_segment(s, SEG_ROWS)
        rc.bulk_load(ids, rows, years, tags)
    return path, rc


def test_full_size_reference_segments_search_like_the_reference(ctx, reference_dir):
    import vdb_b200
    from vdb_b200 import synth
    path, rc = reference_dir
    coll = vdb_b200.Collection.open(ctx, path)
    qs, filters, qf = synth.c4_queries(10_000)
    # Filters from the most to the least frequent tag, up to 24 queries each: both planner outcomes
    # (prefilter for rare tags, filtered graph walks for common ones).
    order = np.argsort(np.bincount(qf, minlength=len(filters)))[::-1]
    picked = list(order[:12]) + list(order[len(order) // 2:len(order) // 2 + 6]) + list(order[-6:])
    strategies = set()
    for f in picked:
        members = np.nonzero(qf == f)[0][:24]
        q = qs[members]
        ids, d = coll.search(q, k=K, ef=EF, filter=filters[f])
        rids, rd = rc.search(q, k=K, ef=EF, filter=filters[f])
        bad = np.nonzero(~np.all(ids == rids, axis=1))[0]
        assert bad.size == 0, (filters[f], bad[:5].tolist())
        np.testing.assert_array_equal(d, rd)
        got = coll.explain(q[0], k=K, ef=EF, filter=filters[f])
        want = rc.explain(q[0], k=K, ef=EF, filter=filters[f])
        assert len(got) == len(want)
        for a, b in zip(got, want):
            for key in ("strategy", "matches", "live_rows", "distance_computations", "results"):
                assert a[key] == b[key], (filters[f], key, a[key], b[key])
            strategies.add(a["strategy"])
    # Unfiltered search over the same graphs.
    ids, d = coll.search(qs[:200], k=K, ef=EF)
    rids, rd = rc.search(qs[:200], k=K, ef=EF)
    np.testing.assert_array_equal(ids, rids)
    np.testing.assert_array_equal(d, rd)
    assert len(strategies) >= 2, strategies
    coll.free()
