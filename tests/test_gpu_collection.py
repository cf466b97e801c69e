"""The collection read path on the GPU against the reference's own Collection (fixtures written
by tests/golden/make_collection_golden.py): filter bitmaps bit-exact per segment, the planner's
strategy / matches / distance computations per segment, and merged ids and distances identical
for every strategy (auto with both planner outcomes, graph, post-filter, prefilter, no filter)."""
import json

import numpy as np
import pytest

from helpers import extract_collection, golden

pytestmark = pytest.mark.gpu

NAMES = ["coll_hnsw", "coll_ivfpq", "coll_flat"]


@pytest.fixture(scope="module")
def colls(tmp_path_factory):
    import vdb_b200
    ctx = vdb_b200.Context(0)
    out = {}
    for name in NAMES:
        g = golden(name)
        path = extract_collection(g, tmp_path_factory.mktemp(name))
        out[name] = (g, vdb_b200.Collection.open(ctx, path), path)
    return ctx, out


def _case(g, ci):
    strategy, thr, ef, nprobe, k, alpha = json.loads(str(g["cases"][ci]))
    return dict(strategy=strategy, prefilter_threshold=thr, ef=ef, nprobe=nprobe, k=k, post_filter_alpha=alpha)


@pytest.mark.parametrize("name", NAMES)
def test_filter_bitmaps_bit_exact(colls, name):
    _, cs = colls
    g, c, _ = cs[name]
    assert c.segments_local == len(g["segment_ids"])
    for fi, f in enumerate(g["filters"]):
        for si, (sid, n) in enumerate(zip(g["segment_ids"], g["sizes"])):
            words, m = c.filter_bitmap(str(f), int(sid), int(n))
            want = g[f"bitmap_{fi}_{si}"]
            assert np.array_equal(words, want), (name, str(f), si)
            assert m == int(np.unpackbits(want.view(np.uint8)).sum())


@pytest.mark.parametrize("name", NAMES)
def test_search_matches_reference(colls, name):
    _, cs = colls
    g, c, _ = cs[name]
    q = g["queries"]
    filters = [str(f) for f in g["filters"]] + [None]
    bad = []
    for ci in range(len(g["cases"])):
        kw = _case(g, ci)
        for fi, f in enumerate(filters):
            ids, d = c.search(q, filter=f, **kw)
            wi, wd = g[f"ids_{ci}_{fi}"], g[f"dist_{ci}_{fi}"]
            rows = np.where(~(np.all(ids == wi, axis=1) & np.all(d == wd, axis=1)))[0]
            if rows.size:
                r = int(rows[0])
                bad.append((ci, fi, rows.size, ids[r].tolist(), wi[r].tolist(), d[r].tolist(), wd[r].tolist()))
    assert not bad, (name, len(bad), bad[:4])


@pytest.mark.parametrize("name", NAMES)
def test_explain_matches_reference(colls, name):
    _, cs = colls
    g, c, _ = cs[name]
    filters = [str(f) for f in g["filters"]] + [None]
    bad = []
    for ci in range(len(g["cases"])):
        kw = _case(g, ci)
        for fi, f in enumerate(filters):
            got = c.explain(g["queries"][0], filter=f, **kw)
            want = json.loads(str(g[f"explain_{ci}_{fi}"]))
            # The fixtures record the disk segments; the reference also explains its (here empty)
            # mutable segment first, as a scan of nothing.
            assert got[0]["kind"] == "mutable" and got[0]["strategy"] == ("scan_filter" if f else "scan")
            assert got[0]["matches"] == got[0]["distance_computations"] == got[0]["results"] == 0
            got = [e for e in got if e["kind"] == "disk"]
            assert len(got) == len(want)
            for a, b in zip(got, want):
                for key in ("id", "strategy", "matches", "live_rows", "distance_computations", "results"):
                    if a[key] != b[key]:
                        bad.append((ci, fi, key, a[key], b[key]))
    assert not bad, (name, len(bad), bad[:12])


@pytest.mark.parametrize("name", NAMES)
def test_grouped_batch_equals_separate_calls(colls, name):
    """One batch with a filter per query gives each query the result of its own SearchBatch."""
    _, cs = colls
    g, c, _ = cs[name]
    q = g["queries"]
    nf = len(g["filters"])
    rng = np.random.default_rng(3)
    qf = rng.integers(-1, nf, size=q.shape[0]).astype(np.int32)
    for ci in (0, 1, 3):
        kw = _case(g, ci)
        ids, d = c.search_grouped(q, [str(f) for f in g["filters"]], qf, **kw)
        for i in range(q.shape[0]):
            fi = nf if qf[i] < 0 else int(qf[i])
            assert np.array_equal(ids[i], g[f"ids_{ci}_{fi}"][i])
            assert np.array_equal(d[i], g[f"dist_{ci}_{fi}"][i])


def test_shards_merge_to_the_whole(colls):
    """Each shard of the segments searched alone, then vdbgpu_merge_hits over the shards' hit
    records, gives the unsharded result (the cross-GPU merge, here on one GPU)."""
    import vdb_b200
    ctx, cs = colls
    g, c, path = cs["coll_hnsw"]
    q = g["queries"]
    nf = len(g["filters"])
    qf = np.random.default_rng(7).integers(-1, nf, size=q.shape[0]).astype(np.int32)
    for world in (2, 3):
        shards = [vdb_b200.Collection.open(ctx, path, shard=r, nshards=world) for r in range(world)]
        for ci in (0, 1, 3):
            kw = _case(g, ci)
            k = kw["k"]
            for fi, f in enumerate([str(x) for x in g["filters"]] + [None]):
                lists = np.empty((world, q.shape[0], k), dtype=vdb_b200.HIT_DTYPE)
                for r, s in enumerate(shards):
                    s.search_grouped(q, [f] if f is not None else [], None, hits=lists[r], **kw)
                ids, d = vdb_b200.merge_hits(ctx, lists, k)
                assert np.array_equal(ids, g[f"ids_{ci}_{fi}"]), (world, ci, f)
                assert np.array_equal(d, g[f"dist_{ci}_{fi}"]), (world, ci, f)
            # Several filters in one batch (queries grouped, so the hit records must come back in
            # the caller's query order).
            lists = np.empty((world, q.shape[0], k), dtype=vdb_b200.HIT_DTYPE)
            for r, s in enumerate(shards):
                s.search_grouped(q, [str(x) for x in g["filters"]], qf, hits=lists[r], **kw)
            ids, d = vdb_b200.merge_hits(ctx, lists, k)
            for i in range(q.shape[0]):
                fi = nf if qf[i] < 0 else int(qf[i])
                assert np.array_equal(ids[i], g[f"ids_{ci}_{fi}"][i]), (world, ci, i)
                assert np.array_equal(d[i], g[f"dist_{ci}_{fi}"][i]), (world, ci, i)


def test_ivfpq_deep_rerank_is_refused(colls):
    """IVF-PQ re-ranks max(10 k, 100) candidates; the GPU path keeps at most 256, so a post-filter
    search of k * 10 = 100 (depth 1000) is refused rather than answered differently."""
    import vdb_b200
    _, cs = colls
    g, c, _ = cs["coll_ivfpq"]
    with pytest.raises(vdb_b200.VdbError) as e:
        c.search(g["queries"][:2], k=10, strategy="postfilter", post_filter_alpha=10, filter=str(g["filters"][0]))
    assert e.value.code == vdb_b200.NOT_SUPPORTED


def test_errors_match_reference(colls):
    _, cs = colls
    g, c, _ = cs["coll_hnsw"]
    q = np.array(g["queries"][:2])
    with pytest.raises(ValueError, match="k must be in 1..10000"):
        c.search(q, k=0)
    with pytest.raises(ValueError, match="unknown filter field nope"):
        c.search(q, filter='{"field": "nope", "eq": 1}')
    bad = q.copy()
    bad[1, 3] = np.nan
    with pytest.raises(ValueError, match="query has a NaN or infinite value"):
        c.search(bad)
    with pytest.raises(ValueError, match="a zero query cannot be normalized for cosine"):
        c.search(np.zeros_like(q))
