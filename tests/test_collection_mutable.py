"""Collections with an unflushed log (fixture tests/golden/coll_mutable.npz, written by the
reference's own Collection: bulk loads, upserts, removes and a flush, closed without a final
Flush). Opening replays the log into the mutable segment as Collection::Open does
(CollectionImpl::Recover step 5 and ApplyOp, src/engine/collection_impl.cc:160-235, 574-599):
new ids, upserts of disk ids (their old rows deleted), an id upserted twice, removals, and records
older than the segment that now holds their id. Searches return the reference's ids and
distances for every strategy and filter; explains list the mutable part as the reference does;
two shards merge to the whole; damaged logs are handled as ParseWal handles them."""
import json
import os

import numpy as np
import pytest

from helpers import crc32c, extract_collection, golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mut(tmp_path_factory):
    import vdb_b200
    g = golden("coll_mutable")
    ctx = vdb_b200.Context(0)
    path = extract_collection(g, tmp_path_factory.mktemp("coll_mutable"))
    return ctx, g, path, vdb_b200.Collection.open(ctx, path)


def _case(g, ci):
    strategy, thr, ef, nprobe, k, alpha = json.loads(str(g["cases"][ci]))
    return dict(strategy=strategy, prefilter_threshold=thr, ef=ef, nprobe=nprobe, k=k, post_filter_alpha=alpha)


def test_search_matches_reference(mut):
    _, g, _, c = mut
    filters = [str(f) for f in g["filters"]] + [None]
    bad = []
    for ci in range(len(g["cases"])):
        for fi, f in enumerate(filters):
            ids, d = c.search(g["queries"], filter=f, **_case(g, ci))
            if not (np.array_equal(ids, g[f"ids_{ci}_{fi}"]) and np.array_equal(d, g[f"dist_{ci}_{fi}"])):
                bad.append((ci, fi))
    assert not bad, bad


def test_explain_lists_the_mutable_part(mut):
    _, g, _, c = mut
    filters = [str(f) for f in g["filters"]] + [None]
    bad = []
    for ci in range(len(g["cases"])):
        for fi, f in enumerate(filters):
            got = c.explain(g["queries"][0], filter=f, **_case(g, ci))
            want = json.loads(str(g[f"explain_{ci}_{fi}"]))
            assert [p["kind"] for p in got] == [p["kind"] for p in want] == ["mutable", "disk", "disk", "disk"]
            for a, b in zip(got, want):
                for key in ("id", "strategy", "matches", "live_rows", "distance_computations", "results"):
                    if a[key] != b[key]:
                        bad.append((ci, fi, a["kind"], key, a[key], b[key]))
    assert not bad, bad[:12]


def test_two_shards_merge_to_the_whole(mut):
    import vdb_b200
    ctx, g, path, _ = mut
    shards = [vdb_b200.Collection.open(ctx, path, shard=r, nshards=2) for r in range(2)]
    assert [s.segments_local for s in shards] == [3, 1]  # the mutable segment lives on shard 0
    q = g["queries"]
    for ci in (0, 3):
        kw = _case(g, ci)
        for fi, f in enumerate([str(x) for x in g["filters"]] + [None]):
            lists = np.empty((2, q.shape[0], kw["k"]), dtype=vdb_b200.HIT_DTYPE)
            for r, s in enumerate(shards):
                s.search_grouped(q, [f] if f is not None else [], None, hits=lists[r], **kw)
            ids, d = vdb_b200.merge_hits(ctx, lists, kw["k"])
            assert np.array_equal(ids, g[f"ids_{ci}_{fi}"]) and np.array_equal(d, g[f"dist_{ci}_{fi}"]), (ci, fi)


def _records(log: bytes):
    """(offset, length, lsn) of every record of a log file (src/storage/wal.cc framing)."""
    out, pos = [], 16
    while pos < len(log):
        plen = int(np.frombuffer(log, "<u4", 1, pos + 4)[0])
        out.append((pos, 17 + plen, int(np.frombuffer(log, "<u8", 1, pos + 9)[0])))
        pos += 17 + plen
    return out


def _log_path(path):
    d = os.path.join(path, "wal")
    (name,) = os.listdir(d)
    return os.path.join(d, name)


def _mutable_live(c, g):
    ex = c.explain(g["queries"][0])
    return [p for p in ex if p["kind"] == "mutable"][0]["live_rows"]


@pytest.mark.parametrize("case", ["torn_tail", "corrupt_middle", "lsn_gap", "bad_header"])
def test_damaged_logs(mut, tmp_path, case):
    import vdb_b200
    ctx, g, _, c = mut
    path = extract_collection(g, tmp_path)
    lp = _log_path(path)
    log = open(lp, "rb").read()
    recs = _records(log)
    assert crc32c(log[recs[0][0] + 4:recs[0][0] + recs[0][1]]) == int(np.frombuffer(log, "<u4", 1, recs[0][0])[0])
    last_off, last_len, _ = recs[-1]
    mid_off, mid_len, mid_lsn = recs[len(recs) // 2]
    if case == "torn_tail":
        # A write cut short by a crash: the last record is ignored (the final upsert of the
        # fixture, a new id, so the mutable part has one live row less).
        data = log[:last_off + last_len - 3]
    elif case == "corrupt_middle":
        b = bytearray(log)
        b[mid_off + 20] ^= 0xFF
        data = bytes(b)
    elif case == "lsn_gap":
        data = log[:mid_off] + log[mid_off + mid_len:]
    else:
        data = b"VDBWAL02" + log[8:]
    open(lp, "wb").write(data)
    if case == "torn_tail":
        c2 = vdb_b200.Collection.open(ctx, path)
        assert _mutable_live(c2, g) == _mutable_live(c, g) - 1
        return
    with pytest.raises(vdb_b200.VdbError) as e:
        vdb_b200.Collection.open(ctx, path)
    assert e.value.code == vdb_b200.CORRUPTION, str(e.value)
    want = {"corrupt_middle": "followed by valid records", "bad_header": "bad log file header",
            "lsn_gap": f"log sequence gap: expected LSN {mid_lsn}, found {mid_lsn + 1}"}[case]
    assert want in str(e.value), str(e.value)


def _search_all(c, g):
    bad = []
    for ci in range(len(g["cases"])):
        for fi, f in enumerate([str(x) for x in g["filters"]] + [None]):
            ids, d = c.search(g["queries"], filter=f, **_case(g, ci))
            if not (np.array_equal(ids, g[f"ids_{ci}_{fi}"]) and np.array_equal(d, g[f"dist_{ci}_{fi}"])):
                bad.append((ci, fi))
    return bad


@pytest.mark.parametrize("keep", ["header_only", "through_last_segment"])
def test_apply_log_reaches_the_recovered_state(mut, tmp_path, keep):
    """A directory whose log is cut short, opened, then fed the missing records with apply_log
    (as a live engine would after each log append) answers as the reference's recovery of the
    whole log. The batch overlaps what the cut log held; those records are skipped."""
    import vdb_b200
    ctx, g, _, _ = mut
    path = extract_collection(g, tmp_path)
    lp = _log_path(path)
    log = open(lp, "rb").read()
    recs = _records(log)
    manifest = json.loads(g[[k for k in g if k.startswith("file:MANIFEST-")][0]].tobytes()[24:])
    last_seg_lsn = max(s["lsn"] for s in manifest["segments"])
    cut = 0 if keep == "header_only" else next(i for i, r in enumerate(recs) if r[2] > last_seg_lsn)
    open(lp, "wb").write(log[:recs[cut][0]])
    start = max(0, cut - 10)
    shards = [vdb_b200.Collection.open(ctx, path, shard=r, nshards=2) for r in range(2)]
    c = vdb_b200.Collection.open(ctx, path)
    for x in [c] + shards:
        assert x.apply_log(log[recs[start][0]:]) == len(recs) - cut
    assert not _search_all(c, g)
    for ci in range(len(g["cases"])):
        got = c.explain(g["queries"][0], **_case(g, ci))
        want = json.loads(str(g[f"explain_{ci}_{len(g['filters'])}"]))
        keys = ("id", "kind", "strategy", "matches", "live_rows", "distance_computations", "results")
        assert [[p[k] for k in keys] for p in got] == [[p[k] for k in keys] for p in want], ci
    kw = _case(g, 0)
    lists = np.empty((2, g["queries"].shape[0], kw["k"]), dtype=vdb_b200.HIT_DTYPE)
    for r, s in enumerate(shards):
        s.search_grouped(g["queries"], [], None, hits=lists[r], **kw)
    ids, d = vdb_b200.merge_hits(ctx, lists, kw["k"])
    assert np.array_equal(ids, g[f"ids_0_{len(g['filters'])}"]) and np.array_equal(d, g[f"dist_0_{len(g['filters'])}"])
    # Everything again: all skipped. A record two LSNs ahead: a gap.
    assert c.apply_log(log[16:]) == 0
    off, ln, lsn = recs[-1]
    rec = bytearray(log[off:off + ln])
    rec[9:17] = np.array([lsn + 2], "<u8").tobytes()
    rec[0:4] = np.array([crc32c(bytes(rec[4:]))], "<u4").tobytes()
    with pytest.raises(vdb_b200.VdbError) as e:
        c.apply_log(bytes(rec))
    assert e.value.code == vdb_b200.CORRUPTION and f"expected LSN {lsn + 1}, found {lsn + 2}" in str(e.value)
    assert not _search_all(c, g)
