"""Persisted delete sets (deletes-<n>.roar, written by the reference's Collection::Flush; read by
Segment::Open, src/storage/segment_reader.cc:101-116) against the reference's own collection
(fixture tests/golden/coll_deletes.npz from tests/golden/make_collection_golden.py).

CPU: the fixture's delete files cover every serialized form the loader must read (both cookies,
runs with and without container offsets, array / run / bitmap containers over four 16-bit keys).
GPU: the collection opened from disk returns the reference's ids and distances with those rows
deleted, and damaged delete files are refused as corruption, as Segment::Open refuses them."""
import json
import os

import numpy as np
import pytest

from helpers import blob, crc32c, decode_portable_roaring, extract_collection, golden


def _manifest(g):
    key = [k for k in g if k.startswith("file:MANIFEST-")][0]
    return key, json.loads(g[key].tobytes()[24:])


def _deletes(g, seg):
    name = seg["deletes_file"]
    raw = g[f"file:segments/seg-{seg['id']:06d}/{name}"].tobytes()
    assert raw[:8] == b"VDBDEL01"
    assert int(np.frombuffer(raw, "<u4", 1, 12)[0]) == crc32c(raw[24:])
    return raw[24:]


def test_fixture_covers_every_serialized_form():
    g = golden("coll_deletes")
    _, m = _manifest(g)
    a, b, c, up = m["segments"]  # manifest order: the three bulk loads, then the flushed upserts
    va, kinds, cookie, count = decode_portable_roaring(_deletes(g, a))
    want = np.union1d(g["deleted_rows_a"], [a["rows"] - 1])  # plus the row the upsert superseded
    assert np.array_equal(va, want) and a["deleted"] == want.size
    assert (cookie, count, kinds) == (12347, 4, ["array", "run", "bitmap", "array"])
    vb, kinds, cookie, _ = decode_portable_roaring(_deletes(g, b))
    assert cookie == 12346 and set(kinds) == {"array"} and vb.size == b["deleted"] == 40
    vc, kinds, cookie, count = decode_portable_roaring(_deletes(g, c))
    assert (cookie, count, kinds) == (12347, 1, ["run"]) and np.array_equal(vc, np.arange(100, 1100))
    assert up["deletes_file"] == "" and up["rows"] == 2


@pytest.fixture(scope="module")
def opened(tmp_path_factory):
    import vdb_b200
    g = golden("coll_deletes")
    ctx = vdb_b200.Context(0)
    path = extract_collection(g, tmp_path_factory.mktemp("coll_deletes"))
    return ctx, g, path, vdb_b200.Collection.open(ctx, path)


@pytest.mark.gpu
@pytest.mark.parametrize("k", [10, 64])
def test_search_with_persisted_deletes_matches_reference(opened, k):
    _, g, _, c = opened
    ids, d = c.search(g["queries"], k=k)
    assert np.array_equal(ids, g[f"ids_{k}"])
    assert np.array_equal(d, g[f"dist_{k}"])
    _, m = _manifest(g)
    a = m["segments"][0]
    gone = set((10 + np.asarray(g["deleted_rows_a"])) * 5) | {(10 + a["rows"] - 1) * 5}
    assert not gone & set(ids.ravel().tolist())


def _rewrite(path, g, payload):
    """Replaces segment C's delete file with a blob holding payload (checksum recomputed)."""
    _, m = _manifest(g)
    seg = m["segments"][2]
    with open(os.path.join(path, "segments", f"seg-{seg['id']:06d}", seg["deletes_file"]), "wb") as f:
        f.write(blob(b"VDBDEL01", payload))


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["out_of_range", "bad_cookie", "truncated", "run_past_key"])
def test_damaged_delete_sets_are_corruption(opened, tmp_path, case):
    import vdb_b200
    ctx, g, _, _ = opened
    path = extract_collection(g, tmp_path)
    ok = np.array([12347], "<u4").tobytes() + b"\x01" + np.array([0, 999, 1, 100, 999], "<u2").tobytes()
    payload = {
        # one run of rows 2990..3009 in a 3000-row segment
        "out_of_range": np.array([12347], "<u4").tobytes() + b"\x01" +
                        np.array([0, 19, 1, 2990, 19], "<u2").tobytes(),
        "bad_cookie": np.array([12345, 0], "<u4").tobytes(),
        "truncated": ok[:-2],
        "run_past_key": np.array([12347], "<u4").tobytes() + b"\x01" +
                        np.array([0, 19, 1, 65530, 19], "<u2").tobytes(),
    }[case]
    _rewrite(path, g, payload)
    with pytest.raises(vdb_b200.VdbError) as e:
        vdb_b200.Collection.open(ctx, path)
    assert e.value.code == vdb_b200.CORRUPTION, str(e.value)
    assert ("out of range" in str(e.value)) == (case == "out_of_range"), str(e.value)
